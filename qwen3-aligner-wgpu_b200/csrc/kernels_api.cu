// extern "C" wrappers for the kernel-level entry points (include/qa_b200_kernels.h).
#include "qa_b200.h"
#include "qa_b200_kernels.h"

#include "gemm_tc.cuh"

using namespace qa;

extern "C" int qa_k_gemm(const void* A, long long lda, const void* B, long long ldb, int M, int N,
                         int K, int bf16, int mode, int act, void* out, long long ldo,
                         const float* bias, const int* row_map, const float* pe, int pe_period,
                         unsigned long long* keys, unsigned* status, int force_bn, void* stream) {
  EpiParams ep;
  ep.mode = mode;
  ep.act = act;
  ep.out = out;
  ep.ldo = ldo;
  ep.bias = bias;
  ep.row_map = row_map;
  ep.pe = pe;
  ep.pe_period = pe_period > 0 ? pe_period : 1;
  ep.keys = keys;
  ep.status = status;
  int rc = gemm_tc(A, lda, B, ldb, M, N, K, bf16 != 0, ep, static_cast<cudaStream_t>(stream),
                   force_bn);
  return rc == 0 ? QA_OK : QA_ERR_CUDA;
}

extern "C" int qa_k_conv3x3s2(const void* x, int n, int h, int w, int c, const void* wt, int c_out,
                              int time_major, int bf16, int mode, int act, void* out, long long ldo,
                              const float* bias, unsigned* status, void* stream) {
  EpiParams ep;
  ep.mode = mode;
  ep.act = act;
  ep.out = out;
  ep.ldo = ldo;
  ep.bias = bias;
  ep.status = status;
  int rc = conv3x3s2_tc(x, n, h, w, c, wt, c_out, time_major != 0, bf16 != 0, ep,
                        static_cast<cudaStream_t>(stream));
  return rc == 0 ? QA_OK : QA_ERR_CUDA;
}
