// extern "C" wrappers for the kernel-level entry points (include/qa_b200_kernels.h).
#include "qa_b200.h"
#include "qa_b200_kernels.h"

#include "gemm_tc.cuh"
#include "kernels.cuh"

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

extern "C" int qa_k_gemm_qkv_rope(const void* A, long long lda, const void* B, long long ldb,
                                  int M, int N, int K, int bf16, void* q_out, long long ldo,
                                  const int* pos_of, const int* clip_of, const int* block_tab,
                                  int max_pages, void* kc, void* vc, const void* cos_t,
                                  const void* sin_t, const float* qn, const float* kn, float eps,
                                  int nq, int nkv, unsigned* status, int force_bn, void* stream) {
  if (!A || !B || !q_out || !pos_of || !clip_of || !block_tab || !kc || !vc || !cos_t || !sin_t ||
      !qn || !kn || nq <= 0 || nkv <= 0 || N != (nq + 2 * nkv) * 128)
    return QA_ERR_ARG;
  EpiParams ep;
  ep.mode = EPI_QKV_ROPE;
  ep.out = q_out;
  ep.ldo = ldo;
  ep.status = status;
  ep.rk.pos_of = pos_of;
  ep.rk.clip_of = clip_of;
  ep.rk.block_tab = block_tab;
  ep.rk.max_pages = max_pages;
  ep.rk.page_size = 64;
  ep.rk.kc = kc;
  ep.rk.vc = vc;
  ep.rk.cos_t = cos_t;
  ep.rk.sin_t = sin_t;
  ep.rk.qn = qn;
  ep.rk.kn = kn;
  ep.rk.eps = eps;
  ep.rk.nq = nq;
  ep.rk.nkv = nkv;
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

extern "C" int qa_k_causal_attention(const void* qkv, long long ldq, long long q_rows, int nqh,
                                     int nkvh, const int* tiles, int n_tiles, const int* block_tab,
                                     int max_pages, const void* kpool, const void* vpool,
                                     int kv_pages, void* out, int bf16, unsigned* status,
                                     void* stream) {
  if (!qkv || !tiles || !block_tab || !kpool || !vpool || !out || n_tiles < 0 || kv_pages <= 0)
    return QA_ERR_ARG;
  PagedKV kv{const_cast<void*>(kpool), const_cast<void*>(vpool), 64};
  const AttnTile* t = reinterpret_cast<const AttnTile*>(tiles);
  const int rc = causal_attention_tc(qkv, ldq, q_rows, nqh, nkvh, 128, t, n_tiles, block_tab,
                                     max_pages, kv, kv_pages, out, bf16 != 0, status,
                                     static_cast<cudaStream_t>(stream));
  return rc == 0 ? QA_OK : QA_ERR_CUDA;
}

extern "C" int qa_k_window_attention(const void* qkv, long long T, int dm, int nh,
                                     const int* windows, int n_windows, int max_window, void* out,
                                     int bf16, unsigned* status, void* stream) {
  if (!qkv || !out || (n_windows > 0 && !windows) || n_windows < 0 || T <= 0 || nh <= 0 ||
      dm != 64 * nh || max_window <= 0 || max_window > 128)
    return QA_ERR_ARG;
  const int rc = window_attention(qkv, T, dm, nh, 64, reinterpret_cast<const int2*>(windows),
                                  n_windows, max_window, out, bf16 != 0, status,
                                  static_cast<cudaStream_t>(stream));
  return rc == 0 ? QA_OK : QA_ERR_CUDA;
}

extern "C" int qa_k_conv1(const float* mel, int n, int h, int w, const float* wt,
                          const float* bias, int c_out, void* out, int bf16, void* stream) {
  if (!mel || !wt || !bias || !out || n < 0 || h <= 0 || w <= 0) return QA_ERR_ARG;
  const int rc = conv1_direct(mel, n, h, w, wt, bias, c_out, c_out, out, bf16 != 0, nullptr,
                              static_cast<cudaStream_t>(stream));
  return rc == 0 ? QA_OK : QA_ERR_CUDA;
}
