#include "tma_host.h"

#include <mutex>

namespace qa {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_once;

void resolve() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}
}  // namespace

int make_tmap_2d(CUtensorMap* map, const void* base, bool bf16, long long inner, long long rows,
                 long long ld, int box_inner, int box_rows) {
  std::call_once(g_once, resolve);
  if (!g_encode) return (int)cudaErrorNotSupported;
  if (box_inner * 2 != 128 || box_rows <= 0 || box_rows > 256) return (int)cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || ((ld * 2) % 16)) return (int)cudaErrorInvalidValue;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

int make_tmap_nd(CUtensorMap* map, const void* base, bool bf16, int rank, const long long* dims,
                 const long long* stride_bytes, const int* box, const int* estr, int swizzle) {
  std::call_once(g_once, resolve);
  if (!g_encode) return (int)cudaErrorNotSupported;
  if (rank < 1 || rank > 5 || (swizzle != 64 && swizzle != 128)) return (int)cudaErrorInvalidValue;
  if (box[0] * 2 > swizzle || (box[0] * 2) % 16 || (reinterpret_cast<uintptr_t>(base) & 15u))
    return (int)cudaErrorInvalidValue;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    if (dims[i] <= 0 || box[i] <= 0 || box[i] > 256 || estr[i] <= 0 || estr[i] > 8)
      return (int)cudaErrorInvalidValue;
    d[i] = (cuuint64_t)dims[i];
    b[i] = (cuuint32_t)box[i];
    e[i] = (cuuint32_t)estr[i];
  }
  for (int i = 0; i + 1 < rank; ++i) {
    if (stride_bytes[i] % 16) return (int)cudaErrorInvalidValue;
    st[i] = (cuuint64_t)stride_bytes[i];
  }
  CUresult r = g_encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        rank, const_cast<void*>(base), d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

}  // namespace qa
