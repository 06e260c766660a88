// HBM-bound row kernels of the alignment path: the audio tower's LayerNorm,
// the decoder's RMSNorm, the embedding gather, and (f) the timestamp-row
// gather + final norm.  (d), the q/k RMSNorm + RoPE + paged K/V append, runs
// in the decoder QKV GEMM's epilogue (gemm_tc.cu, EPI_QKV_ROPE).
//
// One warp per row (or per (token, head)); 16-bit rows are read as 16-byte
// vectors.  Arithmetic follows the reference's CPU order where it decides a
// rounding: products and sums that the reference writes as separate f32
// operations use __fmul_rn/__fadd_rn so nvcc cannot contract them into FMAs.
#include "kernels.cuh"
#include "sm100.cuh"

namespace qa {

namespace {

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

// Two f32 values rounded to 16 bits, a in the low half.
template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float a, float b) {
  const T ha = f2h<T>(a), hb = f2h<T>(b);
  return static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&ha)) |
         (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&hb)) << 16);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// ---------------------------------------------------------------- LayerNorm
// CpuAudioLayerNorm::forward (src/audio_encoder.rs:170-191), eps 1e-5.
template <typename T>
__global__ void layernorm_kernel(const float* __restrict__ x, int rows, int d,
                                 const float* __restrict__ g, const float* __restrict__ b,
                                 float eps, T* __restrict__ out) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + static_cast<long long>(row) * d;
  float v[32];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const int i = lane + 32 * k;
    v[k] = i < d ? xr[i] : 0.f;
    s += v[k];
  }
  const float mean = warp_sum(s) / static_cast<float>(d);
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const int i = lane + 32 * k;
    if (i < d) {
      const float t = v[k] - mean;
      q = fmaf(t, t, q);
    }
  }
  const float var = warp_sum(q) / static_cast<float>(d);
  const float inv = 1.0f / sqrtf(var + eps);
  T* o = out + static_cast<long long>(row) * d;
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const int i = lane + 32 * k;
    if (i < d) o[i] = f2h<T>(__fadd_rn(__fmul_rn(__fmul_rn(v[k] - mean, inv), g[i]), b[i]));
  }
}

// The same row arithmetic with 16-byte loads: rows of d % 4 == 0 f32 elements,
// 16-byte aligned x / g / b, 8-byte aligned output rows.  Lane l holds float4
// vectors l, l + 32, ... of its row.  The block copies the gain and bias into
// shared memory while its rows' loads are in flight, so that the output loop
// after the two reductions does not wait on them.
template <typename T>
__global__ void layernorm_vec_kernel(const float* __restrict__ x, int rows, int d,
                                     const float* __restrict__ g, const float* __restrict__ b,
                                     float eps, T* __restrict__ out) {
  __shared__ float4 sg[256], sb[256];  // d <= 1024
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int nv = d / 4;
  const bool live = row < rows;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<long long>(live ? row : 0) * d);
  float4 v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int i = lane + 32 * k;
    v[k] = (live && i < nv) ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    sg[i] = __ldg(reinterpret_cast<const float4*>(g) + i);
    sb[i] = __ldg(reinterpret_cast<const float4*>(b) + i);
  }
  __syncthreads();
  if (!live) return;
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
  const float mean = warp_sum(s) / static_cast<float>(d);
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (lane + 32 * k < nv) {
      const float t0 = v[k].x - mean, t1 = v[k].y - mean, t2 = v[k].z - mean, t3 = v[k].w - mean;
      q = fmaf(t0, t0, q);
      q = fmaf(t1, t1, q);
      q = fmaf(t2, t2, q);
      q = fmaf(t3, t3, q);
    }
  }
  const float var = warp_sum(q) / static_cast<float>(d);
  const float inv = 1.0f / sqrtf(var + eps);
  uint2* o = reinterpret_cast<uint2*>(out + static_cast<long long>(row) * d);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int i = lane + 32 * k;
    if (i < nv) {
      const float4 gg = sg[i], bb = sb[i];
      const float e0 = __fadd_rn(__fmul_rn(__fmul_rn(v[k].x - mean, inv), gg.x), bb.x);
      const float e1 = __fadd_rn(__fmul_rn(__fmul_rn(v[k].y - mean, inv), gg.y), bb.y);
      const float e2 = __fadd_rn(__fmul_rn(__fmul_rn(v[k].z - mean, inv), gg.z), bb.z);
      const float e3 = __fadd_rn(__fmul_rn(__fmul_rn(v[k].w - mean, inv), gg.w), bb.w);
      o[i] = make_uint2(pack_pair<T>(e0, e1), pack_pair<T>(e2, e3));
    }
  }
}

// ---------------------------------------------------------------- RMSNorm
// rms_norm_row (src/cpu_decoder.rs:289-300): f16(x * inv * w), d % 256 == 0.
template <typename T>
__global__ void rmsnorm_kernel(const T* __restrict__ x, int rows, int d,
                               const float* __restrict__ w, float eps, T* __restrict__ out) {
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<long long>(row) * d);
  const int nv = d / 8;  // 16-byte vectors per row
  float v[32];
  float s2 = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int vi = lane + 32 * k;
    if (vi < nv) {
      uint4 u = xr[vi];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[k * 8 + j] = h2f<T>(e[j]);
        s2 = fmaf(v[k * 8 + j], v[k * 8 + j], s2);
      }
    }
  }
  const float inv = 1.0f / sqrtf(warp_sum(s2) / static_cast<float>(d) + eps);
  uint4* orow = reinterpret_cast<uint4*>(out + static_cast<long long>(row) * d);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int vi = lane + 32 * k;
    if (vi < nv) {
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(w) + 2 * vi);
      const float4 g1 = __ldg(reinterpret_cast<const float4*>(w) + 2 * vi + 1);
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      alignas(16) T e[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] = f2h<T>(__fmul_rn(__fmul_rn(v[k * 8 + j], inv), g[j]));
      orow[vi] = *reinterpret_cast<const uint4*>(e);
    }
  }
}

// ---------------------------------------------------------------- row sums of squares
// The decoder's first RMSNorm input (embedding rows + projected audio rows):
// out[r * (d / 128) + j] = sum of squares of the 128 16-bit values of block j
// of row r, in column order -- the form the residual GEMM epilogues write for
// the later norms (EpiParams::ssq_out).  One warp per row, one block per lane.
template <typename T>
__global__ void row_ssq_kernel(const T* __restrict__ x, int rows, int d, float* __restrict__ out) {
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nblk = d / 128;
  for (int j = lane; j < nblk; j += 32) {
    const uint4* p = reinterpret_cast<const uint4*>(x + static_cast<long long>(row) * d + j * 128);
    float s2 = 0.0f;
#pragma unroll 4
    for (int q = 0; q < 16; ++q) {
      const uint4 u = p[q];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float f = h2f<T>(e[k]);
        s2 = fmaf(f, f, s2);
      }
    }
    out[static_cast<long long>(row) * nblk + j] = s2;
  }
}

// ---------------------------------------------------------------- embedding gather
// src/align_inference.rs:690-715, on the device: one thread per 16 bytes.
__global__ void embed_gather_kernel(const uint32_t* __restrict__ ids, int T_,
                                    const uint4* __restrict__ table, int vocab, int dv,
                                    int audio_id, uint4* __restrict__ out, int* bad) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= static_cast<long long>(T_) * dv) return;
  const int t = static_cast<int>(i / dv);
  const int v = static_cast<int>(i % dv);
  const uint32_t id = ids[t];
  if (static_cast<int>(id) == audio_id) return;  // filled by the projector's scatter
  if (id >= static_cast<uint32_t>(vocab)) {
    if (v == 0) atomicOr(bad, kBadTokenId);
    return;
  }
  out[i] = table[static_cast<long long>(id) * dv + v];
}

// ---------------------------------------------------------------- (f) head rows
// src/align_inference.rs:766-783 (folded) and :748-765 (unfolded): one warp per row.
template <typename T>
__global__ void head_norm_kernel(const T* __restrict__ hidden, int n_hidden,
                                 const int* __restrict__ rows, int n_rows, int d,
                                 const float* __restrict__ w, float eps,
                                 __nv_bfloat16* __restrict__ a, float* __restrict__ unfolded,
                                 int* __restrict__ bad) {
  const int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= n_rows) return;
  const int row = rows[r];
  if (row < 0 || row >= n_hidden) {
    // never read outside the hidden rows: zero this row's outputs and flag it
    if (lane == 0) atomicOr(bad, kBadHeadRow);
    __nv_bfloat16* ar = a + static_cast<long long>(r) * 2 * d;
    for (int i = lane; i < 2 * d; i += 32) ar[i] = __float2bfloat16_rn(0.0f);
    if (unfolded)
      for (int i = lane; i < d; i += 32) unfolded[static_cast<long long>(r) * d + i] = 0.0f;
    return;
  }
  const T* x = hidden + static_cast<long long>(row) * d;
  float v[32];
  float acc = 0.f, a2 = 0.f;
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const int i = lane + 32 * k;
    v[k] = i < d ? to_f32(x[i]) : 0.f;
    const float xf = i < d ? __fmul_rn(v[k], w[i]) : 0.f;
    acc = fmaf(xf, xf, acc);
    a2 = fmaf(v[k], v[k], a2);
  }
  const float inv = 1.0f / sqrtf(warp_sum(acc) / static_cast<float>(d) + eps);
  const float inv2 = 1.0f / sqrtf(warp_sum(a2) / static_cast<float>(d) + eps);
  __nv_bfloat16* ar = a + static_cast<long long>(r) * 2 * d;
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const int i = lane + 32 * k;
    if (i < d) {
      const float nrm = __fmul_rn(__fmul_rn(v[k], w[i]), inv);
      const __nv_bfloat16 hi = __float2bfloat16_rn(nrm);
      ar[i] = hi;
      ar[d + i] = __float2bfloat16_rn(nrm - __bfloat162float(hi));
      if (unfolded) unfolded[static_cast<long long>(r) * d + i] = __fmul_rn(__fmul_rn(v[k], inv2), w[i]);
    }
  }
}

__global__ void argmax_finalize_kernel(const unsigned long long* __restrict__ keys, int n,
                                       double seg_ms, long long* __restrict__ raw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const unsigned long long k = keys[i];
  const long long idx = k == 0ull ? 0 : static_cast<long long>(0xFFFFFFFFull - (k & 0xFFFFFFFFull));
  raw[i] = static_cast<long long>(static_cast<double>(idx) * seg_ms);
}

template <typename T>
__global__ void widen_kernel(const T* __restrict__ x, long long n, float* __restrict__ out) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i < n) out[i] = h2f<T>(x[i]);
}

}  // namespace

int layernorm_rows(const float* x, int rows, int d, const float* g, const float* b, float eps,
                   void* out, bool bf16, cudaStream_t s) {
  if (rows <= 0) return 0;
  if (d > 1024) return (int)cudaErrorInvalidValue;
  const unsigned blocks = (rows + 7) / 8;
  const bool vec = d % 4 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(g) |
                                   reinterpret_cast<uintptr_t>(b)) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 7u) == 0;
  if (vec && bf16)
    return (int)launch_pdl(layernorm_vec_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s, x,
                           rows, d, g, b, eps, static_cast<__nv_bfloat16*>(out));
  if (vec)
    return (int)launch_pdl(layernorm_vec_kernel<__half>, dim3(blocks), dim3(256), 0, s, x, rows, d,
                           g, b, eps, static_cast<__half*>(out));
  if (bf16)
    layernorm_kernel<<<blocks, 256, 0, s>>>(x, rows, d, g, b, eps, static_cast<__nv_bfloat16*>(out));
  else
    layernorm_kernel<<<blocks, 256, 0, s>>>(x, rows, d, g, b, eps, static_cast<__half*>(out));
  return (int)cudaGetLastError();
}

int rmsnorm_rows(const void* x, int rows, int d, const float* w, float eps, void* out, bool bf16,
                 cudaStream_t s) {
  if (rows <= 0) return 0;
  if (d % 8 || d > 1024 || (reinterpret_cast<uintptr_t>(w) & 15u)) return (int)cudaErrorInvalidValue;
  const unsigned blocks = (rows + 7) / 8;
  if (bf16)
    return (int)launch_pdl(rmsnorm_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s,
                           static_cast<const __nv_bfloat16*>(x), rows, d, w, eps,
                           static_cast<__nv_bfloat16*>(out));
  return (int)launch_pdl(rmsnorm_kernel<__half>, dim3(blocks), dim3(256), 0, s,
                         static_cast<const __half*>(x), rows, d, w, eps, static_cast<__half*>(out));
}

int row_ssq(const void* x, int rows, int d, float* out, bool bf16, cudaStream_t s) {
  if (rows <= 0) return 0;
  if (d % 512) return (int)cudaErrorInvalidValue;
  const unsigned blocks = (rows + 7) / 8;
  if (bf16)
    return (int)launch_pdl(row_ssq_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s,
                           static_cast<const __nv_bfloat16*>(x), rows, d, out);
  return (int)launch_pdl(row_ssq_kernel<__half>, dim3(blocks), dim3(256), 0, s,
                         static_cast<const __half*>(x), rows, d, out);
}

int embed_gather(const uint32_t* ids, int T_, const void* table, int vocab, int d, int audio_id,
                 void* out, int* bad, cudaStream_t s) {
  if (T_ <= 0) return 0;
  if (d % 8) return (int)cudaErrorInvalidValue;
  const int dv = d / 8;
  const long long total = static_cast<long long>(T_) * dv;
  embed_gather_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
      ids, T_, static_cast<const uint4*>(table), vocab, dv, audio_id, static_cast<uint4*>(out), bad);
  return (int)cudaGetLastError();
}

int head_gather_norm(const void* hidden, int hidden_kind, int n_hidden, const int* rows,
                     int n_rows, int d, const float* w, float eps, void* a_hilo, float* unfolded,
                     int* bad, cudaStream_t s) {
  if (n_rows <= 0) return 0;
  if (d > 1024 || !bad) return (int)cudaErrorInvalidValue;
  const unsigned blocks = (n_rows + 7) / 8;
  auto* a = static_cast<__nv_bfloat16*>(a_hilo);
  if (hidden_kind == 1)
    head_norm_kernel<<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(hidden), n_hidden,
                                            rows, n_rows, d, w, eps, a, unfolded, bad);
  else if (hidden_kind == 2)
    head_norm_kernel<<<blocks, 256, 0, s>>>(static_cast<const float*>(hidden), n_hidden, rows,
                                            n_rows, d, w, eps, a, unfolded, bad);
  else
    head_norm_kernel<<<blocks, 256, 0, s>>>(static_cast<const __half*>(hidden), n_hidden, rows,
                                            n_rows, d, w, eps, a, unfolded, bad);
  return (int)cudaGetLastError();
}

int argmax_finalize(const unsigned long long* keys, int n, double segment_ms, long long* raw_ms,
                    cudaStream_t s) {
  if (n <= 0) return 0;
  argmax_finalize_kernel<<<(n + 255) / 256, 256, 0, s>>>(keys, n, segment_ms, raw_ms);
  return (int)cudaGetLastError();
}

int widen16(const void* x, long long n, float* out, bool bf16, cudaStream_t s) {
  if (n <= 0) return 0;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (bf16)
    widen_kernel<<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), n, out);
  else
    widen_kernel<<<blocks, 256, 0, s>>>(static_cast<const __half*>(x), n, out);
  return (int)cudaGetLastError();
}

}  // namespace qa
