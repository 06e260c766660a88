// (b) Audio-tower conv stem: conv1 (conv2/conv3 are implicit GEMMs on the
// tensor cores, gemm_tc.cu).  conv1 runs on the tensor cores with split f16
// operands (conv1_tc_kernel); channel counts that do not split into two
// 16-multiple halves take the direct CUDA-core kernel (conv1_kernel).
//
// Reference: CpuConvStem::conv_block_stages (src/audio_encoder.rs:361-447),
// three conv2d(3x3, stride 2, pad 1) + bias + erf-GELU levels over
// [chunk, c, mel, frame].  Activations here are NHWC (channels innermost), so
// one im2col row is nine contiguous channel vectors; the weights of conv2 and
// conv3 are permuted at load to the matching k = (kh*3 + kw)*c_in + ic order.
#include <algorithm>

#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace qa {

namespace {

// One CTA per (chunk, pair of output rows oh0, oh0 + 1).  The five input rows
// 2*oh0 - 1 .. 2*oh0 + 3 are staged in shared memory with a zero column on
// each side (the padding), so the taps need no bounds checks.  Thread j of a
// row owns output channels 4j .. 4j+3: their 36 weights and 4 biases stay in
// registers, each tap read from shared memory (a broadcast) feeds four FMAs,
// and each output position is one 8-byte store, contiguous across the row's
// threads.
constexpr int kC1Ch = 4;  // output channels per thread

template <typename T>
__global__ void __launch_bounds__(256) conv1_kernel(const float* __restrict__ mel, int h, int w,
                                                    const float* __restrict__ wt,
                                                    const float* __restrict__ bias, int c_out,
                                                    int ldc, T* __restrict__ out) {
  extern __shared__ float s_in[];  // [5][w + 2]
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();

  const int ho = (h + 2 - 3) / 2 + 1, wo = (w + 2 - 3) / 2 + 1;
  const int wp = w + 2;
  const int chunk = blockIdx.y, oh0 = 2 * blockIdx.x;
  const float* src = mel + static_cast<long long>(chunk) * h * w;
  for (int i = threadIdx.x; i < 5 * wp; i += blockDim.x) {
    const int r = i / wp, col = i % wp - 1;
    const int ih = 2 * oh0 + r - 1;
    s_in[i] = (ih >= 0 && ih < h && col >= 0 && col < w) ? src[ih * w + col] : 0.0f;
  }
  __syncthreads();
  const int nq = c_out / kC1Ch;
  const int rr = threadIdx.x / nq, quad = threadIdx.x % nq;
  const int oh = oh0 + rr;
  if (rr >= 2 || oh >= ho) return;
  const int oc = quad * kC1Ch;
  // channel pairs (oc, oc+1) and (oc+2, oc+3) as f32x2 lanes: every packed
  // instruction rounds each lane exactly as the scalar one would
  float2 wk[kC1Ch / 2][9], b[kC1Ch / 2];
#pragma unroll
  for (int c = 0; c < kC1Ch / 2; ++c) {
#pragma unroll
    for (int k = 0; k < 9; ++k)
      wk[c][k] = make_float2(wt[(oc + 2 * c) * 9 + k], wt[(oc + 2 * c + 1) * 9 + k]);
    b[c] = make_float2(bias[oc + 2 * c], bias[oc + 2 * c + 1]);
  }
  const float2 kRsqrt2 = make_float2(0.70710678118654752f, 0.70710678118654752f);
  const float2 kHalf = make_float2(0.5f, 0.5f), kOne = make_float2(1.0f, 1.0f);
  const float* rows = s_in + 2 * rr * wp;  // input rows 2*oh - 1 .. 2*oh + 1 (padded)
  T* dst = out + (static_cast<long long>(chunk) * ho + oh) * wo * ldc + oc;
#pragma unroll 2
  for (int ow = 0; ow < wo; ++ow) {
    float2 a[kC1Ch / 2];
#pragma unroll
    for (int c = 0; c < kC1Ch / 2; ++c) a[c] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int kh = 0; kh < 3; ++kh)
#pragma unroll
      for (int kw = 0; kw < 3; ++kw) {
        const float v = rows[kh * wp + 2 * ow + kw];  // column 2*ow + kw - 1, shifted by the pad
        const float2 vv = make_float2(v, v);
#pragma unroll
        for (int c = 0; c < kC1Ch / 2; ++c) a[c] = fma2_rn(wk[c][kh * 3 + kw], vv, a[c]);
      }
    uint32_t pr[kC1Ch / 2];
#pragma unroll
    for (int c = 0; c < kC1Ch / 2; ++c) {
      // GELU on both lanes: taps, then bias; 0.5 * x * (1 + erf(x / sqrt 2)),
      // erf by A&S 7.1.26 (erf_as), as the reference's GPU tower computes it
      const float2 x = add2_rn(a[c], b[c]);
      const float2 z = mul2_rn(x, kRsqrt2);
      const float2 g = mul2_rn(mul2_rn(kHalf, x), add2_rn(kOne, erf_as2(z)));
      const T lo = f2h<T>(g.x), hi = f2h<T>(g.y);
      pr[c] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&lo)) |
              (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
    }
    *reinterpret_cast<uint2*>(dst + static_cast<long long>(ow) * ldc) = make_uint2(pr[0], pr[1]);
  }
}

// conv1 on the tensor cores.  As a GEMM, conv1 is M = output positions,
// N = c_out, K = 9 taps; each tap's product x * w is split so that 16-bit
// operands carry it at f32 grade: x = x_hi + x_lo and w = w_hi + w_lo (each
// part an f16), x * w ~= x_hi w_hi + x_lo w_hi + x_hi w_lo (the dropped x_lo
// w_lo is 2^-22 of the product), so K = 27 columns [x_hi, x_lo, x_hi] against
// [w_hi, w_hi, w_lo] per tap; columns 27 and 28 carry the bias (A = 1,
// B = [b_hi, b_lo]) and the rest is zero up to K = 32.  The products are
// exact in the f32 accumulator; only the summation order differs from the
// CUDA-core form's FMA chain and separate bias add.
//
// Persistent: CTA b takes the output channels of half b & 1 (N = c_out / 2)
// and the 128-position tiles b >> 1, + gridDim.x / 2, ...  Per tile:
//   threads 0-127 build the A tile in shared memory (one position each: nine
//     input values, split, 64 bytes written in the 64-byte-swizzled K-major
//     layout the MMA reads);
//   warp 0 issues the two K = 16 MMAs (M = 128, N = c_out / 2) into TMEM;
//   all 8 warps drain TMEM (warp w: lanes 32 (w & 3).., column half w >> 2),
//     apply erf_as GELU and store 16-bit values through a per-warp staging
//     buffer, four whole row segments per store instruction.
// B (this half's weights, split) is built once per CTA.  Two CTAs per SM (256
// TMEM columns each) overlap one's epilogue with the other's A build; the
// shared-memory request caps residency at two.
constexpr int kT1Rows = 128;
constexpr int kT1K = 32;
constexpr int kT1Threads = 256;
constexpr uint32_t kT1ABytes = kT1Rows * kT1K * 2;  // 8 KB
constexpr uint32_t kT1BMax = 256 * kT1K * 2;        // 16 KB: up to 256 channels
constexpr uint32_t kT1Stage = 4096;                 // per warp
constexpr size_t kT1SmemUsed = 1024 + kT1ABytes + kT1BMax + 8 * kT1Stage + 64;
constexpr size_t kT1Smem = 100 * 1024;  // > a third of the SM: two CTAs at most
static_assert(kT1SmemUsed <= kT1Smem, "conv1 shared memory");

// Byte offset of 16-byte unit u of row r in a K-major tile of 64-byte rows with
// 64-byte swizzling (the unit index XOR (row / 2) mod 4).
__device__ __forceinline__ uint32_t sw64_unit(int r, int u) {
  return static_cast<uint32_t>(r * 64 + 16 * (u ^ ((r >> 1) & 3)));
}

__device__ __forceinline__ uint32_t h2bits(__half x) { return __half_as_ushort(x); }

template <typename T>
__global__ void __launch_bounds__(kT1Threads, 2)
    conv1_tc_kernel(const float* __restrict__ mel, int n, int h, int w,
                    const float* __restrict__ wt, const float* __restrict__ bias, int c_out,
                    int ldc, T* __restrict__ out, unsigned* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + kT1ABytes;
  uint8_t* stage = sB + kT1BMax;
  uint64_t* done = reinterpret_cast<uint64_t*>(stage + 8 * kT1Stage);  // MMAs of a tile complete
  uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nh = c_out / 2;                 // this CTA's channels
  const int ch0 = (blockIdx.x & 1) * nh;    // its first channel
  const int cta = blockIdx.x >> 1, n_ctas = gridDim.x >> 1;
  const int ho = (h - 1) / 2 + 1, wo = (w - 1) / 2 + 1;
  const int hw = ho * wo;
  const int P = n * hw;  // the launcher keeps it below 2^31
  const int n_tiles = (P + kT1Rows - 1) / kT1Rows;
  if (tid == 0) {
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tslot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();

  // B: row c (channel ch0 + c), 27 split columns + zeros, swizzled
  for (int c = tid; c < nh; c += kT1Threads) {
    uint32_t k16[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) k16[i] = 0;
#pragma unroll
    for (int t = 0; t < 9; ++t) {
      const float wv = wt[(ch0 + c) * 9 + t];
      const __half hi = __float2half_rn(wv);
      const __half lo = __float2half_rn(wv - __half2float(hi));
      const uint32_t e[3] = {h2bits(hi), h2bits(hi), h2bits(lo)};
#pragma unroll
      for (int s = 0; s < 3; ++s) {
        const int k = 3 * t + s;
        k16[k >> 1] |= e[s] << (16 * (k & 1));
      }
    }
    {  // the bias in columns 27 (hi) and 28 (lo)
      const float bv = bias[ch0 + c];
      const __half hi = __float2half_rn(bv);
      const __half lo = __float2half_rn(bv - __half2float(hi));
      k16[13] |= h2bits(hi) << 16;
      k16[14] |= h2bits(lo);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      *reinterpret_cast<uint4*>(sB + sw64_unit(c, u)) =
          make_uint4(k16[4 * u], k16[4 * u + 1], k16[4 * u + 2], k16[4 * u + 3]);
  }

  const uint32_t idesc = f16_instr_desc(kT1Rows, nh, false);
  const int q = warp & 3, wg = warp >> 2;
  const int cb = wg == 0 ? 0 : 128, ce = wg == 0 ? min(128, nh) : nh;
  uint8_t* st = stage + warp * kT1Stage;
  uint32_t it = 0;
  for (int t = cta; t < n_tiles; t += n_ctas, ++it) {
    // A: thread m builds the row of position t * 128 + m
    if (tid < kT1Rows) {
      const int p = t * kT1Rows + tid;
      uint32_t k16[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) k16[i] = 0;
      if (p < P) {
        const int chunk = p / hw;
        const int rem = p - chunk * hw;
        const int oh = rem / wo, ow = rem - oh * wo;
        const float* src = mel + static_cast<long long>(chunk) * h * w;
        k16[13] = 0x3C00u << 16;  // columns 27, 28: 1.0 against the bias
        k16[14] = 0x3C00u;
#pragma unroll
        for (int kh = 0; kh < 3; ++kh)
#pragma unroll
          for (int kw = 0; kw < 3; ++kw) {
            const int ih = 2 * oh + kh - 1, iw = 2 * ow + kw - 1;
            const float x = (ih >= 0 && ih < h && iw >= 0 && iw < w) ? __ldg(src + ih * w + iw) : 0.0f;
            const __half hi = __float2half_rn(x);
            const __half lo = __float2half_rn(x - __half2float(hi));
            const uint32_t e[3] = {h2bits(hi), h2bits(lo), h2bits(hi)};
#pragma unroll
            for (int s = 0; s < 3; ++s) {
              const int k = 3 * (kh * 3 + kw) + s;
              k16[k >> 1] |= e[s] << (16 * (k & 1));
            }
          }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(sA + sw64_unit(tid, u)) =
            make_uint4(k16[4 * u], k16[4 * u + 1], k16[4 * u + 2], k16[4 * u + 3]);
    }
    fence_proxy_async_smem();  // A (and B) written by threads, read by the tensor core
    __syncthreads();
    if (warp == 0) {
      tc_fence_after();
      const uint32_t a = smem_u32(sA), b = smem_u32(sB);
#pragma unroll
      for (int ks = 0; ks < kT1K / 16; ++ks)
        mma_f16_e(tbase, sw64_kmajor_desc(a + ks * 32), sw64_kmajor_desc(b + ks * 32), idesc,
                  ks > 0 ? 1u : 0u);
      mma_commit_e(done);
    }
    if (!mbar_wait(done, it & 1)) *abort_flag = 1;
    __syncthreads();  // every thread's wait is over: one decision for the CTA
    if (*abort_flag) break;
    tc_fence_after();
    // epilogue: rows 32q.., columns [cb, ce) of this half
    const int p = t * kT1Rows + q * 32 + lane;
    T* base = p < P ? out + static_cast<long long>(p) * ldc + ch0 : nullptr;
    const uint32_t trow = tbase + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
    for (int c0 = cb; c0 < ce; c0 += 64) {
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        const int col = c0 + 32 * hh;
        if (col >= ce) break;  // warp-uniform
        float x[32];
        tmem_ld32(trow + col, x);  // columns past nh hold no product; never stored
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t u4[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int i = 8 * j + 2 * k;
            u4[k] = cvt2_rn<T>(gelu_as2(make_float2(x[i], x[i + 1])));
          }
          stage_unit(st, 4 * hh + j, make_uint4(u4[0], u4[1], u4[2], u4[3]));
        }
      }
      flush_rows<T>(st, base, c0, c0 + 32, min(64, ce - c0) / 8);
    }
    tc_fence_before();
    __syncthreads();  // TMEM and A free for the next tile
  }
  if (*abort_flag && tid == 0 && status) atomicOr(status, kStatusTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 256);
  }
}

}  // namespace

int conv1_direct(const float* mel, int n, int h, int w, const float* wt, const float* bias,
                 int c_out, int ldc, void* out, bool bf16, unsigned* status, cudaStream_t s) {
  if (n <= 0) return 0;
  // the tensor-core form: two halves of c_out, each a multiple of 16 and at
  // most 256 wide, whole 8-channel units; 16-byte aligned output rows
  if (c_out % 32 == 0 && c_out <= 512 && (c_out / 2) % 8 == 0 && ldc >= c_out && ldc % 8 == 0 &&
      (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
    const int ho = (h - 1) / 2 + 1, wo = (w - 1) / 2 + 1;
    const long long positions = static_cast<long long>(n) * ho * wo;
    if (positions >= (1ll << 31) - kT1Rows) return (int)cudaErrorInvalidValue;
    const long long tiles = (positions + kT1Rows - 1) / kT1Rows;
    const int grid = static_cast<int>(2 * std::min<long long>(tiles, device_sm_count()));
    if (bf16) {
      auto k = conv1_tc_kernel<__nv_bfloat16>;
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kT1Smem);
      if (e != cudaSuccess) return (int)e;
      return (int)launch_pdl(k, dim3(grid), dim3(kT1Threads), kT1Smem, s, mel, n, h, w, wt, bias, c_out,
                             ldc, static_cast<__nv_bfloat16*>(out), status);
    }
    auto k = conv1_tc_kernel<__half>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kT1Smem);
    if (e != cudaSuccess) return (int)e;
    return (int)launch_pdl(k, dim3(grid), dim3(kT1Threads), kT1Smem, s, mel, n, h, w, wt, bias, c_out,
                           ldc, static_cast<__half*>(out), status);
  }
  if (c_out % kC1Ch || 2 * (c_out / kC1Ch) > 256 || 5 * (w + 2) * sizeof(float) > 48 * 1024 ||
      ldc < c_out || ldc % kC1Ch)
    return (int)cudaErrorInvalidValue;
  const int ho = (h + 2 - 3) / 2 + 1;
  const size_t smem = 5 * (w + 2) * sizeof(float);
  dim3 grid((ho + 1) / 2, n);
  if (bf16)
    return (int)launch_pdl(conv1_kernel<__nv_bfloat16>, grid, dim3(256), smem, s, mel, h, w, wt,
                           bias, c_out, ldc, static_cast<__nv_bfloat16*>(out));
  return (int)launch_pdl(conv1_kernel<__half>, grid, dim3(256), smem, s, mel, h, w, wt, bias,
                         c_out, ldc, static_cast<__half*>(out));
}

}  // namespace qa
