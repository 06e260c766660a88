// (b) Audio-tower conv stem: conv1 as a direct convolution (conv2/conv3 are
// implicit GEMMs on the tensor cores, gemm_tc.cu).
//
// Reference: CpuConvStem::conv_block_stages (src/audio_encoder.rs:361-447),
// three conv2d(3x3, stride 2, pad 1) + bias + erf-GELU levels over
// [chunk, c, mel, frame].  Activations here are NHWC (channels innermost), so
// one im2col row is nine contiguous channel vectors; the weights of conv2 and
// conv3 are permuted at load to the matching k = (kh*3 + kw)*c_in + ic order.
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

}  // namespace

int conv1_direct(const float* mel, int n, int h, int w, const float* wt, const float* bias,
                 int c_out, int ldc, void* out, bool bf16, cudaStream_t s) {
  if (n <= 0) return 0;
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
