// (b) Audio-tower conv stem helpers: conv1 as a direct convolution and the
// im2col gather that turns conv2/conv3 into tcgen05 GEMMs.
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

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

// One CTA per (chunk, output row oh).  The three input rows are staged in
// shared memory; thread j owns output channels 2j and 2j+1, keeps their 18
// weights and 2 biases in registers and walks the row's output positions, so
// each input tap is a shared-memory broadcast and each store is a coalesced
// 2 x 16-bit word.
template <typename T>
__global__ void __launch_bounds__(256) conv1_kernel(const float* __restrict__ mel, int h, int w,
                                                    const float* __restrict__ wt,
                                                    const float* __restrict__ bias, int c_out,
                                                    T* __restrict__ out) {
  extern __shared__ float s_in[];  // [3][w]
  const int ho = (h + 2 - 3) / 2 + 1, wo = (w + 2 - 3) / 2 + 1;
  const int chunk = blockIdx.y, oh = blockIdx.x;
  const float* src = mel + static_cast<long long>(chunk) * h * w;
  for (int i = threadIdx.x; i < 3 * w; i += blockDim.x) {
    const int r = i / w, col = i % w;
    const int ih = 2 * oh + r - 1;
    s_in[i] = (ih >= 0 && ih < h) ? src[ih * w + col] : 0.0f;
  }
  __syncthreads();
  T* dst = out + (static_cast<long long>(chunk) * ho + oh) * wo * c_out;
  for (int pair = threadIdx.x; pair < c_out / 2; pair += blockDim.x) {
    const int oc = 2 * pair;
    float w0[9], w1[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      w0[k] = wt[oc * 9 + k];
      w1[k] = wt[(oc + 1) * 9 + k];
    }
    const float b0 = bias[oc], b1 = bias[oc + 1];
    for (int ow = 0; ow < wo; ++ow) {
      float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
      for (int kh = 0; kh < 3; ++kh)
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) {
          const int iw = 2 * ow + kw - 1;
          const float v = (iw >= 0 && iw < w) ? s_in[kh * w + iw] : 0.0f;
          a0 = fmaf(w0[kh * 3 + kw], v, a0);
          a1 = fmaf(w1[kh * 3 + kw], v, a1);
        }
      T pr[2] = {f2h<T>(gelu_erf(a0 + b0)), f2h<T>(gelu_erf(a1 + b1))};
      *reinterpret_cast<uint32_t*>(dst + static_cast<long long>(ow) * c_out + oc) =
          *reinterpret_cast<const uint32_t*>(pr);
    }
  }
}

// One thread per 16-byte vector of the output row.
__global__ void im2col_kernel(const uint4* __restrict__ x, int n, int h, int w, int cv,
                              uint4* __restrict__ cols, bool time_major) {
  const int ho = (h + 2 - 3) / 2 + 1, wo = (w + 2 - 3) / 2 + 1;
  const long long total = static_cast<long long>(n) * ho * wo * 9 * cv;
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= total) return;
  const int v = static_cast<int>(i % cv);
  const int seg = static_cast<int>((i / cv) % 9);
  const long long row = i / (9LL * cv);
  const int p = static_cast<int>(row % (ho * wo));
  const int chunk = static_cast<int>(row / (ho * wo));
  int oh, ow;
  if (time_major) {
    ow = p / ho;
    oh = p % ho;
  } else {
    oh = p / wo;
    ow = p % wo;
  }
  const int ih = 2 * oh + seg / 3 - 1, iw = 2 * ow + seg % 3 - 1;
  uint4 val = make_uint4(0, 0, 0, 0);
  if (ih >= 0 && ih < h && iw >= 0 && iw < w)
    val = x[((static_cast<long long>(chunk) * h + ih) * w + iw) * cv + v];
  cols[i] = val;
}

}  // namespace

int conv1_direct(const float* mel, int n, int h, int w, const float* wt, const float* bias,
                 int c_out, void* out, bool bf16, cudaStream_t s) {
  if (n <= 0) return 0;
  if (c_out % 2 || 3 * w * sizeof(float) > 48 * 1024) return (int)cudaErrorInvalidValue;
  const int ho = (h + 2 - 3) / 2 + 1;
  const size_t smem = 3 * w * sizeof(float);
  dim3 grid(ho, n);
  if (bf16)
    conv1_kernel<__nv_bfloat16><<<grid, 256, smem, s>>>(mel, h, w, wt, bias, c_out,
                                                        static_cast<__nv_bfloat16*>(out));
  else
    conv1_kernel<__half><<<grid, 256, smem, s>>>(mel, h, w, wt, bias, c_out,
                                                 static_cast<__half*>(out));
  return (int)cudaGetLastError();
}

int im2col_3x3s2(const void* x, int n, int h, int w, int c, void* cols, bool time_major,
                 cudaStream_t s) {
  if (n <= 0) return 0;
  if (c % 8) return (int)cudaErrorInvalidValue;
  const int ho = (h + 2 - 3) / 2 + 1, wo = (w + 2 - 3) / 2 + 1;
  const long long total = static_cast<long long>(n) * ho * wo * 9 * (c / 8);
  im2col_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
      static_cast<const uint4*>(x), n, h, w, c / 8, static_cast<uint4*>(cols), time_major);
  return (int)cudaGetLastError();
}

}  // namespace qa
