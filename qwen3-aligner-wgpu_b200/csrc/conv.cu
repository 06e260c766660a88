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

// One CTA per (chunk, output row oh): stage the three input rows and the
// weights in shared memory, write [wo][c_out] contiguously.
template <typename T>
__global__ void __launch_bounds__(256) conv1_kernel(const float* __restrict__ mel, int h, int w,
                                                    const float* __restrict__ wt,
                                                    const float* __restrict__ bias, int c_out,
                                                    T* __restrict__ out) {
  extern __shared__ float sm[];
  const int ho = (h + 2 - 3) / 2 + 1, wo = (w + 2 - 3) / 2 + 1;
  const int chunk = blockIdx.y, oh = blockIdx.x;
  float* s_in = sm;              // [3][w]
  float* s_w = sm + 3 * w;       // [c_out][9]
  float* s_b = s_w + c_out * 9;  // [c_out]
  const float* src = mel + static_cast<long long>(chunk) * h * w;
  for (int i = threadIdx.x; i < 3 * w; i += blockDim.x) {
    const int r = i / w, col = i % w;
    const int ih = 2 * oh + r - 1;
    s_in[i] = (ih >= 0 && ih < h) ? src[ih * w + col] : 0.0f;
  }
  for (int i = threadIdx.x; i < c_out * 9; i += blockDim.x) s_w[i] = wt[i];
  for (int i = threadIdx.x; i < c_out; i += blockDim.x) s_b[i] = bias[i];
  __syncthreads();
  T* dst = out + (static_cast<long long>(chunk) * ho + oh) * wo * c_out;
  for (int i = threadIdx.x; i < wo * c_out; i += blockDim.x) {
    const int oc = i % c_out, ow = i / c_out;
    float acc = 0.0f;
#pragma unroll
    for (int kh = 0; kh < 3; ++kh)
#pragma unroll
      for (int kw = 0; kw < 3; ++kw) {
        const int iw = 2 * ow + kw - 1;
        const float v = (iw >= 0 && iw < w) ? s_in[kh * w + iw] : 0.0f;
        acc = fmaf(s_w[oc * 9 + kh * 3 + kw], v, acc);
      }
    dst[i] = f2h<T>(gelu_erf(acc + s_b[oc]));
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
  const int ho = (h + 2 - 3) / 2 + 1;
  const size_t smem = (3 * w + c_out * 10) * sizeof(float);
  dim3 grid(ho, n);
  if (bf16) {
    cudaFuncSetAttribute(conv1_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    conv1_kernel<__nv_bfloat16><<<grid, 256, smem, s>>>(mel, h, w, wt, bias, c_out,
                                                        static_cast<__nv_bfloat16*>(out));
  } else {
    cudaFuncSetAttribute(conv1_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    conv1_kernel<__half><<<grid, 256, smem, s>>>(mel, h, w, wt, bias, c_out,
                                                 static_cast<__half*>(out));
  }
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
