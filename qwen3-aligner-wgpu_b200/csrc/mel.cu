// (a) Log-mel spectrogram on the GPU, batched over clips.
//
// Same steps as src/mel.rs:198-242: reflect-pad 200, periodic Hann (400),
// 400-point DFT power (201 bins), 128-bin slaney filterbank applied in
// ascending-bin order, log10 with a 1e-10 floor, per-clip max, clamp at
// max - 8, (x + 4) / 4, trailing frame dropped (n_samples / 160 frames).
//
// Pass 1 computes 16 frames per CTA: the frames' samples (with reflection)
// are staged in shared memory once, each thread evaluates one DFT bin for 8
// frames at a time from a 400-entry twiddle table (the direct DFT is 32
// MFLOP per audio-second — well under a millisecond for a whole batch — and
// keeps every frame's arithmetic independent of the batch layout), then the
// sparse filterbank and the log run out of shared memory.  The per-clip
// maximum is an atomicMax on an order-preserving integer encoding.
#include "kernels.cuh"
#include "sm100.cuh"

namespace qa {

namespace {

constexpr int kNfft = 400;
constexpr int kBins = 201;
constexpr int kHop = 160;
constexpr int kPad = 200;
constexpr int kMels = 128;
constexpr int kFT = 16;                          // frames per CTA
constexpr int kSpan = (kFT - 1) * kHop + kNfft;  // samples staged per CTA

__device__ __forceinline__ long long reflect_index(long long i, long long n) {
  if (n <= 1) return 0;
  const long long period = 2 * (n - 1);
  long long x = i % period;
  if (x < 0) x += period;
  return x > n - 1 ? period - x : x;
}

__device__ __forceinline__ unsigned float_key(float v) {
  const unsigned u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(unsigned k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__global__ void __launch_bounds__(256) mel_logpower_kernel(
    const float* __restrict__ samples, const MelClip* __restrict__ clips,
    const float* __restrict__ window, const float2* __restrict__ twiddle, MelBank bank,
    float log10_factor, float* __restrict__ scratch, unsigned* __restrict__ maxkey) {
  __shared__ float s_x[kSpan];
  __shared__ float s_win[kNfft];
  __shared__ float2 s_tw[kNfft];
  __shared__ float s_pow[kFT][kBins + 1];
  __shared__ unsigned s_max;

  const MelClip c = clips[blockIdx.y];
  const int f0 = blockIdx.x * kFT;
  if (f0 >= c.n_frames) return;
  const int nf = min(kFT, c.n_frames - f0);
  const float* x = samples + c.sample_off;
  const long long n = c.n_samples;

  for (int i = threadIdx.x; i < kSpan; i += blockDim.x) {
    const long long pp = static_cast<long long>(f0) * kHop + i;  // index into the padded signal
    s_x[i] = x[reflect_index(pp - kPad, n)];
  }
  for (int i = threadIdx.x; i < kNfft; i += blockDim.x) {
    s_win[i] = window[i];
    s_tw[i] = twiddle[i];
  }
  if (threadIdx.x == 0) s_max = 0u;
  __syncthreads();

  // DFT power: item = (bin, group of 8 frames)
  for (int item = threadIdx.x; item < kBins * (kFT / 8); item += blockDim.x) {
    const int k = item % kBins;
    const int g = item / kBins;
    float re[8], im[8];
#pragma unroll
    for (int f = 0; f < 8; ++f) re[f] = im[f] = 0.f;
    int idx = 0;
    const float* xs = s_x + g * 8 * kHop;
    for (int j = 0; j < kNfft; ++j) {
      const float2 t = s_tw[idx];
      const float wj = s_win[j];
#pragma unroll
      for (int f = 0; f < 8; ++f) {
        const float v = xs[f * kHop + j] * wj;
        re[f] = fmaf(v, t.x, re[f]);
        im[f] = fmaf(-v, t.y, im[f]);
      }
      idx += k;
      if (idx >= kNfft) idx -= kNfft;
    }
#pragma unroll
    for (int f = 0; f < 8; ++f)
      s_pow[g * 8 + f][k] = __fadd_rn(__fmul_rn(re[f], re[f]), __fmul_rn(im[f], im[f]));
  }
  __syncthreads();

  // filterbank + log10, ascending bins (src/mel.rs:215-234)
  float local_max = -INFINITY;
  for (int item = threadIdx.x; item < kMels * kFT; item += blockDim.x) {
    const int m = item % kMels;
    const int f = item / kMels;
    if (f >= nf) continue;
    const int st = bank.start[m], ln = bank.len[m], wo = bank.woff[m];
    float acc = 0.f;
    for (int j = 0; j < ln; ++j) acc = __fadd_rn(acc, __fmul_rn(bank.w[wo + j], s_pow[f][st + j]));
    const float v = __fmul_rn(logf(fmaxf(acc, 1e-10f)), log10_factor);
    scratch[static_cast<long long>(c.frame_off + f0 + f) * kMels + m] = v;
    local_max = fmaxf(local_max, v);
  }
  atomicMax(&s_max, float_key(local_max));
  __syncthreads();
  if (threadIdx.x == 0) atomicMax(&maxkey[blockIdx.y], s_max);
}

__device__ __forceinline__ float finalize(float v, float mx) {
  return (fmaxf(v, mx - 8.0f) + 4.0f) / 4.0f;
}

__global__ void mel_finalize_chunked_kernel(const float* __restrict__ scratch,
                                            const MelClip* __restrict__ clips,
                                            const int* __restrict__ chunk_clip, int total_chunks,
                                            int cf, const unsigned* __restrict__ maxkey,
                                            float* __restrict__ out) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long total = static_cast<long long>(total_chunks) * kMels * cf;
  if (i >= total) return;
  const int j = static_cast<int>(i % cf);
  const int m = static_cast<int>((i / cf) % kMels);
  const int ch = static_cast<int>(i / (static_cast<long long>(cf) * kMels));
  const int ci = chunk_clip[ch];
  const MelClip c = clips[ci];
  const int frame = (ch - c.chunk_off) * cf + j;
  float v = 0.f;  // the processor pads with 0.0 (src/align_input.rs:24-26)
  if (frame < c.n_frames)
    v = finalize(scratch[static_cast<long long>(c.frame_off + frame) * kMels + m],
                 key_float(maxkey[ci]));
  out[i] = v;
}

__global__ void mel_finalize_rows_kernel(const float* __restrict__ scratch, int n_frames,
                                         const unsigned* __restrict__ maxkey,
                                         float* __restrict__ out) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= static_cast<long long>(n_frames) * kMels) return;
  const int t = static_cast<int>(i % n_frames);
  const int m = static_cast<int>(i / n_frames);
  out[i] = finalize(scratch[static_cast<long long>(t) * kMels + m], key_float(maxkey[0]));
}

}  // namespace

int mel_logpower(const float* samples, const MelClip* clips, int n_clips, int max_frames,
                 const float* window, const float2* twiddle, MelBank bank, float log10_factor,
                 float* scratch, unsigned* maxkey, cudaStream_t s) {
  if (n_clips <= 0 || max_frames <= 0) return 0;
  dim3 grid((max_frames + kFT - 1) / kFT, n_clips);
  mel_logpower_kernel<<<grid, 256, 0, s>>>(samples, clips, window, twiddle, bank, log10_factor,
                                           scratch, maxkey);
  return (int)cudaGetLastError();
}

int mel_finalize_chunked(const float* scratch, const MelClip* clips, const int* chunk_clip,
                         int total_chunks, int chunk_frames, const unsigned* maxkey, float* chunked,
                         cudaStream_t s) {
  const long long total = static_cast<long long>(total_chunks) * kMels * chunk_frames;
  if (total <= 0) return 0;
  mel_finalize_chunked_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
      scratch, clips, chunk_clip, total_chunks, chunk_frames, maxkey, chunked);
  return (int)cudaGetLastError();
}

int mel_finalize_rows(const float* scratch, int n_frames, const unsigned* maxkey, float* out,
                      cudaStream_t s) {
  const long long total = static_cast<long long>(n_frames) * kMels;
  if (total <= 0) return 0;
  mel_finalize_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(scratch, n_frames,
                                                                          maxkey, out);
  return (int)cudaGetLastError();
}

}  // namespace qa
