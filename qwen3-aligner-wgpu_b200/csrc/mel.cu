// (a) Log-mel spectrogram on the GPU, batched over clips.
//
// Same steps as src/mel.rs:198-242: reflect-pad 200, periodic Hann (400),
// 400-point DFT power (201 bins), 128-bin slaney filterbank applied in
// ascending-bin order, log10 with a 1e-10 floor, per-clip max, clamp at
// max - 8, (x + 4) / 4, trailing frame dropped (n_samples / 160 frames).
//
// Pass 1 runs the DFT on the tensor cores: a row builder writes every frame's
// reflected samples (scaled by 2^12, an exact power of two) as f16 hi + lo
// parts, one GEMM against the Hann-windowed cos / -sin rows (also split into
// hi + lo) gives re and im in f32, and a third kernel forms the power (the
// scaling undone exactly), applies the sparse filterbank and the log, and
// takes the per-clip maximum as an atomicMax on an order-preserving integer
// encoding.  Pass 2 clamps and writes the chunked encoder input.
#include <cmath>

#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace qa {

namespace {

constexpr int kNfft = 400;
constexpr int kBins = 201;
constexpr int kHop = 160;
constexpr int kPad = 200;
constexpr int kMels = 128;
constexpr int kFT = 16;  // frames per CTA of the power / filterbank kernel

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

// ---- tensor-core pass 1
constexpr int kFrRows = 8;          // frames per CTA of the row builder
constexpr float kMelScale = 4096.0f;  // 2^12: keeps the lo halves normal f16

// A rows: frame f of clip c -> row frame_off + f, [hi | lo | hi] of
// 2^12 * x[reflect(160 f + j - 200)], two samples per thread.
__global__ void __launch_bounds__(256) mel_frames_kernel(const float* __restrict__ samples,
                                                         const MelClip* __restrict__ clips,
                                                         __half* __restrict__ a) {
  const MelClip c = clips[blockIdx.y];
  const int f0 = blockIdx.x * kFrRows;
  if (f0 >= c.n_frames) return;
  const float* x = samples + c.sample_off;
  const long long n = c.n_samples;
  for (int item = threadIdx.x; item < kFrRows * (kNfft / 2); item += blockDim.x) {
    const int f = f0 + item / (kNfft / 2);
    if (f >= c.n_frames) break;
    const int j = 2 * (item % (kNfft / 2));
    const long long p0 = static_cast<long long>(f) * kHop + j - kPad;
    const float v0 = x[reflect_index(p0, n)] * kMelScale;
    const float v1 = x[reflect_index(p0 + 1, n)] * kMelScale;
    const __half2 hi = __floats2half2_rn(v0, v1);
    const float2 hf = __half22float2(hi);
    const __half2 lo = __floats2half2_rn(v0 - hf.x, v1 - hf.y);
    __half2* row = reinterpret_cast<__half2*>(a + static_cast<long long>(c.frame_off + f) * kMelDftK);
    row[j / 2] = hi;
    row[(kNfft + j) / 2] = lo;
    row[(2 * kNfft + j) / 2] = hi;
  }
}

// Power (the scaling undone exactly), filterbank in ascending-bin order, log10,
// per-clip max, in the reference's operation order.
__global__ void __launch_bounds__(256) mel_power_kernel(const float* __restrict__ spec,
                                                        const MelClip* __restrict__ clips,
                                                        MelBank bank, float log10_factor,
                                                        float* __restrict__ scratch,
                                                        unsigned* __restrict__ maxkey) {
  __shared__ float s_pow[kFT][kBins + 1];
  __shared__ unsigned s_max;
  const MelClip c = clips[blockIdx.y];
  const int f0 = blockIdx.x * kFT;
  if (f0 >= c.n_frames) return;
  const int nf = min(kFT, c.n_frames - f0);
  if (threadIdx.x == 0) s_max = 0u;
  constexpr float kUnscale = 1.0f / (kMelScale * kMelScale);
  for (int item = threadIdx.x; item < kFT * kBins; item += blockDim.x) {
    const int f = item / kBins, k = item % kBins;
    if (f >= nf) break;
    const float* r = spec + static_cast<long long>(c.frame_off + f0 + f) * kMelDftRows;
    const float re = r[k], im = r[kMelImRow + k];
    s_pow[f][k] = __fmul_rn(__fadd_rn(__fmul_rn(re, re), __fmul_rn(im, im)), kUnscale);
  }
  __syncthreads();
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

int mel_logpower_tc(const float* samples, const MelClip* clips, int n_clips, int max_frames,
                    int total_frames, const void* dft_hilo, MelBank bank, float log10_factor,
                    void* frames_ws, float* spec_ws, float* scratch, unsigned* maxkey,
                    unsigned* status, cudaStream_t s) {
  if (n_clips <= 0 || max_frames <= 0 || total_frames <= 0) return 0;
  mel_frames_kernel<<<dim3((max_frames + kFrRows - 1) / kFrRows, n_clips), 256, 0, s>>>(
      samples, clips, static_cast<__half*>(frames_ws));
  int rc = (int)cudaGetLastError();
  if (rc) return rc;
  EpiParams ep;
  ep.mode = EPI_STORE32;
  ep.out = spec_ws;
  ep.ldo = kMelDftRows;
  ep.status = status;
  rc = gemm_tc(frames_ws, kMelDftK, dft_hilo, kMelDftK, total_frames, kMelDftRows, kMelDftK, false,
               ep, s);
  if (rc) return rc;
  mel_power_kernel<<<dim3((max_frames + kFT - 1) / kFT, n_clips), 256, 0, s>>>(
      spec_ws, clips, bank, log10_factor, scratch, maxkey);
  return (int)cudaGetLastError();
}

void mel_dft_hilo(const float* window400, uint16_t* out) {
  for (int n = 0; n < kMelDftRows * kMelDftK; ++n) out[n] = 0;
  for (int n = 0; n < kMelDftRows; ++n) {
    const bool is_re = n < kBins;
    const bool is_im = n >= kMelImRow && n < kMelImRow + kBins;
    if (!is_re && !is_im) continue;
    const int k = is_re ? n : n - kMelImRow;
    for (int j = 0; j < kNfft; ++j) {
      const double ang = 2.0 * M_PI * static_cast<double>((k * j) % kNfft) / kNfft;
      const double t = is_re ? std::cos(ang) : -std::sin(ang);
      const float w = static_cast<float>(static_cast<double>(window400[j]) * t);
      const __half hi = __float2half_rn(w);
      const __half lo = __float2half_rn(w - __half2float(hi));
      uint16_t* row = out + static_cast<long long>(n) * kMelDftK;
      row[j] = __half_as_ushort(hi);
      row[kNfft + j] = __half_as_ushort(hi);
      row[2 * kNfft + j] = __half_as_ushort(lo);
    }
  }
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
