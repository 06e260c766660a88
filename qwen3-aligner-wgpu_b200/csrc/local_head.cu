// The Local Head refinement stage (src/local_head.rs:179-611) on the GPU,
// batched over every endpoint (word start / word end) of every clip of a
// batch.  The dense parts (two 5-tap conv1d layers, the audio K/V projection
// and the context projection) are tensor-core GEMMs launched by the runtime
// through gemm_tc with f32-accurate three-term bf16 operands; the kernels here
// are the parts around them:
//
//   lh_masked_argmax   duration-masked argmax of the head logits (one warp
//                      per row), raw_ms = argmax * 80 (src/local_head.rs:209-218)
//   lh_fix             fix_timestamps per clip (src/postprocess.rs:33-113), one
//                      warp per clip: the O(n^2) longest non-decreasing
//                      subsequence with the reference's tie rules, then the
//                      anomaly repair
//   lh_features        one CTA per endpoint: 41 Hann-windowed frames, 512-point
//                      FFTs in f64 in shared memory (the reference's FFT is
//                      f64), the 91 feature channels in the reference's
//                      summation order, the normalizer, written as the
//                      [hi | lo | hi] rows of the first conv's A operand
//                      (src/local_head.rs:359-507)
//   lh_ctx_pack        the context rows: each slot's unfolded final-norm row
//                      and each word's average of its two rows, split into
//                      [hi | lo | hi] (src/local_head.rs:309-346)
//   lh_tail            eight endpoints per CTA: role tokens, the context
//                      attention over four masked rows, query LayerNorm, the
//                      attention over the 41 acoustic frames, audio LayerNorm,
//                      activity / boundary logits and the temperature-1.5
//                      posterior mean over the 13 offsets
//                      (src/local_head.rs:555-611)
//   lh_repair          per clip: fixed + offset intervals, the short-interval
//                      and negative-start rules, remove_neighbor_overlaps and
//                      bound_to_duration in f64 (src/local_head.rs:256-307,
//                      1084-1130)
#include "kernels.cuh"
#include "sm100.cuh"

#include <cuda_bf16.h>

namespace qa {

namespace {

constexpr int kCtxFrames = 20;

__device__ __forceinline__ uint16_t bf16_bits(float x) {
  const __nv_bfloat16 h = __float2bfloat16_rn(x);
  return *reinterpret_cast<const uint16_t*>(&h);
}

__device__ __forceinline__ float bf16_val(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// ---------------------------------------------------------------- argmax

// One warp per row: the first maximum over the clip's valid classes (a strict
// `>` scan, so NaN never wins), as (idx * 80.0) truncated to i64.
__global__ void lh_masked_argmax_kernel(const float* __restrict__ logits, int E, int n_labels,
                                        const LhClip* __restrict__ clips,
                                        const int* __restrict__ ep_clip, long long* raw) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= E) return;
  const int valid = clips[ep_clip[warp]].valid;
  const float* row = logits + static_cast<long long>(warp) * n_labels;
  float best = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int i = lane; i < valid; i += 32) {
    const float v = row[i];
    if (v > best) {  // ascending i per lane: the first maximum of the lane
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  // no lane saw a value above -inf: the scan keeps index 0
  if (lane == 0) raw[warp] = static_cast<long long>(static_cast<double>(bi == 0x7FFFFFFF ? 0 : bi) * 80.0);
}

// ---------------------------------------------------------------- fix_timestamps

// One warp per clip; dynamic shared memory holds the clip's values, LIS
// lengths, parents and flags.
__global__ void lh_fix_kernel(const long long* __restrict__ raw, const LhClip* __restrict__ clips,
                              long long* fixed) {
  extern __shared__ uint8_t smem[];
  pdl_wait();
  pdl_trigger();
  const LhClip cl = clips[blockIdx.x];
  const int n = 2 * cl.n_words;
  const int lane = threadIdx.x;
  long long* v = reinterpret_cast<long long*>(smem);
  int* dp = reinterpret_cast<int*>(v + n);
  int* parent = dp + n;
  int* normal = parent + n;
  const long long* src = raw + cl.ep_off;
  for (int i = lane; i < n; i += 32) {
    v[i] = src[i];
    normal[i] = 0;
  }
  __syncwarp();
  // dp[i] = 1 + max dp[j] over j < i with v[j] <= v[i]; parent = the first
  // such j reaching the maximum (the reference's strict `>` update in j order)
  for (int i = 0; i < n; ++i) {
    const long long vi = v[i];
    int best = 0, bj = -1;
    for (int j = lane; j < i; j += 32)
      if (v[j] <= vi && dp[j] > best) {
        best = dp[j];
        bj = j;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const int ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      const int oj = __shfl_xor_sync(0xFFFFFFFFu, bj, o);
      if (ob > best || (ob == best && ob > 0 && (bj < 0 || (oj >= 0 && oj < bj)))) {
        best = ob;
        bj = oj;
      }
    }
    if (lane == 0) {
      dp[i] = best + 1;
      parent[i] = best > 0 ? bj : -1;
    }
    __syncwarp();
  }
  if (lane == 0 && n > 0) {
    int mi = 0;
    for (int i = 1; i < n; ++i)
      if (dp[i] > dp[mi]) mi = i;  // first position of the maximum
    for (int i = mi; i != -1; i = parent[i]) normal[i] = 1;
    // anomaly blocks: nearest normal value on each side, then the reference's
    // snap (<= 2 values) / interpolate / fill rules
    long long* out = fixed + cl.ep_off;
    for (int i = 0; i < n; ++i) out[i] = v[i];
    int bs = 0;
    while (bs < n) {
      if (normal[bs]) {
        ++bs;
        continue;
      }
      int be = bs;
      while (be < n && !normal[be]) ++be;
      const int cnt = be - bs;
      const bool hl = bs > 0;   // the element before a block is normal
      const bool hr = be < n;   // so is the one after it
      const long long lv = hl ? v[bs - 1] : 0, rv = hr ? v[be] : 0;
      if (hl || hr) {
        if (cnt <= 2) {
          for (int p = bs; p < be; ++p)
            out[p] = (hl && hr) ? ((p - (bs - 1) <= be - p) ? lv : rv) : (hl ? lv : rv);
        } else if (hl && hr) {
          const double step = static_cast<double>(rv - lv) / static_cast<double>(cnt + 1);
          for (int p = bs; p < be; ++p)
            out[p] = static_cast<long long>(static_cast<double>(lv) + step * static_cast<double>(p - bs + 1));
        } else {
          for (int p = bs; p < be; ++p) out[p] = hl ? lv : rv;
        }
      }
      bs = be;
    }
  }
}

// ---------------------------------------------------------------- features

constexpr int kFeatThreads = 256;
constexpr int kMagStride = kLhBins;  // 257 floats per frame

// The 41 real frames go through the FFT two at a time, frame 2p as the real
// and frame 2p + 1 as the imaginary part of one complex transform (21 complex
// transforms, the last with one frame), kFftGroup transforms at once.  The
// endpoint's audio under the 41 frames (6,800 samples: the frames are 160
// apart and 400 long) and the Hann window are staged in shared memory first,
// so that the energy and FFT passes read no global memory.  The staging and
// the transforms' buffers are dead once the magnitudes are out, so the
// mean-removed log spectrum reuses their space.  Two CTAs fit on an SM.
constexpr int kFftGroup = 3;
static_assert(kLhNfft == 512 && kFeatThreads == 256, "the butterfly indexing assumes 512 points");
constexpr int kFftPairs = (kLhFrames + 1) / 2;
constexpr int kWinLen = (kLhFrames - 1) * 160 + kLhFrameLen;

struct FftStage {
  double2 tw[kLhNfft / 2];
  double2 buf[kFftGroup][kLhNfft];
  float win[kWinLen];       // audio[center - 3400 + i], zero outside the clip
  float hann[kLhFrameLen];
};

struct FeatSmem {
  union {
    FftStage fs;
    float nrm[kLhFrames * kMagStride];
  };
  float mag[kLhFrames * kMagStride];
  float feat[kLhFrames * kLhFeat];
  float energy[kLhFrames];
  float fmean[kLhFrames];
};

__device__ __forceinline__ int bitrev9(int x) { return static_cast<int>(__brev(static_cast<unsigned>(x)) >> 23); }

__global__ void __launch_bounds__(kFeatThreads)
    lh_features_kernel(const float* __restrict__ samples, const LhClip* __restrict__ clips,
                       const int* __restrict__ ep_clip, const long long* __restrict__ fixed,
                       LhFeatConst kc, uint16_t* __restrict__ x1, uint16_t* __restrict__ x2,
                       float* __restrict__ feat_out) {
  extern __shared__ uint8_t smem_raw[];
  FeatSmem& S = *reinterpret_cast<FeatSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 15) & ~static_cast<uintptr_t>(15));
  const int e = blockIdx.x;
  const int tid = threadIdx.x;
  FftStage& F = S.fs;
  for (int i = tid; i < kLhNfft / 2; i += kFeatThreads) F.tw[i] = kc.twiddle[i];
  for (int j = tid; j < kLhFrameLen; j += kFeatThreads) F.hann[j] = kc.hann[j];
  pdl_wait();
  pdl_trigger();
  const LhClip cl = clips[ep_clip[e]];
  const float* audio = samples + cl.sample_off;
  const long long center = fixed[e] * 16000 / 1000;
  // frame f starts at center + (f - 20) * 160 - 200 = win start + 160 f
  const long long win0 = center - static_cast<long long>(kCtxFrames) * 160 - 200;
  for (int i = tid; i < kWinLen; i += kFeatThreads) {
    const long long idx = win0 + i;
    F.win[i] = (idx >= 0 && idx < cl.n_samples) ? audio[idx] : 0.f;
  }
  __syncthreads();
  // sample j of frame f, Hann-windowed (zero past the 400-sample frame: the
  // FFT input is zero-padded to 512, and past the last frame)
  auto frame_sample = [&](int f, int j) -> float {
    if (f >= kLhFrames || j >= kLhFrameLen) return 0.f;
    return F.win[f * 160 + j] * F.hann[j];
  };
  // frame energies: one warp per frame, lanes strided over the samples
  for (int f = tid >> 5; f < kLhFrames; f += kFeatThreads / 32) {
    float en = 0.f;
    for (int j = tid & 31; j < kLhFrameLen; j += 32) {
      const float x = frame_sample(f, j);
      en = fmaf(x, x, en);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) en += __shfl_xor_sync(0xFFFFFFFFu, en, o);
    if ((tid & 31) == 0) S.energy[f] = en;
  }
  for (int p0 = 0; p0 < kFftPairs; p0 += kFftGroup) {
    const int ng = min(kFftGroup, kFftPairs - p0);
    // bit-reversed load: element i of transform g holds sample bitrev(i) of
    // frames 2(p0 + g) (real) and 2(p0 + g) + 1 (imaginary)
    for (int idx = tid; idx < ng * kLhNfft; idx += kFeatThreads) {
      const int g = idx / kLhNfft, i = idx - g * kLhNfft;
      const int src = bitrev9(i), f = 2 * (p0 + g);
      F.buf[g][i] = make_double2(static_cast<double>(frame_sample(f, src)),
                                 static_cast<double>(frame_sample(f + 1, src)));
    }
    __syncthreads();
    // radix-2 decimation-in-time stages, kLhNfft / 2 butterflies per
    // transform; stage lh pairs elements 2^lh apart (shifts, no divisions)
    for (int lh = 0; lh < 9; ++lh) {
      const int half = 1 << lh;
      for (int b = tid; b < ng * (kLhNfft / 2); b += kFeatThreads) {
        const int g = b >> 8, bb = b & (kLhNfft / 2 - 1);
        const int k = bb & (half - 1);
        const int i0 = ((bb >> lh) << (lh + 1)) + k, i1 = i0 + half;
        const double2 w = F.tw[k << (8 - lh)];
        const double2 u = F.buf[g][i0], x = F.buf[g][i1];
        const double tr = w.x * x.x - w.y * x.y;
        const double ti = w.x * x.y + w.y * x.x;
        F.buf[g][i0] = make_double2(u.x + tr, u.y + ti);
        F.buf[g][i1] = make_double2(u.x - tr, u.y - ti);
      }
      __syncthreads();
    }
    // split Z = A + iB of the real frames a, b:
    // A[k] = (Z[k] + conj Z[N-k]) / 2, B[k] = (Z[k] - conj Z[N-k]) / 2i
    for (int idx = tid; idx < ng * kLhBins; idx += kFeatThreads) {
      const int g = idx / kLhBins, k = idx - g * kLhBins;
      const int f = 2 * (p0 + g);
      const double2 z = F.buf[g][k], c = F.buf[g][(kLhNfft - k) & (kLhNfft - 1)];
      S.mag[f * kMagStride + k] = static_cast<float>(hypot(0.5 * (z.x + c.x), 0.5 * (z.y - c.y)));
      if (f + 1 < kLhFrames)
        S.mag[(f + 1) * kMagStride + k] =
            static_cast<float>(hypot(0.5 * (z.y + c.y), 0.5 * (c.x - z.x)));
    }
    __syncthreads();
  }

  // log-mel: the bank row's nonzero bins in ascending order (the zero weights
  // of the reference's full-row sum add exact zeros)
  for (int idx = tid; idx < kLhFrames * kLhMels; idx += kFeatThreads) {
    const int f = idx / kLhMels, m = idx - f * kLhMels;
    const int2 r = kc.bank_range[m];
    const float* mg = S.mag + f * kMagStride;
    const float* bw = kc.bank + m * kLhBins;
    float acc = 0.f;
    for (int b = r.x; b < r.y; ++b) {
      const float p = __fmul_rn(mg[b], mg[b]);
      acc = __fadd_rn(acc, __fmul_rn(bw[b], p));
    }
    S.feat[f * kLhFeat + m] = logf(fmaxf(acc, 1e-6f));
  }
  // mean-removed log spectrum: per frame, sequential sums (one thread a frame)
  for (int idx = tid; idx < kLhFrames * kLhBins; idx += kFeatThreads) {
    const int f = idx / kLhBins, b = idx - f * kLhBins;
    S.nrm[f * kMagStride + b] = logf(fmaxf(S.mag[f * kMagStride + b], 1e-6f));
  }
  __syncthreads();
  if (tid < kLhFrames) {  // per frame: the spectrum's mean and the flux
    const int f = tid;
    float mean = 0.f;
    for (int b = 0; b < kLhBins; ++b) mean = __fadd_rn(mean, S.nrm[f * kMagStride + b]);
    S.fmean[f] = __fdiv_rn(mean, static_cast<float>(kLhBins));
    float flux = 0.f;
    if (f > 0) {
      float pos = 0.f, tot = 0.f;
      const float* cur = S.mag + f * kMagStride;
      const float* prv = S.mag + (f - 1) * kMagStride;
      for (int b = 0; b < kLhBins; ++b) {
        pos = __fadd_rn(pos, fmaxf(__fsub_rn(cur[b], prv[b]), 0.f));
        tot = __fadd_rn(tot, prv[b]);
      }
      flux = __fdiv_rn(pos, __fadd_rn(tot, 1e-6f));
    }
    S.feat[f * kLhFeat + kLhMels + 2] = flux;
  }
  __syncthreads();
  for (int idx = tid; idx < kLhFrames * kLhBins; idx += kFeatThreads) {
    const int f = idx / kLhBins, b = idx - f * kLhBins;
    S.nrm[f * kMagStride + b] = __fsub_rn(S.nrm[f * kMagStride + b], S.fmean[f]);
  }
  __syncthreads();
  // band distances: (frame, band, side) per thread, sequential over the band;
  // band edges 1 + 256 i / 4 (src/local_head.rs:975-982)
  for (int idx = tid; idx < kLhFrames * kLhBands * 2; idx += kFeatThreads) {
    const int f = idx / (kLhBands * 2), r = idx - f * (kLhBands * 2);
    const int band = r % kLhBands, side = r / kLhBands;
    const int left = static_cast<int>(1.0 + (kLhBins - 1.0) * band / kLhBands);
    const int right = max(static_cast<int>(1.0 + (kLhBins - 1.0) * (band + 1) / kLhBands), left + 1);
    const int g = side == 0 ? (f == 0 ? f : f - 1) : (f + 1 == kLhFrames ? f : f + 1);
    const float* cur = S.nrm + f * kMagStride;
    const float* nb = S.nrm + g * kMagStride;
    float acc = 0.f;
    for (int b = left; b < right; ++b) acc = __fadd_rn(acc, fabsf(__fsub_rn(cur[b], nb[b])));
    S.feat[f * kLhFeat + kLhMels + 3 + side * kLhBands + band] =
        __fdiv_rn(acc, static_cast<float>(right - left));
  }
  __syncthreads();
  // log-RMS and its delta
  if (tid < kLhFrames) {
    const int f = tid;
    auto lrms = [&](int k) {
      return logf(fmaxf(sqrtf(__fadd_rn(__fdiv_rn(S.energy[k], static_cast<float>(kLhFrameLen)), 1e-6f)), 1e-6f));
    };
    const float cur = lrms(f);
    S.feat[f * kLhFeat + kLhMels] = cur;
    S.feat[f * kLhFeat + kLhMels + 1] = f == 0 ? 0.f : __fsub_rn(cur, lrms(f - 1));
  }
  __syncthreads();
  // normalizer, then the conv A rows [hi | lo | hi] (channels >= 91 zero) of
  // the endpoint's 45-row block (rows 0, 1, 43, 44 are the conv padding);
  // the second conv's padding rows are cleared here too
  uint16_t* xb = x1 + static_cast<long long>(e) * kLhRows * kLhXw;
  uint16_t* x2b = x2 + static_cast<long long>(e) * kLhRows * kLhXw;
  for (int idx = tid; idx < kLhRows * kLhCh; idx += kFeatThreads) {
    const int r = idx / kLhCh, c = idx - r * kLhCh;
    const int f = r - 2;
    float v = 0.f;
    if (f >= 0 && f < kLhFrames && c < kLhFeat) {
      v = __fdiv_rn(__fsub_rn(S.feat[f * kLhFeat + c], kc.mean[c]), kc.stdv[c]);
      if (feat_out) feat_out[(static_cast<long long>(e) * kLhFrames + f) * kLhFeat + c] = v;
    }
    const uint16_t hi = bf16_bits(v);
    const uint16_t lo = bf16_bits(v - bf16_val(hi));
    uint16_t* row = xb + r * kLhXw;
    row[c] = hi;
    row[kLhCh + c] = lo;
    row[2 * kLhCh + c] = hi;
    if (f < 0 || f >= kLhFrames) {
      uint16_t* row2 = x2b + r * kLhXw;
      row2[c] = 0;
      row2[kLhCh + c] = 0;
      row2[2 * kLhCh + c] = 0;
    }
  }
}

// ---------------------------------------------------------------- context rows

// Row i < E: the slot's row; row E + j: word j's average (row 2j + row 2j+1) / 2
// (the reference's 0 + a + b, then / 2).  [hi | lo | hi] of width 3H.
__global__ void lh_ctx_pack_kernel(const float* __restrict__ normed, int E, int H,
                                   uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const int words = E / 2;
  if (row >= E + words) return;
  uint16_t* dst = out + static_cast<long long>(row) * 3 * H;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float v;
    if (row < E) {
      v = normed[static_cast<long long>(row) * H + c];
    } else {
      const int j = row - E;
      const float a = normed[static_cast<long long>(2 * j) * H + c];
      const float b = normed[static_cast<long long>(2 * j + 1) * H + c];
      v = __fdiv_rn(__fadd_rn(__fadd_rn(0.f, a), b), 2.0f);
    }
    const uint16_t hi = bf16_bits(v);
    dst[c] = hi;
    dst[H + c] = bf16_bits(v - bf16_val(hi));
    dst[2 * H + c] = hi;
  }
}

// ---------------------------------------------------------------- tail

constexpr int kTailEp = 8;        // endpoints per CTA
constexpr int kTailThreads = 256;
constexpr int kD = 128;

struct TailSmem {
  float tok[kTailEp][4][kD];
  float kc[kTailEp][4][kD];
  float vc[kTailEp][4][kD];
  float base[kTailEp][kD];
  float q[kTailEp][kD];
  float att[kTailEp][kD];
  float qry[kTailEp][kD];
  float sc[kTailEp][4][kLhFrames];
  float act[kTailEp][16];
  float loc[kTailEp][16];
  float mask[kTailEp][4];
  int ok[kTailEp];
};

// y[v][d] = b[d] + sum_j wt[j][d] x[v][j] for v < nv (x, y rows kD apart in
// shared memory, wt transposed [in][out] so that the d lanes read one line).
__device__ __forceinline__ void tail_mv(const float* __restrict__ wt, const float* __restrict__ b,
                                        const float* x, float* y, int nv) {
  const int d = threadIdx.x & (kD - 1);
  const int g = threadIdx.x >> 7;  // two groups of vectors
  const float bd = __ldg(b + d);
  for (int v0 = g * 4; v0 < nv; v0 += 8) {
    const int cnt = min(4, nv - v0);
    float acc[4] = {bd, bd, bd, bd};
#pragma unroll 4
    for (int j = 0; j < kD; ++j) {
      const float w = __ldg(wt + j * kD + d);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (k < cnt) acc[k] = fmaf(w, x[(v0 + k) * kD + j], acc[k]);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (k < cnt) y[(v0 + k) * kD + d] = acc[k];
  }
}

// LayerNorm (eps 1e-5) of one 128-vector by one warp, in place.
__device__ __forceinline__ void warp_ln(float* x, const float* __restrict__ w,
                                        const float* __restrict__ b) {
  const int lane = threadIdx.x & 31;
  float v[4];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[k] = x[lane + 32 * k];
    s += v[k];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  const float mean = s / kD;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) q += (v[k] - mean) * (v[k] - mean);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
  const float inv = 1.0f / sqrtf(q / kD + 1e-5f);
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = lane + 32 * k;
    x[d] = (v[k] - mean) * inv * __ldg(w + d) + __ldg(b + d);
  }
  __syncwarp();
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__global__ void __launch_bounds__(kTailThreads)
    lh_tail_kernel(const float* __restrict__ P, const float* __restrict__ kv,
                   const float* __restrict__ audio, const LhClip* __restrict__ clips,
                   const int* __restrict__ ep_clip, int E, LhTailW W, float* __restrict__ offsets) {
  extern __shared__ uint8_t smem_raw[];
  TailSmem& S = *reinterpret_cast<TailSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 15) & ~static_cast<uintptr_t>(15));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int e0 = blockIdx.x * kTailEp;
  const int nep = min(kTailEp, E - e0);
  pdl_wait();
  pdl_trigger();
  // 1. role tokens and the endpoint query (src/local_head.rs:555-568)
  for (int idx = tid; idx < kTailEp * 4 * kD; idx += kTailThreads) {
    const int i = idx / (4 * kD), r = (idx / kD) & 3, d = idx & (kD - 1);
    float v = 0.f;
    if (i < nep) {
      const int e = e0 + i;
      const LhClip cl = clips[ep_clip[e]];
      const int slot = e - cl.ep_off, w = slot >> 1;
      const int wg = e >> 1;  // global word index (clips hold whole words)
      int row = -1;
      if (r == 0) row = e;
      else if (r == 1) row = E + wg;
      else if (r == 2 && w > 0) row = E + wg - 1;
      else if (r == 3 && w + 1 < cl.n_words) row = E + wg + 1;
      // a missing neighbour is a zero row: its projection is the bias
      v = (row >= 0 ? P[static_cast<long long>(row) * kD + d] : __ldg(W.ctx_b + d)) +
          __ldg(W.role + r * kD + d);
      if (d == 0) S.mask[i][r] = (r < 2 || row >= 0) ? 1.f : 0.f;
      if (r == 0 && d == 0) S.ok[i] = slot & 1;
    } else if (d == 0) {
      S.mask[i][r] = 1.f;
      if (r == 0) S.ok[i] = 0;
    }
    S.tok[i][r][d] = v;
  }
  __syncthreads();
  for (int idx = tid; idx < kTailEp * kD; idx += kTailThreads) {
    const int i = idx / kD, d = idx & (kD - 1);
    S.base[i][d] = i < nep ? S.tok[i][0][d] + __ldg(W.endpoint + S.ok[i] * kD + d) : 0.f;
  }
  __syncthreads();
  // 2. context attention: q from the endpoint query, k / v from the 4 tokens
  tail_mv(W.cq, W.cbq, &S.base[0][0], &S.q[0][0], kTailEp);
  tail_mv(W.ck, W.cbk, &S.tok[0][0][0], &S.kc[0][0][0], kTailEp * 4);
  tail_mv(W.cv, W.cbv, &S.tok[0][0][0], &S.vc[0][0][0], kTailEp * 4);
  __syncthreads();
  const float scale = 1.0f / sqrtf(32.0f);
  if (tid < kTailEp * 4 * 4) {  // (endpoint, head, key)
    const int i = tid >> 4, h = (tid >> 2) & 3, r = tid & 3;
    float acc = 0.f;
    for (int d = 0; d < 32; ++d) acc += S.q[i][h * 32 + d] * S.kc[i][r][h * 32 + d];
    S.sc[i][h][r] = S.mask[i][r] == 0.f ? -INFINITY : acc * scale;
  }
  __syncthreads();
  if (tid < kTailEp * 4) {  // softmax over the 4 keys
    const int i = tid >> 2, h = tid & 3;
    float mx = -INFINITY;
    for (int r = 0; r < 4; ++r) mx = fmaxf(mx, S.sc[i][h][r]);
    float p[4], tot = 0.f;
    for (int r = 0; r < 4; ++r) {
      p[r] = expf(S.sc[i][h][r] - mx);
      tot += p[r];
    }
    for (int r = 0; r < 4; ++r) S.sc[i][h][r] = p[r] / tot;
  }
  __syncthreads();
  for (int idx = tid; idx < kTailEp * kD; idx += kTailThreads) {
    const int i = idx / kD, d = idx & (kD - 1), h = d >> 5;
    float acc = 0.f;
    for (int r = 0; r < 4; ++r) acc += S.sc[i][h][r] * S.vc[i][r][d];
    S.att[i][d] = acc;
  }
  __syncthreads();
  tail_mv(W.co, W.co_b, &S.att[0][0], &S.qry[0][0], kTailEp);
  __syncthreads();
  // residual + query_norm (one warp per endpoint)
  for (int i = warp; i < kTailEp; i += kTailThreads / 32) {
    for (int d = lane; d < kD; d += 32) S.qry[i][d] += S.base[i][d];
    __syncwarp();
    warp_ln(&S.qry[i][0], W.qn_w, W.qn_b);
  }
  __syncthreads();
  // 3. attention over the 41 acoustic frames (k = kv columns 0..127, v = 128..255)
  tail_mv(W.aq, W.abq, &S.qry[0][0], &S.q[0][0], kTailEp);
  __syncthreads();
  for (int idx = tid; idx < kTailEp * 4 * kLhFrames; idx += kTailThreads) {
    const int i = idx / (4 * kLhFrames), rem = idx - i * 4 * kLhFrames;
    const int h = rem / kLhFrames, t = rem - h * kLhFrames;
    float acc = -INFINITY;
    if (i < nep) {
      const float4* k4 = reinterpret_cast<const float4*>(
          kv + (static_cast<long long>(e0 + i) * kLhFrames + t) * 2 * kD + h * 32);
      acc = 0.f;
#pragma unroll
      for (int d4 = 0; d4 < 8; ++d4) {
        const float4 k = k4[d4];
        const float* q = &S.q[i][h * 32 + 4 * d4];
        acc += q[0] * k.x + q[1] * k.y + q[2] * k.z + q[3] * k.w;
      }
      acc *= scale;
    }
    S.sc[i][h][t] = acc;
  }
  __syncthreads();
  if (tid < kTailEp * 4) {
    const int i = tid >> 2, h = tid & 3;
    if (i < nep) {
      float mx = -INFINITY;
      for (int t = 0; t < kLhFrames; ++t) mx = fmaxf(mx, S.sc[i][h][t]);
      float tot = 0.f;
      for (int t = 0; t < kLhFrames; ++t) {
        const float p = expf(S.sc[i][h][t] - mx);
        S.sc[i][h][t] = p;
        tot += p;
      }
      for (int t = 0; t < kLhFrames; ++t) S.sc[i][h][t] /= tot;
    }
  }
  __syncthreads();
  for (int idx = tid; idx < kTailEp * kD; idx += kTailThreads) {
    const int i = idx / kD, d = idx & (kD - 1), h = d >> 5;
    float acc = 0.f;
    if (i < nep) {
      const float* vcol = kv + static_cast<long long>(e0 + i) * kLhFrames * 2 * kD + kD + d;
      for (int t = 0; t < kLhFrames; ++t) acc += S.sc[i][h][t] * vcol[t * 2 * kD];
    }
    S.att[i][d] = acc;
  }
  __syncthreads();
  tail_mv(W.ao, W.ao_b, &S.att[0][0], &S.base[0][0], kTailEp);  // base reused as scratch
  __syncthreads();
  for (int i = warp; i < kTailEp; i += kTailThreads / 32) {
    for (int d = lane; d < kD; d += 32) S.qry[i][d] += S.base[i][d];
    __syncwarp();
    warp_ln(&S.qry[i][0], W.qn_w, W.qn_b);
  }
  __syncthreads();
  // 4. audio_norm rows 13..26 (the ones the decode reads), activity and
  // boundary logits (src/local_head.rs:590-605)
  const float root = sqrtf(static_cast<float>(kD));
  for (int job = warp; job < kTailEp * 14; job += kTailThreads / 32) {
    const int i = job / 14, t = 13 + job % 14;
    if (i >= nep) continue;
    const float* src = audio + (static_cast<long long>(e0 + i) * kLhFrames + t) * kD;
    float v[4];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[k] = src[lane + 32 * k];
      s += v[k];
    }
    s = warp_sum(s);
    const float mean = s / kD;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) q += (v[k] - mean) * (v[k] - mean);
    q = warp_sum(q);
    const float inv = 1.0f / sqrtf(q / kD + 1e-5f);
    float dq = 0.f, da = 0.f, db = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int d = lane + 32 * k;
      const float n = (v[k] - mean) * inv * __ldg(W.an_w + d) + __ldg(W.an_b + d);
      dq += n * S.qry[i][d];
      da += __ldg(W.act_w + d) * n;
      db += __ldg(W.bnd_w + d) * n;
    }
    dq = warp_sum(dq);
    da = warp_sum(da);
    db = warp_sum(db);
    if (lane == 0) {
      S.act[i][t - 13] = dq / root + da + W.act_b;
      S.loc[i][t - 13] = dq / root + db + W.bnd_b;
    }
  }
  __syncthreads();
  // 5. posterior mean over the 13 offsets at temperature 1.5
  if (tid < nep) {
    const int i = tid;
    const int is_end = S.ok[i];
    float lg[13];
    float mx = -INFINITY;
    for (int j = 0; j < 13; ++j) {
      const float der = S.act[i][j + 1] - S.act[i][j];
      const float dir = is_end == 0 ? der : -der;
      lg[j] = (S.loc[i][j + 1] + W.derivative_scale * dir + __ldg(W.prior + j)) / 1.5f;
      mx = fmaxf(mx, lg[j]);
    }
    float tot = 0.f;
    for (int j = 0; j < 13; ++j) {
      lg[j] = expf(lg[j] - mx);
      tot += lg[j];
    }
    float off = 0.f;
    for (int j = 0; j < 13; ++j) off += (lg[j] / tot) * static_cast<float>(10 * j - 60);
    offsets[e0 + i] = off;
  }
}

// ---------------------------------------------------------------- repair

__global__ void lh_repair_kernel(const long long* __restrict__ fixed, const float* __restrict__ off,
                                 const LhClip* __restrict__ clips, int n_clips, double* out) {
  pdl_wait();
  pdl_trigger();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n_clips) return;
  const LhClip cl = clips[c];
  const int W = cl.n_words;
  const double min_ms = 10.0;
  const double duration = static_cast<double>(cl.n_samples) * 1000.0 / 16000.0;
  double* iv = out + static_cast<long long>(cl.ep_off);  // [W][2], ep_off = 2 * word offset
  const long long* fx = fixed + cl.ep_off;
  const float* of = off + cl.ep_off;
  for (int i = 0; i < W; ++i) {
    const double fs = static_cast<double>(fx[2 * i]), fe = static_cast<double>(fx[2 * i + 1]);
    double s = fs + static_cast<double>(of[2 * i]), e = fe + static_cast<double>(of[2 * i + 1]);
    if (!isfinite(s) || !isfinite(e)) {
      s = fs;
      e = fe;
    } else if (e - s < min_ms) {
      const double mid = (s + e) / 2.0;
      if (mid < min_ms / 2.0) {
        s = 0.0;
        e = min_ms;
      } else {
        s = mid - min_ms / 2.0;
        e = mid + min_ms / 2.0;
      }
    } else if (s < 0.0) {
      e -= s;
      s = 0.0;
    }
    if (!isfinite(s) || !isfinite(e) || s < 0.0 || e < 0.0 || e - s < min_ms) {
      s = 0.0;
      e = min_ms;
    }
    iv[2 * i] = s;
    iv[2 * i + 1] = e;
  }
  // remove_neighbor_overlaps
  for (int i = 0; i + 1 < W; ++i) {
    if (iv[2 * i + 1] <= iv[2 * i + 2]) continue;
    double cut = iv[2 * i + 2];
    const double minimum_cut = iv[2 * i] + min_ms;
    if (cut < minimum_cut) {
      cut = minimum_cut;
      iv[2 * i + 2] = cut;
      iv[2 * i + 3] = fmax(iv[2 * i + 3], cut + min_ms);
    }
    iv[2 * i + 1] = cut;
  }
  // bound_to_duration
  if (W > 0) {
    const double minimum = fmin(min_ms, duration / W);
    bool inside = true;
    for (int i = 0; i < W; ++i) {
      const double s = iv[2 * i], e = iv[2 * i + 1];
      if (!(isfinite(s) && isfinite(e) && s >= 0.0 && s < e && e <= duration)) inside = false;
    }
    if (!inside) {
      double cursor = 0.0;
      for (int i = 0; i < W; ++i) {
        double s = iv[2 * i], e = iv[2 * i + 1];
        if (!isfinite(s) || !isfinite(e)) {
          s = 0.0;
          e = duration;
        }
        const double remaining = static_cast<double>(W - i - 1);
        const double latest_start = duration - minimum * (remaining + 1.0);
        s = fmin(fmax(s, cursor), latest_start);
        const double earliest_end = s + minimum;
        const double latest_end = duration - minimum * remaining;
        e = fmin(fmax(e, earliest_end), latest_end);
        iv[2 * i] = s;
        iv[2 * i + 1] = e;
        cursor = e;
      }
    }
  }
  for (int i = 0; i < 2 * W; ++i) iv[i] /= 1000.0;
}

}  // namespace

// 228 KB of shared memory per SM, 1 KB of it reserved per resident CTA
static_assert(2 * (sizeof(FeatSmem) + 16 + 1024) <= 228 * 1024, "two feature CTAs per SM");
size_t lh_features_smem() { return sizeof(FeatSmem) + 16; }
size_t lh_tail_smem() { return sizeof(TailSmem) + 16; }

int lh_masked_argmax(const float* logits, int E, int n_labels, const LhClip* clips,
                     const int* ep_clip, long long* raw, cudaStream_t s) {
  if (E <= 0) return 0;
  const int threads = 256;
  const int blocks = (E * 32 + threads - 1) / threads;
  return (int)launch_pdl(lh_masked_argmax_kernel, dim3(blocks), dim3(threads), 0, s, logits, E,
                         n_labels, clips, ep_clip, raw);
}

int lh_fix(const long long* raw, const LhClip* clips, int n_clips, int max_slots, long long* fixed,
           cudaStream_t s) {
  if (n_clips <= 0) return 0;
  const size_t smem = static_cast<size_t>(max_slots) * (8 + 4 + 4 + 4);
  if (smem > 200 * 1024) return (int)cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(lh_fix_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return (int)e;
  return (int)launch_pdl(lh_fix_kernel, dim3(n_clips), dim3(32), smem, s, raw, clips, fixed);
}

int lh_features(const float* samples, const LhClip* clips, const int* ep_clip,
                const long long* fixed, int E, const LhFeatConst& kc, uint16_t* x1, uint16_t* x2,
                float* feat_out, cudaStream_t s) {
  if (E <= 0) return 0;
  const size_t smem = lh_features_smem();
  cudaError_t e = cudaFuncSetAttribute(lh_features_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return (int)e;
  // the whole 228 KB of the SM as shared memory: two CTAs resident
  e = cudaFuncSetAttribute(lh_features_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return (int)e;
  return (int)launch_pdl(lh_features_kernel, dim3(E), dim3(kFeatThreads), smem, s, samples, clips,
                         ep_clip, fixed, kc, x1, x2, feat_out);
}

int lh_ctx_pack(const float* normed, int E, int H, uint16_t* out, cudaStream_t s) {
  if (E <= 0) return 0;
  return (int)launch_pdl(lh_ctx_pack_kernel, dim3(E + E / 2), dim3(256), 0, s, normed, E, H, out);
}

int lh_tail(const float* P, const float* kv, const float* audio, const LhClip* clips,
            const int* ep_clip, int E, const LhTailW& w, float* offsets, cudaStream_t s) {
  if (E <= 0) return 0;
  const size_t smem = lh_tail_smem();
  cudaError_t e = cudaFuncSetAttribute(lh_tail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return (int)e;
  return (int)launch_pdl(lh_tail_kernel, dim3((E + kTailEp - 1) / kTailEp), dim3(kTailThreads),
                         smem, s, P, kv, audio, clips, ep_clip, E, w, offsets);
}

int lh_repair(const long long* fixed, const float* offsets, const LhClip* clips, int n_clips,
              double* intervals, cudaStream_t s) {
  if (n_clips <= 0) return 0;
  return (int)launch_pdl(lh_repair_kernel, dim3((n_clips + 63) / 64), dim3(64), 0, s, fixed,
                         offsets, clips, n_clips, intervals);
}

}  // namespace qa
