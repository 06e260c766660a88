// tcgen05 / TMEM / TMA GEMM with fused epilogues (see gemm_tc.cuh).
//
// One CTA computes 128 x BN tiles.  Warp roles (320 threads):
//   warp 0      TMA producer: streams 128x64 A and BNx64 B tiles (128B swizzle)
//               into a STAGES-deep shared-memory ring, one mbarrier per slot;
//   warp 1      allocates the TMEM accumulator and issues tcgen05.mma
//               (M=128, N=BN, K=16) from one thread; tcgen05.commit frees a
//               ring slot when the MMAs reading it retire;
//   warps 2..9  epilogue, two warpgroups that split each tile's columns:
//               tcgen05.ld 32x32b pulls one accumulator row per thread (warp
//               w reads TMEM lanes 32*(w%4) .. +31), applies the fused
//               epilogue and stores to global memory.
// Nothing here uses cluster multicast: each CTA loads its own tiles.
#include "gemm_tc.cuh"

#include <algorithm>
#include "sm100.cuh"
#include "tma_host.h"

#include <cstdio>

namespace qa {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;

template <int BN>
struct GemmCfg {
  static constexpr int kStages = (BN >= 192) ? 4 : 6;
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kTmemCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr size_t kSmem = 1024 + kStages * (kABytes + kBBytes) + 256;
};

// GELU with libm-grade erff: the Local Head's conv layers (src/local_head.rs:
// 984-986 computes it on the CPU with erff).
__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int col) {
  uint32_t u = __float_as_uint(v);
  uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(ord) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(col));
}

// Output row of accumulator row `row` (< 0: skip): the periodic layout when
// row_period > 0, else row_map, else the row itself.
__device__ __forceinline__ int out_row(const EpiParams& ep, int row) {
  if (ep.row_period > 0) {
    const int r = row % ep.row_period;
    if (r >= ep.row_valid) return -1;
    return (row / ep.row_period) * ep.row_out_period + ep.row_out_off + r;
  }
  return ep.row_map ? ep.row_map[row] : row;
}

template <typename T>
__device__ __forceinline__ void store16_row(T* dst, const float (&v)[32], int ncols) {
  if (ncols == 32 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = cvt2_rn<T>(make_float2(v[2 * i], v[2 * i + 1]));
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < ncols) dst[i] = f2h<T>(v[i]);
  }
}

template <typename T>
__device__ __forceinline__ void load16_row(const T* src, float (&v)[32], int ncols) {
  if (ncols == 32 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
    alignas(16) T tmp[32];
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(tmp);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = s[i];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = h2f<T>(tmp[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = (i < ncols) ? h2f<T>(src[i]) : 0.f;
  }
}

// 32 consecutive f32 of one row: 16-byte vector accesses when the row
// segment is whole and aligned.
__device__ __forceinline__ bool vec_ok(const void* p, int ncols) {
  return ncols == 32 && (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

__device__ __forceinline__ uint32_t pack_bits(uint16_t lo, uint16_t hi) {
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

template <typename T>
__device__ __forceinline__ uint16_t bits_of(T x) {
  return *reinterpret_cast<const uint16_t*>(&x);
}

template <typename T>
__device__ __forceinline__ float word_half(uint32_t w, int hi) {
  const uint16_t b = hi ? static_cast<uint16_t>(w >> 16) : static_cast<uint16_t>(w & 0xFFFFu);
  return h2f<T>(*reinterpret_cast<const T*>(&b));
}


// The two 16-bit values of a packed word, widened.
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  return make_float2(word_half<T>(w, 0), word_half<T>(w, 1));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2_rn(float2 v) {
  return cvt2_rn<T>(v);
}
// round16 on two lanes: one packed conversion there and two widenings back.
template <typename T>
__device__ __forceinline__ float2 round16x2(float2 v) {
  return unpack2<T>(pack2_rn<T>(v));
}

// Per-row inputs of EPI_QKV_ROPE, loaded before the tile's accumulator is
// ready (their latency then overlaps the tile's MMAs): the row's position,
// its offset in the paged K/V cache (without the K/V head's term), and L1
// prefetches of the row's cos / sin table lines.
struct QkvRow {
  int pos = 0;
  long long kv_off = 0;
  float inv = 1.0f;  // the row's folded RMSNorm factor (ssq_in), else 1
};

// Folded RMSNorm statistics: sums of squares per 128-column block of a row.
constexpr int kSsqCols = 128;
constexpr int kSsqMax = 8;  // blocks per row read by the consumer (rows up to 1024 wide)

// The row's block sums (EpiParams::ssq_in), loaded ahead of their use: the
// epilogue loops issue them for the next tile while they process this one.
struct SsqRow {
  float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f), b = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
};
__device__ __forceinline__ SsqRow ssq_load(const EpiParams& ep, int row, int M) {
  SsqRow r;
  if (!ep.ssq_in || row >= M) return r;
  const float4* p = reinterpret_cast<const float4*>(ep.ssq_in + static_cast<long long>(row) * ep.ssq_n);
  r.a = __ldg(p);
  if (ep.ssq_n > 4) r.b = __ldg(p + 1);
  return r;
}
// 1 / rms of the row from its block sums, summed in block order.
__device__ __forceinline__ float row_rms_inv(const EpiParams& ep, const SsqRow& q) {
  if (!ep.ssq_in) return 1.0f;
  float s = __fadd_rn(__fadd_rn(__fadd_rn(q.a.x, q.a.y), q.a.z), q.a.w);
  if (ep.ssq_n > 4) s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, q.b.x), q.b.y), q.b.z), q.b.w);
  return 1.0f / sqrtf(s / ep.rms_d + ep.rms_eps);
}

template <typename T, bool kPrefetch = true>
__device__ __forceinline__ QkvRow qkv_row_meta(const EpiParams& ep, int row, int M) {
  QkvRow r;
  if (row >= M) return r;
  const RopeKV& rk = ep.rk;
  r.pos = rk.pos_of[row];
  const int clip = rk.clip_of[row];
  const int page = rk.block_tab[clip * rk.max_pages + r.pos / rk.page_size];
  r.kv_off = (static_cast<long long>(page) * rk.nkv * rk.page_size + r.pos % rk.page_size) * 128;
  if constexpr (kPrefetch) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(static_cast<const T*>(rk.cos_t) + r.pos * 64));
    asm volatile("prefetch.global.L1 [%0];" ::"l"(static_cast<const T*>(rk.sin_t) + r.pos * 64));
  }
  return r;
}

// Request the cos (table 0) or sin (table 1) lines of the warp's 32 rows at
// their positions (lane r's `pos`; rows with !ok arrive as zeros) into a 4 KB
// buffer: 128 bytes a row, 16-byte units XOR-swizzled by row, four whole rows
// per cp.async instruction.
template <typename T>
__device__ __forceinline__ void qkv_cs_issue(const EpiParams& ep, uint8_t* buf, int table, int pos,
                                             bool ok) {
  const int lane = threadIdx.x & 31;
  const T* tab = static_cast<const T*>(table ? ep.rk.sin_t : ep.rk.cos_t);
  const uint32_t sb = smem_u32(buf);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (lane >> 3), u = lane & 7;
    const int p = __shfl_sync(0xFFFFFFFFu, pos, r);
    const bool rok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, r) != 0;
    cp_async16(sb + r * 128 + 16 * (u ^ (r & 7)), rok ? tab + p * 64 + 8 * u : tab, rok ? 16u : 0u);
  }
}

// EPI_QKV_ROPE for one 128-column head of this thread's row.  The head's
// values are rounded to the storage type (the GEMM output's rounding point).
// A v head is appended to the cache as rounded.  A q or k head takes RMSNorm
// (the sum of squares of the rounded values in four partial sums), the
// per-element gain and the rotate-half RoPE at the row's position, with every
// product and sum rounded as in the reference's loop (norm_rope_head,
// src/cpu_decoder.rs:305-321), two lanes per f32x2 instruction.  The head is
// read from TMEM twice (sums, then the 32-column chunks d and d + 64 together)
// instead of being held in registers (the 10-warp GEMM kernels have 168
// registers a thread; holding the head spills).  `gain` is the q_norm |
// k_norm gains staged in shared memory; each chunk's four cos and four sin
// 16-byte loads (read-only path) are issued before its TMEM read so that
// their latencies overlap.
template <typename T, bool kStaged>
__device__ __forceinline__ bool qkv_rope_head(const EpiParams& ep, uint32_t tmem_col0, int row,
                                              int M, int head, const QkvRow& meta,
                                              const float* gain, uint8_t* ost, const uint8_t* cs,
                                              uint64_t* csfull, uint32_t cs_parity) {
  constexpr int HD = 128;
  const RopeKV& rk = ep.rk;
  const bool ok = row < M;
  const bool is_q = head < rk.nq, is_v = head >= rk.nq + rk.nkv;
  T* dst;
  if (is_q) {
    dst = static_cast<T*>(ep.out) + (long long)row * ep.ldo + head * HD;
  } else {
    const int kvh = is_v ? head - rk.nq - rk.nkv : head - rk.nq;
    dst = static_cast<T*>(is_v ? rk.vc : rk.kc) + meta.kv_off +
          static_cast<long long>(kvh) * rk.page_size * HD;
  }
  if (is_v) {
#pragma unroll 1
    for (int c = 0; c < HD / 32; c += 2) {
      float v[2][32];
      tmem_ld2x32(tmem_col0 + c * 32, tmem_col0 + (c + 1) * 32, v[0], v[1]);  // warp-collective
      if constexpr (!kStaged) {
        if (!ok) continue;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pack2_rn<T>(mul2_rn(make_float2(v[h][2 * i], v[h][2 * i + 1]), make_float2(meta.inv, meta.inv)));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 d = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
          if constexpr (kStaged)
            stage_unit(ost, 4 * h + j, d);
          else
            reinterpret_cast<uint4*>(dst + (c + h) * 32)[j] = d;
        }
      }
      if constexpr (kStaged) flush_rows<T>(ost, ok ? dst : nullptr, c * 32, c * 32 + 32);
    }
    return true;
  }
  // pass 1: sum of squares of the rounded values (two 32-column chunks per wait)
  float2 s2a = make_float2(0.0f, 0.0f), s2b = make_float2(0.0f, 0.0f);
#pragma unroll 1
  for (int c = 0; c < HD / 32; c += 2) {
    float v[32], w[32];
    tmem_ld2x32(tmem_col0 + c * 32, tmem_col0 + (c + 1) * 32, v, w);
    const float2 r = make_float2(meta.inv, meta.inv);
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float2 x0 = round16x2<T>(mul2_rn(make_float2(v[i], v[i + 1]), r));
      const float2 x1 = round16x2<T>(mul2_rn(make_float2(v[i + 2], v[i + 3]), r));
      s2a = add2_rn(s2a, mul2_rn(x0, x0));
      s2b = add2_rn(s2b, mul2_rn(x1, x1));
    }
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float2 x0 = round16x2<T>(mul2_rn(make_float2(w[i], w[i + 1]), r));
      const float2 x1 = round16x2<T>(mul2_rn(make_float2(w[i + 2], w[i + 3]), r));
      s2a = add2_rn(s2a, mul2_rn(x0, x0));
      s2b = add2_rn(s2b, mul2_rn(x1, x1));
    }
  }
  const float s2 = __fadd_rn(__fadd_rn(s2a.x, s2a.y), __fadd_rn(s2b.x, s2b.y));
  const float inv = 1.0f / sqrtf(s2 / static_cast<float>(HD) + rk.eps);
  const float2 inv2 = make_float2(inv, inv);
  const float* nw = is_q ? gain : gain + HD;
  const uint4* ct = reinterpret_cast<const uint4*>(static_cast<const T*>(rk.cos_t) + meta.pos * (HD / 2));
  const uint4* st = reinterpret_cast<const uint4*>(static_cast<const T*>(rk.sin_t) + meta.pos * (HD / 2));
  if constexpr (kStaged) {  // the rows' cos | sin lines, requested at the top of the tile
    if (!mbar_wait_warp(csfull, cs_parity)) return false;
  }
  // pass 2: elements d in [32c, 32c + 32) with their partners d + 64; the
  // chunk's cos / sin lines are requested before its TMEM read, so the two
  // latencies overlap
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    uint4 cu[4], su[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if constexpr (kStaged) {
        const int o = (threadIdx.x & 31) * 128 + 16 * ((4 * c + q) ^ (threadIdx.x & 7));
        cu[q] = *reinterpret_cast<const uint4*>(cs + o);
        su[q] = *reinterpret_cast<const uint4*>(cs + 4096 + o);
      } else {
        cu[q] = ok ? __ldg(ct + c * 4 + q) : make_uint4(0, 0, 0, 0);
        su[q] = ok ? __ldg(st + c * 4 + q) : make_uint4(0, 0, 0, 0);
      }
    }
    float va[32], vb[32];
    tmem_ld2x32(tmem_col0 + c * 32, tmem_col0 + 64 + c * 32, va, vb);
    if constexpr (!kStaged) {
      if (!ok) continue;
    }  // staged: rows past M are computed (from zeros) and not stored
#pragma unroll
    for (int j0 = 0; j0 < 32; j0 += 8) {
      const int d0 = c * 32 + j0;
      const uint32_t cw[4] = {cu[j0 / 8].x, cu[j0 / 8].y, cu[j0 / 8].z, cu[j0 / 8].w};
      const uint32_t sw[4] = {su[j0 / 8].x, su[j0 / 8].y, su[j0 / 8].z, su[j0 / 8].w};
      const float4 na0 = *reinterpret_cast<const float4*>(nw + d0);
      const float4 na1 = *reinterpret_cast<const float4*>(nw + d0 + 4);
      const float4 nb0 = *reinterpret_cast<const float4*>(nw + d0 + 64);
      const float4 nb1 = *reinterpret_cast<const float4*>(nw + d0 + 68);
      const float2 ga[4] = {make_float2(na0.x, na0.y), make_float2(na0.z, na0.w),
                            make_float2(na1.x, na1.y), make_float2(na1.z, na1.w)};
      const float2 gb[4] = {make_float2(nb0.x, nb0.y), make_float2(nb0.z, nb0.w),
                            make_float2(nb1.x, nb1.y), make_float2(nb1.z, nb1.w)};
      uint32_t lo[4], hi[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int i = j0 + 2 * p;
        const float2 r = make_float2(meta.inv, meta.inv);
        const float2 xa = mul2_rn(mul2_rn(round16x2<T>(mul2_rn(make_float2(va[i], va[i + 1]), r)), inv2), ga[p]);
        const float2 xb = mul2_rn(mul2_rn(round16x2<T>(mul2_rn(make_float2(vb[i], vb[i + 1]), r)), inv2), gb[p]);
        const float2 cc = unpack2<T>(cw[p]), sn = unpack2<T>(sw[p]);
        const float2 nxb = make_float2(-xb.x, -xb.y);
        lo[p] = pack2_rn<T>(add2_rn(mul2_rn(xa, cc), mul2_rn(nxb, sn)));
        hi[p] = pack2_rn<T>(add2_rn(mul2_rn(xb, cc), mul2_rn(xa, sn)));
      }
      if constexpr (kStaged) {
        stage_unit(ost, j0 / 8, make_uint4(lo[0], lo[1], lo[2], lo[3]));
        stage_unit(ost, 4 + j0 / 8, make_uint4(hi[0], hi[1], hi[2], hi[3]));
      } else {
        *reinterpret_cast<uint4*>(dst + d0) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(dst + d0 + 64) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      }
    }
    if constexpr (kStaged) flush_rows<T>(ost, ok ? dst : nullptr, c * 32, 64 + c * 32);
  }
  return true;
}

// The epilogue warps (threads 64 .. 64 + 32 * 8 - 1 of the two GEMM kernels)
// copy the q_norm | k_norm gains into shared memory and meet at named
// barrier 1.
__device__ __forceinline__ void stage_qkv_gains(const EpiParams& ep, float* gain) {
  constexpr int kEpiThreads = 256;
  for (int e = threadIdx.x - 64; e < 256; e += kEpiThreads)
    gain[e] = e < 128 ? ep.rk.qn[e] : ep.rk.kn[e - 128];
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
}

// The fused epilogue over columns [cb, ce) of this thread's tile row (cb, ce
// multiples of 32; two epilogue warpgroups split a tile between them).  For
// SwiGLU the range is over the output columns [0, BN/2).
// Returns false only when a staged QKV epilogue's wait for its cos | sin
// lines ran out.
// kOnly: 0 = every mode, 1 = EPI_QKV_ROPE only, 2 = every mode but EPI_QKV_ROPE.
template <int BN, typename T, bool kStagedQkv = false, int kOnly = 0>
__device__ __forceinline__ bool epilogue(const EpiParams& ep, uint32_t tmem_row, int row, int M,
                                         int n0, int N, int cb, int ce, const QkvRow& meta = {},
                                         const float* gain = nullptr, uint8_t* stage = nullptr,
                                         const uint8_t* cs = nullptr, uint64_t* csfull = nullptr,
                                         uint32_t cs_parity = 0) {
  if constexpr (BN % 128 == 0 && kOnly != 2) {
    if (ep.mode == EPI_QKV_ROPE) {
#pragma unroll 1
      for (int hb = cb / 128; hb < ce / 128; ++hb)
        if (n0 + hb * 128 < N &&
            !qkv_rope_head<T, kStagedQkv>(ep, tmem_row + hb * 128, row, M, (n0 + hb * 128) / 128,
                                          meta, gain, stage, cs, csfull, cs_parity))
          return false;
      return true;
    }
  }
  if constexpr (kOnly == 1) return true;
  if (ep.mode == EPI_SWIGLU16) {
    // gate in columns [0, BN/2), up in [BN/2, BN) of this tile
    constexpr int H = BN / 2;
    T* out = static_cast<T*>(ep.out);
    if constexpr (kStagedQkv) {
      // CTA pairs: the thread's 64 output columns (one 128-byte row segment)
      // go through the warp's buffer and leave four whole segments per store
      if (stage && ce - cb == 64 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 &&
          ep.ldo % 8 == 0) {
        T* base = row < M ? out + (long long)row * ep.ldo + n0 / 2 : nullptr;
#pragma unroll 1
        for (int k = 0; k < 2; ++k) {
          float g[32], u[32];
          tmem_ld2x32(tmem_row + cb + 32 * k, tmem_row + H + cb + 32 * k, g, u);  // warp-collective
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float h2[2];
#pragma unroll
              for (int l = 0; l < 2; ++l) {
                const int i = 8 * j + 2 * e + l;
                const float gh = round16<T>(g[i] * meta.inv);
                const float uh = round16<T>(u[i] * meta.inv);
                h2[l] = __fdividef(gh, 1.0f + __expf(-gh)) * uh;
              }
              w[e] = cvt2_rn<T>(make_float2(h2[0], h2[1]));
            }
            stage_unit(stage, 4 * k + j, make_uint4(w[0], w[1], w[2], w[3]));
          }
        }
        flush_rows<T>(stage, base, cb, cb + 32);
        return true;
      }
    }
#pragma unroll 1
    for (int c0 = cb; c0 < ce; c0 += 32) {
      float g[32], u[32];
      tmem_ld2x32(tmem_row + c0, tmem_row + H + c0, g, u);
      if (row < M) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float gh = round16<T>(g[i] * meta.inv);
          const float uh = round16<T>(u[i] * meta.inv);
          const float silu = __fdividef(gh, 1.0f + __expf(-gh));
          g[i] = silu * uh;
        }
        const int oc = n0 / 2 + c0;
        const int nc = min(32, N / 2 - oc);
        if (nc > 0) store16_row<T>(out + (long long)row * ep.ldo + oc, g, nc);
      }
    }
    return true;
  }

  if (ep.mode == EPI_ARGMAX) {
    unsigned long long best = 0ull;
    float* out = static_cast<float*>(ep.out);
#pragma unroll 1
    for (int c0 = cb; c0 < ce; c0 += 32) {
      float v[32];
      tmem_ld32(tmem_row + c0, v);
      if (row < M) {
        const int nc = min(min(32, BN - c0), N - (n0 + c0));
        float* orow = out ? out + (long long)row * ep.ldo + n0 + c0 : nullptr;
        if (orow && vec_ok(orow, nc)) {
          float4* d4 = reinterpret_cast<float4*>(orow);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          orow = nullptr;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (i >= nc) continue;
          const float x = v[i];
          if (orow) orow[i] = x;
          if (x == x) {  // NaN never wins, as in a strict `>` scan
            const unsigned long long k = argmax_key(x, n0 + c0 + i);
            best = k > best ? k : best;
          }
        }
      }
    }
    if (row < M && best != 0ull) atomicMax(ep.keys + row, best);
    return true;
  }

  float ssq_acc = 0.0f;  // EPI_RESID16 with ssq_out: the current 128-column block
  // one 32-column chunk: bias, then the mode's operation
  auto chunk = [&](int c0, float (&v)[32]) {
    if (row >= M) return;
    const int col = n0 + c0;
    const int nc = min(min(32, BN - c0), N - col);  // BN need not be a multiple of 32
    if (nc <= 0) return;
    if (ep.bias) {
      const float* bp = ep.bias + col;
      if (vec_ok(bp, nc)) {
        const float4* b4 = reinterpret_cast<const float4*>(bp);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 t = __ldg(b4 + i);
          v[4 * i] += t.x;
          v[4 * i + 1] += t.y;
          v[4 * i + 2] += t.z;
          v[4 * i + 3] += t.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < nc) v[i] += bp[i];
      }
    }
    switch (ep.mode) {
      case EPI_STORE16: {
        if (ep.act == ACT_GELU) {  // the tower's GELU (conv2/conv3, fc1, proj1)
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 g = gelu_as2(make_float2(v[i], v[i + 1]));
            v[i] = g.x;
            v[i + 1] = g.y;
          }
        }
        int orow = row;
        if (ep.row_map) orow = ep.row_map[row];
        if (orow >= 0) store16_row<T>(static_cast<T*>(ep.out) + (long long)orow * ep.ldo + col, v, nc);
        break;
      }
      case EPI_RESID16: {
        T* dst = static_cast<T*>(ep.out) + (long long)row * ep.ldo + col;
        float h[32];
        load16_row<T>(dst, h, nc);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += h[i];
        store16_row<T>(dst, v, nc);
        if (ep.ssq_out) {  // the 128-column block's sum of squares of the stored values
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float x = i < nc ? round16<T>(v[i]) : 0.0f;
            ssq_acc = fmaf(x, x, ssq_acc);
          }
          if ((col + 32) % kSsqCols == 0 || col + 32 >= N) {
            ep.ssq_out[static_cast<long long>(row) * ep.ssq_n + col / kSsqCols] = ssq_acc;
            ssq_acc = 0.0f;
          }
        }
        break;
      }
      case EPI_RESID32: {
        float* dst = static_cast<float*>(ep.out) + (long long)row * ep.ldo + col;
        if (vec_ok(dst, nc)) {
          float4* d4 = reinterpret_cast<float4*>(dst);
          float4 h[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) h[i] = d4[i];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            d4[i] = make_float4(h[i].x + v[4 * i], h[i].y + v[4 * i + 1], h[i].z + v[4 * i + 2],
                                h[i].w + v[4 * i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < nc) dst[i] += v[i];
        }
        break;
      }
      case EPI_STORE32: {
        const int orow = out_row(ep, row);
        if (orow < 0) break;
        if (ep.pe) {
          const float* pe = ep.pe + (long long)(row % ep.pe_period) * N + col;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < nc) v[i] += pe[i];
        }
        float* dst = static_cast<float*>(ep.out) + (long long)orow * ep.ldo + col;
        if (vec_ok(dst, nc)) {
          float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < nc) dst[i] = v[i];
        }
        break;
      }
      case EPI_SPLIT3: {
        const int orow = out_row(ep, row);
        if (orow < 0) break;
        if (ep.act == ACT_GELU) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
        }
        if (ep.out2) {
          float* dst = ep.out2 + (long long)orow * ep.ldo2 + col;
          if (vec_ok(dst, nc)) {
            float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < nc) dst[i] = v[i];
          }
        }
        float lo[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float hi = h2f<T>(f2h<T>(v[i]));
          lo[i] = v[i] - hi;
          v[i] = hi;
        }
        T* base = static_cast<T*>(ep.out) + (long long)orow * ep.ldo + col;
        store16_row<T>(base, v, nc);
        store16_row<T>(base + N, lo, nc);
        store16_row<T>(base + 2 * N, v, nc);
        break;
      }
      default:
        break;
    }
  };
  if constexpr (kStagedQkv) {
    // EPI_STORE16 on CTA pairs (N a multiple of BN): each 64-column block of
    // the warp's 32 rows is staged in the warp's buffer and stored four whole
    // rows per instruction, instead of 16 bytes from each of 32 rows
    if (ep.mode == EPI_STORE16 && stage && (reinterpret_cast<uintptr_t>(ep.out) & 15u) == 0 &&
        ep.ldo % 8 == 0 && (reinterpret_cast<uintptr_t>(ep.bias) & 15u) == 0 && N % BN == 0) {
      int orow = row;
      if (ep.row_map && row < M) orow = ep.row_map[row];
      T* base = (row < M && orow >= 0) ? static_cast<T*>(ep.out) + (long long)orow * ep.ldo + n0
                                       : nullptr;
#pragma unroll 1
      for (int c0 = cb; c0 < ce; c0 += 64) {
        const bool two = c0 + 32 < ce;
        // whole 16-byte units inside the tile (BN = 240: the last chunk has 2)
        const int nv = two ? 4 + min(32, BN - c0 - 32) / 8 : min(32, BN - c0) / 8;
#pragma unroll 1
        for (int h = 0; h < (two ? 2 : 1); ++h) {
          float x[32];
          tmem_ld32(tmem_row + c0 + 32 * h, x);  // warp-collective (h's bound is warp-uniform)
          if (ep.bias) {
            const float4* b4 = reinterpret_cast<const float4*>(ep.bias + n0 + c0 + 32 * h);
            const int nb = min(32, BN - c0 - 32 * h) / 4;  // bias entries inside the tile
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 t = i < nb ? __ldg(b4 + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
              x[4 * i] += t.x;
              x[4 * i + 1] += t.y;
              x[4 * i + 2] += t.z;
              x[4 * i + 3] += t.w;
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t u[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              float2 g = make_float2(x[8 * j + 2 * k], x[8 * j + 2 * k + 1]);
              if (ep.act == ACT_GELU) g = gelu_as2(g);
              u[k] = cvt2_rn<T>(g);
            }
            stage_unit(stage, 4 * h + j, make_uint4(u[0], u[1], u[2], u[3]));
          }
        }
        flush_rows<T>(stage, base, c0, c0 + 32, nv);
      }
      return true;
    }
  }
  // chunks are read from TMEM two at a time behind one wait
#pragma unroll 1
  for (int c0 = cb; c0 < ce; c0 += 64) {
    float v[32], w[32];
    if (c0 + 32 < ce) {
      tmem_ld2x32(tmem_row + c0, tmem_row + c0 + 32, v, w);
      chunk(c0, v);
      chunk(c0 + 32, w);
    } else {
      tmem_ld32(tmem_row + c0, v);
      chunk(c0, v);
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// EPI_RESID32 / EPI_RESID16 with the residual staged in shared memory.  An
// epilogue thread owns one row, so reading the residual straight from global
// memory puts 32 rows (32 lines) behind every warp load and leaves the
// epilogue waiting on memory latency for each 32-column chunk.  Here each
// epilogue warp has a 4 KB buffer: the 32 rows x 32 columns of residual for
// its next chunk are copied in by coalesced 16-byte cp.async (four or eight
// whole rows per instruction) while the current chunk is processed, and the
// tile's first chunk is requested before the tile's accumulator wait.  The
// buffer is XOR-swizzled in 16-byte units so that both the copies and the
// row-per-thread reads are free of bank conflicts.
constexpr int kEpiStageBytes = 4096;  // per epilogue warp

// Whether the staged path applies (warp-uniform): a residual mode with 16-byte
// aligned rows and whole 16-byte units at the row ends.
template <typename T>
__device__ __forceinline__ bool resid_stageable(const EpiParams& ep, int N) {
  if (ep.mode != EPI_RESID32 && ep.mode != EPI_RESID16) return false;
  const int per16 = ep.mode == EPI_RESID32 ? 4 : 16 / static_cast<int>(sizeof(T));
  return (reinterpret_cast<uintptr_t>(ep.out) & 15u) == 0 && ep.ldo % per16 == 0 && N % per16 == 0;
}

// Request the residual of rows row0 .. row0 + 31, columns col .. col + 31,
// into the warp's buffer (rows past M and columns past N arrive as zeros).
template <typename T>
__device__ __forceinline__ void resid_issue(const EpiParams& ep, uint8_t* buf, int row0, int col,
                                            int M, int N) {
  const int lane = threadIdx.x & 31;
  const uint32_t sb = smem_u32(buf);
  if (ep.mode == EPI_RESID32) {
    const float* src0 = static_cast<const float*>(ep.out);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = 4 * i + (lane >> 3), q = lane & 7;  // 128-byte rows, 8 units
      const int grow = row0 + r, gcol = col + 4 * q;
      const bool ok = grow < M && gcol < N;
      const float* src = src0 + (ok ? static_cast<long long>(grow) * ep.ldo + gcol : 0);
      cp_async16(sb + r * 128 + 16 * (q ^ (r & 7)), src, ok ? 16u : 0u);
    }
  } else {
    const T* src0 = static_cast<const T*>(ep.out);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 8 * i + (lane >> 2), q = lane & 3;  // 64-byte rows, 4 units
      const int grow = row0 + r, gcol = col + 8 * q;
      const bool ok = grow < M && gcol < N;
      const T* src = src0 + (ok ? static_cast<long long>(grow) * ep.ldo + gcol : 0);
      cp_async16(sb + r * 64 + 16 * (q ^ ((r >> 1) & 3)), src, ok ? 16u : 0u);
    }
  }
  cp_async_commit();
}

// The staged epilogue over columns [cb, ce) of the warp's 32 tile rows from
// row0.  The chunk at cb must already be requested; the last chunk requests
// the first chunk of the warp's next tile (rows nxt_row0, columns from
// nxt_n0 + cb) when nxt_n0 >= 0.  Same arithmetic as the direct path: bias,
// then the residual, rounded once at the store.
// kOut (CTA pairs: N a multiple of BN, whole 32-column chunks, 16-byte
// aligned bias): the results also leave through a second 4 KB buffer, four
// whole row segments per store instruction.
template <int BN, typename T, bool kOut = false>
__device__ __forceinline__ void epilogue_resid_staged(const EpiParams& ep, uint32_t tmem_row,
                                                      int row0, int M, int n0, int N, int cb,
                                                      int ce, uint8_t* buf, int nxt_row0,
                                                      int nxt_n0, uint8_t* obuf = nullptr) {
  const int lane = threadIdx.x & 31;
  const int row = row0 + lane;
  float ssq_acc = 0.0f;
#pragma unroll 1
  for (int c0 = cb; c0 < ce; c0 += 32) {
    cp_async_wait_all();
    __syncwarp();
    float h[32];
    if (ep.mode == EPI_RESID32) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 t = *reinterpret_cast<const float4*>(buf + lane * 128 + 16 * (j ^ (lane & 7)));
        h[4 * j] = t.x;
        h[4 * j + 1] = t.y;
        h[4 * j + 2] = t.z;
        h[4 * j + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 t = *reinterpret_cast<const uint4*>(buf + lane * 64 + 16 * (j ^ ((lane >> 1) & 3)));
        const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack2<T>(w[k]);
          h[8 * j + 2 * k] = f.x;
          h[8 * j + 2 * k + 1] = f.y;
        }
      }
    }
    __syncwarp();  // every lane has read the buffer before it is refilled
    const bool more = c0 + 32 < ce;
    if (more || nxt_n0 >= 0)
      resid_issue<T>(ep, buf, more ? row0 : nxt_row0, more ? n0 + c0 + 32 : nxt_n0 + cb, M, N);
    float v[32];
    tmem_ld32(tmem_row + c0, v);  // warp-collective: every lane, every chunk
    const int col = n0 + c0;
    if constexpr (kOut) {
      // every lane computes (rows past M from their zero rows); only live
      // rows are stored
      const bool live = row < M;
      if (ep.bias) {
        const float4* b4 = reinterpret_cast<const float4*>(ep.bias + col);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 t = __ldg(b4 + i);
          v[4 * i] += t.x;
          v[4 * i + 1] += t.y;
          v[4 * i + 2] += t.z;
          v[4 * i + 3] += t.w;
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += h[i];
      if (ep.mode == EPI_RESID32) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          stage_unit(obuf, j, make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                                         __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3])));
        flush_rows<float>(obuf, live ? static_cast<float*>(ep.out) + static_cast<long long>(row) * ep.ldo : nullptr,
                          col, col + 16, 8);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) w[k] = cvt2_rn<T>(make_float2(v[8 * j + 2 * k], v[8 * j + 2 * k + 1]));
          stage_unit(obuf, j, make_uint4(w[0], w[1], w[2], w[3]));
        }
        flush_rows<T>(obuf, live ? static_cast<T*>(ep.out) + static_cast<long long>(row) * ep.ldo : nullptr,
                      col, col, 4);
        if (ep.ssq_out && live) {  // the 128-column block's sum of squares of the stored values
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float x = round16<T>(v[i]);
            ssq_acc = fmaf(x, x, ssq_acc);
          }
          if ((col + 32) % kSsqCols == 0 || col + 32 >= N) {
            ep.ssq_out[static_cast<long long>(row) * ep.ssq_n + col / kSsqCols] = ssq_acc;
            ssq_acc = 0.0f;
          }
        }
      }
      continue;
    }
    const int nc = min(min(32, BN - c0), N - col);
    if (row >= M || nc <= 0) continue;
    if (ep.bias) {
      const float* bp = ep.bias + col;
      if (vec_ok(bp, nc)) {
        const float4* b4 = reinterpret_cast<const float4*>(bp);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 t = __ldg(b4 + i);
          v[4 * i] += t.x;
          v[4 * i + 1] += t.y;
          v[4 * i + 2] += t.z;
          v[4 * i + 3] += t.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < nc) v[i] += bp[i];
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += h[i];
    if (ep.mode == EPI_RESID32) {
      float* dst = static_cast<float*>(ep.out) + static_cast<long long>(row) * ep.ldo + col;
      if (vec_ok(dst, nc)) {
        float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < nc) dst[i] = v[i];
      }
    } else {
      T* dst = static_cast<T*>(ep.out) + static_cast<long long>(row) * ep.ldo + col;
      store16_row<T>(dst, v, nc);
      if (ep.ssq_out) {  // the 128-column block's sum of squares of the stored values
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float x = i < nc ? round16<T>(v[i]) : 0.0f;
          ssq_acc = fmaf(x, x, ssq_acc);
        }
        if ((col + 32) % kSsqCols == 0 || col + 32 >= N) {
          ep.ssq_out[static_cast<long long>(row) * ep.ssq_n + col / kSsqCols] = ssq_acc;
          ssq_acc = 0.0f;
        }
      }
    }
  }
}

// Column range of epilogue warpgroup `wg` out of `nwg` for a BN-wide tile.
template <int BN>
__device__ __forceinline__ void epi_range(int mode, int wg, int nwg, int& cb, int& ce) {
  const int span = mode == EPI_SWIGLU16 ? BN / 2 : BN;
  if (nwg == 1) {
    cb = 0;
    ce = span;
    return;
  }
  const int chunks = (span + 31) / 32;
  const int split = ((chunks + 1) / 2) * 32;
  cb = wg == 0 ? 0 : split;
  ce = wg == 0 ? split : chunks * 32;
}

// Persistent kernel: gridDim.x CTAs (at most one per SM) walk the tile list
// t = blockIdx.x, blockIdx.x + gridDim.x, ... with tiles numbered N-fastest so
// that the CTAs in flight share A row-blocks and the whole B operand stays in
// L2.  The accumulator is double-buffered in TMEM (2 x BN columns): the MMA
// warp starts tile i+1 while the epilogue warps drain tile i.
constexpr int kGemmEpiWarps = 8;                          // two warpgroups
constexpr int kGemmThreads = (2 + kGemmEpiWarps) * 32;     // TMA, MMA, epilogue

template <int BN, typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   int M, int N, int K, EpiParams ep) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  constexpr uint32_t kAccCols = Cfg::kTmemCols;      // columns per accumulator buffer
  constexpr uint32_t kAllocCols = 2 * Cfg::kTmemCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;   // [2] accumulator ready for the epilogue
  uint64_t* tempty = tfull + 2;  // [2] accumulator drained by the epilogue
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nkb = (K + kBK - 1) / kBK;
  const int n_tiles_n = (N + BN - 1) / BN;
  const int n_tiles = n_tiles_n * ((M + kBM - 1) / kBM);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 32 * kGemmEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tslot, kAllocCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();

  auto timed_out = [&]() {
    *abort_flag = 1;
    if (ep.status) atomicOr(ep.status, kStatusTimeout);
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t c = 0;  // k-blocks issued so far (ring position)
      for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += gridDim.x) {
        const int m0 = (t / n_tiles_n) * kBM, n0 = (t % n_tiles_n) * BN;
        for (int kb = 0; kb < nkb; ++kb, ++c) {
          const int s = c % S;
          const uint32_t ph = (c / S) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1u)) {
            timed_out();
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::kABytes + Cfg::kBBytes);
          if (ep.conv_kb > 0)  // implicit conv: tap kb / conv_kb shifts the A rows
            tma_load_2d(&tmA, &full[s], sA + s * Cfg::kABytes, (kb % ep.conv_kb) * kBK,
                        m0 + kb / ep.conv_kb);
          else
            tma_load_2d(&tmA, &full[s], sA + s * Cfg::kABytes, kb * kBK, m0);
          tma_load_2d(&tmB, &full[s], sB + s * Cfg::kBBytes, kb * kBK, n0);
        }
      }
    }
  } else if (warp == 1) {
    {  // the whole warp; one elected lane issues
      constexpr uint32_t idesc = f16_instr_desc(kBM, BN, H16Traits<T>::kBf16);
      uint32_t c = 0;
      int lt = 0;  // tiles done by this CTA
      for (int t = blockIdx.x; t < n_tiles && !__any_sync(0xFFFFFFFFu, *abort_flag != 0); t += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait_warp(&tempty[buf], ((lt >> 1) & 1) ^ 1u)) {
          timed_out();
          break;
        }
        tc_fence_after();
        const uint32_t acc = tbase + buf * kAccCols;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++c) {
          const int s = c % S;
          const uint32_t ph = (c / S) & 1;
          if (!mbar_wait_warp(&full[s], ph)) {
            timed_out();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(sB + s * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t da = sw128_kmajor_desc(a_addr + k * 32);
            const uint64_t db = sw128_kmajor_desc(b_addr + k * 32);
            mma_f16_e(acc, da, db, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit_e(&empty[s]);
        }
        if (!ok) break;
        mma_commit_e(&tfull[buf]);
      }
    }
  } else {
    const int q = warp & 3;              // TMEM lane quarter this warp may read
    const int wg = (warp - 2) / 4;       // column half of the tile
    int cb, ce;
    epi_range<BN>(ep.mode, wg, kGemmEpiWarps / 4, cb, ce);
    __shared__ float gain[256];  // EPI_QKV_ROPE: q_norm | k_norm gains
    if (ep.mode == EPI_QKV_ROPE) stage_qkv_gains(ep, gain);
    int lt = 0;
    // the row's folded-norm statistics are loaded one tile ahead
    auto tile_row = [&](int t) { return (t / n_tiles_n) * kBM + q * 32 + lane; };
    SsqRow ssq = ssq_load(ep, tile_row(blockIdx.x), M);
    if (resid_stageable<T>(ep, N)) {
      // residual modes: the warp's staging buffer, the first tile's first
      // chunk requested before the first accumulator wait
      uint8_t* stage = smem + S * (Cfg::kABytes + Cfg::kBBytes) + 256 + (warp - 2) * kEpiStageBytes;
      auto warp_row0 = [&](int t) { return (t / n_tiles_n) * kBM + q * 32; };
      if (static_cast<int>(blockIdx.x) < n_tiles)
        resid_issue<T>(ep, stage, warp_row0(blockIdx.x), (blockIdx.x % n_tiles_n) * BN + cb, M, N);
      for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (*abort_flag || !mbar_wait(&tfull[buf], (lt >> 1) & 1)) {
          if (lane == 0) timed_out();
          break;
        }
        tc_fence_after();
        const uint32_t trow = tbase + buf * kAccCols + (static_cast<uint32_t>(q * 32) << 16);
        const int tn = t + gridDim.x;
        epilogue_resid_staged<BN, T>(ep, trow, warp_row0(t), M, (t % n_tiles_n) * BN, N, cb, ce,
                                     stage, tn < n_tiles ? warp_row0(tn) : 0,
                                     tn < n_tiles ? (tn % n_tiles_n) * BN : -1);
        tc_fence_before();
        mbar_arrive(&tempty[buf]);
      }
      cp_async_wait_all();  // nothing in flight into shared memory at exit
    } else {
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++lt) {
      const int buf = lt & 1;
      const int m0 = (t / n_tiles_n) * kBM, n0 = (t % n_tiles_n) * BN;
      const int row = m0 + q * 32 + lane;
      QkvRow meta;
      if (ep.mode == EPI_QKV_ROPE) meta = qkv_row_meta<T>(ep, row, M);  // before the wait
      meta.inv = row_rms_inv(ep, ssq);
      if (*abort_flag || !mbar_wait(&tfull[buf], (lt >> 1) & 1)) {
        if (lane == 0) timed_out();
        break;
      }
      ssq = ssq_load(ep, tile_row(t + gridDim.x), M);  // arrives during this epilogue
      tc_fence_after();
      const uint32_t trow = tbase + buf * kAccCols + (static_cast<uint32_t>(q * 32) << 16);
      epilogue<BN, T>(ep, trow, row, M, n0, N, cb, ce, meta, gain);
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kAllocCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair version (tcgen05 cta_group::2) for 256 x 256 output tiles: the two
// CTAs of a cluster run on neighbouring SMs; each TMA-loads its own 128 rows
// of A and its own 128 rows (output columns) of B per k-block, the first CTA
// issues M=256, N=256 MMAs that read both CTAs' shared memory, and each CTA
// holds its 128 accumulator rows (all 256 columns) in its own TMEM, drained by
// its own epilogue warps.  Per SM this moves half the B bytes of a 128 x 256
// tile for the same MMA work, which takes the operand stream from about three
// quarters of the L2-to-SM bandwidth down to one half.
//   full[s]    (first CTA) both CTAs' A and B halves of stage s landed;
//   empty[s]   (each CTA, by multicast commit) stage s may be refilled;
//   tfull[b]   (each CTA, by multicast commit) accumulator b complete;
//   tempty[b]  (first CTA) both CTAs' epilogues drained accumulator b
//              (one remote arrival per epilogue warp, 16 in all).
// BN (256 or 224) is the pair tile's width: each CTA loads BN/2 rows of B.
constexpr int kPairStages = 6;
constexpr uint32_t kPairHalf = kBM * kBK * 2;  // 16 KB: 128 rows x 64 k of A
template <int BN>
struct PairCfg {
  static constexpr uint32_t kBHalf = (BN / 2) * kBK * 2;  // BN/2 rows x 64 k of B
  static constexpr size_t kSmem = 1024 + kPairStages * (kPairHalf + kBHalf) + 256;
};

// kVar: 1 = the EPI_QKV_ROPE instantiation (its epilogue only), 2 = the
// residual modes' (EPI_RESID16 / EPI_RESID32), 0 = every other mode.  Separate
// instantiations keep each epilogue's registers apart; 1 and 2 run one ring
// stage fewer and stage 64 KB of epilogue data instead of 32 KB.
template <int BN, typename T, int kVar>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     int M, int N, int K, EpiParams ep) {
  // EPI_QKV_ROPE gives one ring stage to the epilogue's cos | sin staging
  constexpr bool kQkv = kVar == 1;
  constexpr int S = kVar ? kPairStages - 1 : kPairStages;
  constexpr uint32_t kBHalf = PairCfg<BN>::kBHalf;
  constexpr uint32_t kAccCols = 256;
  constexpr uint32_t kAllocCols = 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kPairHalf;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * kBHalf);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* csfull = tempty + 2;   // [4] EPI_QKV_ROPE: a lane quarter's cos | sin lines landed
  uint64_t* csempty = csfull + 4;  // [4] ... and were read by both of its warps
  uint32_t* tslot = reinterpret_cast<uint32_t*>(csempty + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  uint8_t* epi_smem = smem + S * (kPairHalf + kBHalf) + 256;  // epilogue staging buffers

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int nkb = (K + kBK - 1) / kBK;
  const int n_tiles_n = N / BN;
  const int n_tiles = n_tiles_n * ((M + 2 * kBM - 1) / (2 * kBM));

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * kGemmEpiWarps);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&csfull[i], 64);  // both warps' lanes, as their copies land
      mbar_init(&csempty[i], 2);  // one arrival per warp
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(tslot, kAllocCols);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();

  auto timed_out = [&]() {
    *abort_flag = 1;
    if (ep.status) atomicOr(ep.status, kStatusTimeout);
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full_lead = mapa_shared(smem_u32(full), 0);
      int s = 0;        // ring slot and its phase, advanced per k-block
      uint32_t ph = 0;  // (S is a runtime value here: no division per k-block)
      for (int t = pair; t < n_tiles && !*abort_flag; t += n_pairs) {
        const int m0 = (t / n_tiles_n) * 2 * kBM, n0 = (t % n_tiles_n) * BN;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, s = (s + 1 == S) ? 0 : s + 1, ph ^= (s == 0)) {
          if (!mbar_wait(&empty[s], ph ^ 1u)) {
            timed_out();
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (kPairHalf + kBHalf));  // both CTAs
          const uint32_t bar = full_lead + s * 8;
          tma_load_2d_pair(&tmA, bar, sA + s * kPairHalf, kb * kBK, m0 + rank * kBM);
          tma_load_2d_pair(&tmB, bar, sB + s * kBHalf, kb * kBK, n0 + rank * (BN / 2));
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {  // the whole warp; one elected lane issues
      constexpr uint32_t idesc = f16_instr_desc(2 * kBM, BN, H16Traits<T>::kBf16);
      int s = 0;        // ring slot and its phase, advanced per k-block
      uint32_t ph = 0;
      int lt = 0;
      for (int t = pair; t < n_tiles && !__any_sync(0xFFFFFFFFu, *abort_flag != 0); t += n_pairs, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait_cluster_warp(&tempty[buf], ((lt >> 1) & 1) ^ 1u)) {
          timed_out();
          break;
        }
        tc_fence_after();
        const uint32_t acc = tbase + buf * kAccCols;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, s = (s + 1 == S) ? 0 : s + 1, ph ^= (s == 0)) {
          if (!mbar_wait_warp(&full[s], ph)) {
            timed_out();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * kPairHalf);
          const uint32_t b_addr = smem_u32(sB + s * kBHalf);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_f16_pair_e(acc, sw128_kmajor_desc(a_addr + k * 32), sw128_kmajor_desc(b_addr + k * 32),
                         idesc, (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit_pair_e(&empty[s], 0x3);
        }
        if (!ok) break;
        mma_commit_pair_e(&tfull[buf], 0x3);
      }
    }
  } else {
    const int q = warp & 3;
    const int wg = (warp - 2) / 4;
    int cb, ce;
    epi_range<BN>(ep.mode, wg, kGemmEpiWarps / 4, cb, ce);
    const uint32_t tempty_lead = mapa_shared(smem_u32(tempty), 0);
    __shared__ float gain[256];  // EPI_QKV_ROPE: q_norm | k_norm gains
    if (ep.mode == EPI_QKV_ROPE) stage_qkv_gains(ep, gain);
    int lt = 0;
    // the row's folded-norm statistics are loaded one tile ahead
    auto tile_row = [&](int t) { return (t / n_tiles_n) * 2 * kBM + rank * kBM + q * 32 + lane; };
    SsqRow ssq = ssq_load(ep, tile_row(pair), M);
    if (kVar == 2 && resid_stageable<T>(ep, N) &&
        (reinterpret_cast<uintptr_t>(ep.bias) & 15u) == 0) {
      // residual modes: the warp's staging buffer, the first tile's first
      // chunk requested before the first accumulator wait
      uint8_t* stage = epi_smem + (warp - 2) * kEpiStageBytes;
      uint8_t* ostage = stage + kGemmEpiWarps * kEpiStageBytes;  // the results
      auto warp_row0 = [&](int t) { return (t / n_tiles_n) * 2 * kBM + rank * kBM + q * 32; };
      if (pair < n_tiles)
        resid_issue<T>(ep, stage, warp_row0(pair), (pair % n_tiles_n) * BN + cb, M, N);
      for (int t = pair; t < n_tiles; t += n_pairs, ++lt) {
        const int buf = lt & 1;
        if (*abort_flag || !mbar_wait(&tfull[buf], (lt >> 1) & 1)) {
          if (lane == 0) timed_out();
          break;
        }
        tc_fence_after();
        const uint32_t trow = tbase + buf * kAccCols + (static_cast<uint32_t>(q * 32) << 16);
        const int tn = t + n_pairs;
        epilogue_resid_staged<BN, T, true>(ep, trow, warp_row0(t), M, (t % n_tiles_n) * BN, N, cb,
                                           ce, stage, tn < n_tiles ? warp_row0(tn) : 0,
                                           tn < n_tiles ? (tn % n_tiles_n) * BN : -1, ostage);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote_relaxed(tempty_lead + buf * 8);
      }
      cp_async_wait_all();  // nothing in flight into shared memory at exit
    } else {
    // EPI_QKV_ROPE: the warp's buffer stages each head's rows for coalesced
    // stores; the two warps of a TMEM lane quarter (one per column half)
    // share the cos | sin lines of their 32 rows, each warp copying one table
    constexpr bool qkv = kQkv;
    uint8_t* qstage = (qkv || ep.mode == EPI_STORE16 || ep.mode == EPI_SWIGLU16)
                          ? epi_smem + (warp - 2) * kEpiStageBytes
                          : nullptr;
    uint8_t* cs = qkv ? epi_smem + kGemmEpiWarps * kEpiStageBytes + q * 8192 : nullptr;
    for (int t = pair; t < n_tiles; t += n_pairs, ++lt) {
      const int buf = lt & 1;
      const int m0 = (t / n_tiles_n) * 2 * kBM, n0 = (t % n_tiles_n) * BN;
      const int row = m0 + rank * kBM + q * 32 + lane;
      QkvRow meta;
      if (qkv) {
        meta = qkv_row_meta<T, false>(ep, row, M);  // before the wait
        // both warps have read the previous tile's lines; request this tile's
        if (lt > 0 && !mbar_wait_warp(&csempty[q], (lt - 1) & 1)) {
          if (lane == 0) timed_out();
          break;
        }
        qkv_cs_issue<T>(ep, cs + wg * 4096, wg, meta.pos, row < M);
        cp_async_mbar_arrive_noinc(&csfull[q]);
      }
      meta.inv = row_rms_inv(ep, ssq);
      if (*abort_flag || !mbar_wait(&tfull[buf], (lt >> 1) & 1)) {
        if (lane == 0) timed_out();
        break;
      }
      ssq = ssq_load(ep, tile_row(t + n_pairs), M);  // arrives during this epilogue
      tc_fence_after();
      const uint32_t trow = tbase + buf * kAccCols + (static_cast<uint32_t>(q * 32) << 16);
      const bool ep_ok = epilogue<BN, T, true, kQkv ? 1 : 2>(ep, trow, row, M, n0, N, cb, ce, meta, gain,
                                                            qstage, cs, &csfull[q], lt & 1);
      tc_fence_before();
      __syncwarp();
      if (!ep_ok) {
        if (lane == 0) timed_out();
        break;
      }
      if (lane == 0) {
        mbar_arrive_remote_relaxed(tempty_lead + buf * 8);
        if (qkv) mbar_arrive(&csempty[q]);
      }
    }
    if (qkv) cp_async_wait_all();  // nothing in flight into shared memory at exit
    }
  }

  tc_fence_before();
  cluster_sync();  // neither CTA leaves while the other may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, kAllocCols);
  }
}

// ---------------------------------------------------------------------------
// 3x3 / stride 2 / pad 1 convolution as a persistent GEMM whose A operand is
// loaded by TMA straight from the NHWC activations: an M tile is R whole
// output rows of one image (R = floor(128 / wo)), and the k-block for tap
// (kh, kw) and channels [cb, cb + 32) is ONE 4-D box of the input viewed as
// [n][h][w][c] with traversal strides (1, 2, 2, 1): wo pixels along w from
// kw - 1 and R rows along h from 2*oh0 + kh - 1, 32 channels each (64-byte
// rows, 64-byte swizzle).  Padding pixels (coordinate -1 or past the edge)
// arrive as zeros from the TMA unit.  The box fills tile rows m = r*wo + c;
// rows past R*wo (and rows past the image's last output row) are computed
// from stale shared memory and never stored.  Same warp roles, TMEM
// double-buffering and epilogue as gemm_tc_kernel.
constexpr int kCvBK = 32;  // k-block: 32 channels of one tap

template <int BN>
struct ConvCfg {
  static constexpr int kStages = 8;
  static constexpr uint32_t kABytes = kBM * kCvBK * 2;  // 8 KB (the box fills R*wo rows)
  static constexpr uint32_t kBBytes = BN * kCvBK * 2;
  static constexpr uint32_t kTmemCols = GemmCfg<BN>::kTmemCols;
  static constexpr size_t kSmem = 1024 + kStages * (kABytes + kBBytes) + 256;
};

struct ConvTiles {
  int ho, wo, c;       // output geometry, input channels
  int rows;            // output rows per tile (R)
  int tiles_per_img;   // ceil(ho / R)
  int n_mtiles;        // images x tiles_per_img
  int time_major;      // output positions ordered (ow, oh) instead of (oh, ow)
  uint32_t a_bytes;    // bytes one A box delivers: R * wo * 64
};

template <int BN, typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    conv_tma_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmB,
                    ConvTiles g, int N, int K, EpiParams ep) {
  using Cfg = ConvCfg<BN>;
  constexpr int S = Cfg::kStages;
  constexpr uint32_t kAccCols = Cfg::kTmemCols;
  constexpr uint32_t kAllocCols = 2 * Cfg::kTmemCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nkb = K / kCvBK;
  const int n_tiles_n = (N + BN - 1) / BN;
  const int n_tiles = n_tiles_n * g.n_mtiles;
  const int M = g.n_mtiles / g.tiles_per_img * g.ho * g.wo;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 32 * kGemmEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tslot, kAllocCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();

  auto timed_out = [&]() {
    *abort_flag = 1;
    if (ep.status) atomicOr(ep.status, kStatusTimeout);
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t c = 0;
      for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += gridDim.x) {
        const int mt = t / n_tiles_n, n0 = (t % n_tiles_n) * BN;
        const int img = mt / g.tiles_per_img;
        const int oh0 = (mt % g.tiles_per_img) * g.rows;
        for (int kb = 0; kb < nkb; ++kb, ++c) {
          const int s = c % S;
          const uint32_t ph = (c / S) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1u)) {
            timed_out();
            break;
          }
          const int k0 = kb * kCvBK;
          const int tap = k0 / g.c, cb = k0 - tap * g.c;
          const int kh = tap / 3, kw = tap - kh * 3;
          mbar_arrive_expect_tx(&full[s], g.a_bytes + Cfg::kBBytes);
          tma_load_4d(&tmX, &full[s], sA + s * Cfg::kABytes, cb, kw - 1, 2 * oh0 + kh - 1, img);
          tma_load_2d(&tmB, &full[s], sB + s * Cfg::kBBytes, k0, n0);
        }
      }
    }
  } else if (warp == 1) {
    {  // the whole warp; one elected lane issues
      constexpr uint32_t idesc = f16_instr_desc(kBM, BN, H16Traits<T>::kBf16);
      uint32_t c = 0;
      int lt = 0;
      for (int t = blockIdx.x; t < n_tiles && !__any_sync(0xFFFFFFFFu, *abort_flag != 0); t += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait_warp(&tempty[buf], ((lt >> 1) & 1) ^ 1u)) {
          timed_out();
          break;
        }
        tc_fence_after();
        const uint32_t acc = tbase + buf * kAccCols;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++c) {
          const int s = c % S;
          const uint32_t ph = (c / S) & 1;
          if (!mbar_wait_warp(&full[s], ph)) {
            timed_out();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(sB + s * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kCvBK / 16; ++k)
            mma_f16_e(acc, sw64_kmajor_desc(a_addr + k * 32), sw64_kmajor_desc(b_addr + k * 32),
                    idesc, (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit_e(&empty[s]);
        }
        if (!ok) break;
        mma_commit_e(&tfull[buf]);
      }
    }
  } else {
    const int q = warp & 3;
    const int wg = (warp - 2) / 4;
    int cb, ce;
    epi_range<BN>(ep.mode, wg, kGemmEpiWarps / 4, cb, ce);
    int lt = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++lt) {
      const int buf = lt & 1;
      if (*abort_flag || !mbar_wait(&tfull[buf], (lt >> 1) & 1)) {
        if (lane == 0) timed_out();
        break;
      }
      tc_fence_after();
      const int mt = t / n_tiles_n, n0 = (t % n_tiles_n) * BN;
      const int img = mt / g.tiles_per_img;
      const int oh0 = (mt % g.tiles_per_img) * g.rows;
      const int m = q * 32 + lane;
      const int oh = oh0 + m / g.wo, ow = m % g.wo;
      const bool valid = m < g.rows * g.wo && oh < g.ho;
      const int orow = img * g.ho * g.wo + (g.time_major ? ow * g.ho + oh : oh * g.wo + ow);
      const uint32_t trow = tbase + buf * kAccCols + (static_cast<uint32_t>(q * 32) << 16);
      epilogue<BN, T>(ep, trow, valid ? orow : M, M, n0, N, cb, ce);
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kAllocCols);
  }
}

// CTA-pair version of conv_tma_kernel: the two CTAs of a cluster take two
// consecutive M tiles (R output rows each), each loads its own strided A box
// and half of B (BN/2 output channels) per k-block, and the first CTA issues
// M=256 MMAs over both (the same barrier protocol as gemm_pair_kernel).  With
// an odd number of M tiles the last pair's second CTA loads an in-range box
// and stores nothing.
// BK = 64 (128-byte rows, 128B swizzle) when the channel count allows it,
// else 32: the TMA unit's cost is per box row, so wider rows carry twice the
// MMA work per request.
template <int BN, int BK>
struct ConvPairCfg {
  static constexpr int kStages = BK == 64 ? 6 : 12;
  static constexpr uint32_t kABytes = kBM * BK * 2;
  static constexpr uint32_t kBHalf = (BN / 2) * BK * 2;  // BN/2 rows x BK k (a swizzle-atom multiple)
  static constexpr size_t kSmem = 1024 + kStages * (kABytes + kBHalf) + 256;
};

template <int BK>
__device__ __forceinline__ uint64_t conv_desc(uint32_t addr) {
  return BK == 64 ? sw128_kmajor_desc(addr) : sw64_kmajor_desc(addr);
}

template <int BN, int BK, typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    conv_pair_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmB,
                     ConvTiles g, int N, int K, EpiParams ep) {
  using Cfg = ConvPairCfg<BN, BK>;
  constexpr int S = Cfg::kStages;
  constexpr uint32_t kAccCols = 256;
  constexpr uint32_t kAllocCols = 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBHalf);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int nkb = K / BK;
  const int n_tiles_n = N / BN;
  const int n_tiles = n_tiles_n * ((g.n_mtiles + 1) / 2);
  const int M = g.n_mtiles / g.tiles_per_img * g.ho * g.wo;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * kGemmEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(tslot, kAllocCols);
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();

  auto timed_out = [&]() {
    *abort_flag = 1;
    if (ep.status) atomicOr(ep.status, kStatusTimeout);
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full_lead = mapa_shared(smem_u32(full), 0);
      uint32_t c = 0;
      for (int t = pair; t < n_tiles && !*abort_flag; t += n_pairs) {
        const int mt0 = 2 * (t / n_tiles_n) + static_cast<int>(rank);
        const int mt = mt0 < g.n_mtiles ? mt0 : 0;  // past the end: an in-range box, not stored
        const int n0 = (t % n_tiles_n) * BN;
        const int img = mt / g.tiles_per_img;
        const int oh0 = (mt % g.tiles_per_img) * g.rows;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++c) {
          const int s = c % S;
          const uint32_t ph = (c / S) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1u)) {
            timed_out();
            ok = false;
            break;
          }
          const int k0 = kb * BK;
          const int tap = k0 / g.c, cb = k0 - tap * g.c;
          const int kh = tap / 3, kw = tap - kh * 3;
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (g.a_bytes + Cfg::kBHalf));
          const uint32_t bar = full_lead + s * 8;
          tma_load_4d_pair(&tmX, bar, sA + s * Cfg::kABytes, cb, kw - 1, 2 * oh0 + kh - 1, img);
          tma_load_2d_pair(&tmB, bar, sB + s * Cfg::kBHalf, k0, n0 + static_cast<int>(rank) * (BN / 2));
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {  // the whole warp; one elected lane issues
      constexpr uint32_t idesc = f16_instr_desc(2 * kBM, BN, H16Traits<T>::kBf16);
      uint32_t c = 0;
      int lt = 0;
      for (int t = pair; t < n_tiles && !__any_sync(0xFFFFFFFFu, *abort_flag != 0); t += n_pairs, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait_cluster_warp(&tempty[buf], ((lt >> 1) & 1) ^ 1u)) {
          timed_out();
          break;
        }
        tc_fence_after();
        const uint32_t acc = tbase + buf * kAccCols;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++c) {
          const int s = c % S;
          const uint32_t ph = (c / S) & 1;
          if (!mbar_wait_warp(&full[s], ph)) {
            timed_out();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(sB + s * Cfg::kBHalf);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16_pair_e(acc, conv_desc<BK>(a_addr + k * 32), conv_desc<BK>(b_addr + k * 32), idesc,
                         (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit_pair_e(&empty[s], 0x3);
        }
        if (!ok) break;
        mma_commit_pair_e(&tfull[buf], 0x3);
      }
    }
  } else {
    const int q = warp & 3;
    const int wg = (warp - 2) / 4;
    int cb, ce;
    epi_range<BN>(ep.mode, wg, kGemmEpiWarps / 4, cb, ce);
    const uint32_t tempty_lead = mapa_shared(smem_u32(tempty), 0);
    // EPI_STORE16: the warp's buffer stages its rows for coalesced stores
    uint8_t* stage = ep.mode == EPI_STORE16
                         ? smem + S * (Cfg::kABytes + Cfg::kBHalf) + 256 + (warp - 2) * kEpiStageBytes
                         : nullptr;
    int lt = 0;
    for (int t = pair; t < n_tiles; t += n_pairs, ++lt) {
      const int buf = lt & 1;
      if (*abort_flag || !mbar_wait(&tfull[buf], (lt >> 1) & 1)) {
        if (lane == 0) timed_out();
        break;
      }
      tc_fence_after();
      const int mt = 2 * (t / n_tiles_n) + static_cast<int>(rank);
      const int n0 = (t % n_tiles_n) * BN;
      const int img = mt / g.tiles_per_img;
      const int oh0 = (mt % g.tiles_per_img) * g.rows;
      const int m = q * 32 + lane;
      const int oh = oh0 + m / g.wo, ow = m % g.wo;
      const bool valid = mt < g.n_mtiles && m < g.rows * g.wo && oh < g.ho;
      const int orow = img * g.ho * g.wo + (g.time_major ? ow * g.ho + oh : oh * g.wo + ow);
      const uint32_t trow = tbase + buf * kAccCols + (static_cast<uint32_t>(q * 32) << 16);
      epilogue<BN, T, true, 2>(ep, trow, valid ? orow : M, M, n0, N, cb, ce, {}, nullptr, stage);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote_relaxed(tempty_lead + buf * 8);
    }
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, kAllocCols);
  }
}

int num_sms() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!sms[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = v > 0 ? v : 148;
  }
  return sms[dev];
}

// ---------------------------------------------------------------------------
// Implicit-GEMM 3x3 / stride 2 / pad 1 convolution over NHWC activations.
// Same MMA warp and epilogue as gemm_tc_kernel; the A operand is not a matrix
// in memory but gathered per k-block by four producer warps: row r of the tile
// is output position m0 + r, 16-byte chunk c of the 64-wide k-block is
// channels [ic, ic + 8) of tap (kh, kw), read from input pixel
// (2*oh + kh - 1, 2*ow + kw - 1) with cp.async (zero-filled off the image) and
// written at the 128B-swizzled place TMA would have used.  Each producer
// thread keeps two k-blocks of copies in flight: after issuing block i it
// waits for block i-1, fences the async proxy and arrives on that stage's
// barrier.
// Warp roles (288 threads): 0-3 gather A (thread 0 also TMA-loads B),
// 4 MMA + TMEM, 5-8 epilogue.
struct ConvGeom {
  int h, w, c;       // input NHWC geometry (per image)
  int ho, wo;        // output geometry
  int time_major;    // output positions ordered (ow, oh) instead of (oh, ow)
};

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}

template <int BN, typename T>
__global__ void __launch_bounds__(288, 1)
    conv_gemm_kernel(const T* __restrict__ x, ConvGeom g, const __grid_constant__ CUtensorMap tmB,
                     int M, int N, int K, EpiParams ep) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  constexpr uint32_t kAccCols = Cfg::kTmemCols;
  constexpr uint32_t kAllocCols = 2 * Cfg::kTmemCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nkb = (K + kBK - 1) / kBK;
  const int n_tiles_n = (N + BN - 1) / BN;
  const int n_tiles = n_tiles_n * ((M + kBM - 1) / kBM);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 128 + 1);  // 128 gather threads + the B expect_tx arrive
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) tma_prefetch_desc(&tmB);
  if (warp == 4) tmem_alloc(tslot, kAllocCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();
  auto timed_out = [&]() {
    *abort_flag = 1;
    if (ep.status) atomicOr(ep.status, kStatusTimeout);
  };

  if (warp < 4) {
    // ---- A gather (+ B TMA from thread 0)
    const int r = threadIdx.x;  // tile row of this thread
    // k-blocks of copies a thread keeps unpublished.  1 is measured best: every
    // unpublished block is one the MMA warp cannot start, and a longer lag
    // leaves it waiting on each publish (S - 1 ran 30 % slower on conv2).
    constexpr int kLag = 1;
    uint32_t c = 0;
    int pend[S];                // stages issued but not yet published, oldest first
    int npend = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles && ok && !*abort_flag; t += gridDim.x) {
      const int m0 = (t / n_tiles_n) * kBM, n0 = (t % n_tiles_n) * BN;
      const int p = m0 + r;
      const bool row_ok = p < M;
      int img = 0, oh = 0, ow = 0;
      if (row_ok) {
        const int plane = g.ho * g.wo;
        img = p / plane;
        const int q = p - img * plane;
        if (g.time_major) {
          ow = q / g.ho;
          oh = q - ow * g.ho;
        } else {
          oh = q / g.wo;
          ow = q - oh * g.wo;
        }
      }
      const T* ximg = x + static_cast<long long>(img) * g.h * g.w * g.c;
      for (int kb = 0; kb < nkb; ++kb, ++c) {
        const int s = c % S;
        const uint32_t ph = (c / S) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1u)) {
          timed_out();
          ok = false;
          break;
        }
        if (threadIdx.x == 0) {
          mbar_arrive_expect_tx(&full[s], Cfg::kBBytes);
          tma_load_2d(&tmB, &full[s], sB + s * Cfg::kBBytes, kb * kBK, n0);
        }
        const uint32_t arow = smem_u32(sA + s * Cfg::kABytes) + r * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const int k = kb * kBK + ch * 8;
          const int tap = k / g.c;
          const int ic = k - tap * g.c;
          const int ih = 2 * oh + tap / 3 - 1, iw = 2 * ow + tap % 3 - 1;
          const bool v = row_ok && k < K && ih >= 0 && ih < g.h && iw >= 0 && iw < g.w;
          const T* src = v ? ximg + (static_cast<long long>(ih) * g.w + iw) * g.c + ic : x;
          cp_async16_zfill(arow + ((ch ^ (r & 7)) * 16), src, v);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        pend[npend++] = s;
        if (npend > kLag) {
          // all but the kLag newest groups have landed: publish the oldest
          asm volatile("cp.async.wait_group %0;" ::"n"(kLag) : "memory");
          fence_proxy_async_smem();
          mbar_arrive(&full[pend[0]]);
#pragma unroll
          for (int i = 0; i + 1 < S; ++i) pend[i] = pend[i + 1];
          --npend;
        }
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    fence_proxy_async_smem();
    for (int i = 0; i < npend; ++i) mbar_arrive(&full[pend[i]]);
  } else if (warp == 4) {
    {  // the whole warp; one elected lane issues
      constexpr uint32_t idesc = f16_instr_desc(kBM, BN, H16Traits<T>::kBf16);
      uint32_t c = 0;
      int lt = 0;
      for (int t = blockIdx.x; t < n_tiles && !__any_sync(0xFFFFFFFFu, *abort_flag != 0); t += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait_warp(&tempty[buf], ((lt >> 1) & 1) ^ 1u)) {
          timed_out();
          break;
        }
        tc_fence_after();
        const uint32_t acc = tbase + buf * kAccCols;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++c) {
          const int s = c % S;
          const uint32_t ph = (c / S) & 1;
          if (!mbar_wait_warp(&full[s], ph)) {
            timed_out();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(sB + s * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t da = sw128_kmajor_desc(a_addr + k * 32);
            const uint64_t db = sw128_kmajor_desc(b_addr + k * 32);
            mma_f16_e(acc, da, db, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit_e(&empty[s]);
        }
        if (!ok) break;
        mma_commit_e(&tfull[buf]);
      }
    }
  } else {
    const int q = warp & 3;
    int lt = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++lt) {
      const int buf = lt & 1;
      if (*abort_flag || !mbar_wait(&tfull[buf], (lt >> 1) & 1)) {
        if (lane == 0) timed_out();
        break;
      }
      tc_fence_after();
      const int m0 = (t / n_tiles_n) * kBM, n0 = (t % n_tiles_n) * BN;
      const int row = m0 + q * 32 + lane;
      const uint32_t trow = tbase + buf * kAccCols + (static_cast<uint32_t>(q * 32) << 16);
      int cb, ce;
      epi_range<BN>(ep.mode, 0, 1, cb, ce);
      epilogue<BN, T>(ep, trow, row, M, n0, N, cb, ce);
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tbase, kAllocCols);
  }
}

template <int BN, typename T>
int launch_conv(const void* x, const ConvGeom& g, const void* B, int M, int N, int K,
                const EpiParams& ep, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  CUtensorMap tb;
  int rc = make_tmap_2d(&tb, B, H16Traits<T>::kBf16, K, N, K, kBK, BN);
  if (rc) return rc;
  auto kern = conv_gemm_kernel<BN, T>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::kSmem);
  if (e != cudaSuccess) return (int)e;
  const int tiles = ((N + BN - 1) / BN) * ((M + kBM - 1) / kBM);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  e = launch_pdl(kern, dim3(grid), dim3(288), Cfg::kSmem, stream, static_cast<const T*>(x), g, tb,
                 M, N, K, ep);
  if (e != cudaSuccess) return (int)e;
  return (int)cudaGetLastError();
}

template <int BN, int BK, typename T>
int launch_conv_pair(const void* x, int n, int h, int w, int c, const void* wt, int N,
                     bool time_major, const EpiParams& ep, cudaStream_t stream) {
  using Cfg = ConvPairCfg<BN, BK>;
  ConvTiles g;
  g.ho = (h - 1) / 2 + 1;
  g.wo = (w - 1) / 2 + 1;
  g.c = c;
  g.rows = std::min(kBM / g.wo, g.ho);
  g.tiles_per_img = (g.ho + g.rows - 1) / g.rows;
  g.n_mtiles = n * g.tiles_per_img;
  g.time_major = time_major ? 1 : 0;
  g.a_bytes = static_cast<uint32_t>(g.rows * g.wo * BK * 2);
  const int K = 9 * c;
  const long long dims[4] = {c, w, h, n};
  const long long strides[3] = {2LL * c, 2LL * c * w, 2LL * c * w * h};
  const int box[4] = {BK, 2 * g.wo - 1, 2 * g.rows - 1, 1};
  const int estr[4] = {1, 2, 2, 1};
  CUtensorMap tx, tb;
  int rc = make_tmap_nd(&tx, x, H16Traits<T>::kBf16, 4, dims, strides, box, estr, 2 * BK);
  if (rc) return rc;
  const long long bdims[2] = {K, N};
  const long long bstr[1] = {2LL * K};
  const int bbox[2] = {BK, BN / 2};
  const int bestr[2] = {1, 1};
  rc = make_tmap_nd(&tb, wt, H16Traits<T>::kBf16, 2, bdims, bstr, bbox, bestr, 2 * BK);
  if (rc) return rc;
  auto kern = conv_pair_kernel<BN, BK, T>;
  // the 16-bit store epilogue adds the epilogue warps' staging buffers
  const size_t smem = Cfg::kSmem + (ep.mode == EPI_STORE16 ? kGemmEpiWarps * kEpiStageBytes : 0);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // added for the launch
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static int max_pairs[64] = {0};  // per instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!max_pairs[dev]) {
    cfg.gridDim = dim3(2 * (num_sms() / 2), 1, 1);
    int np = 0;
    if (cudaOccupancyMaxActiveClusters(&np, kern, &cfg) != cudaSuccess || np <= 0) np = num_sms() / 2;
    max_pairs[dev] = np;
  }
  const int tiles = (N / BN) * ((g.n_mtiles + 1) / 2);
  const int pairs = tiles < max_pairs[dev] ? tiles : max_pairs[dev];
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.numAttrs = 2;  // cluster + programmatic serialization
  e = cudaLaunchKernelEx(&cfg, kern, tx, tb, g, N, K, ep);
  if (e != cudaSuccess) return (int)e;
  return (int)cudaGetLastError();
}

template <int BN, typename T>
int launch_conv_tma(const void* x, int n, int h, int w, int c, const void* wt, int N,
                    bool time_major, const EpiParams& ep, cudaStream_t stream) {
  using Cfg = ConvCfg<BN>;
  ConvTiles g;
  g.ho = (h - 1) / 2 + 1;
  g.wo = (w - 1) / 2 + 1;
  g.c = c;
  g.rows = std::min(kBM / g.wo, g.ho);
  g.tiles_per_img = (g.ho + g.rows - 1) / g.rows;
  g.n_mtiles = n * g.tiles_per_img;
  g.time_major = time_major ? 1 : 0;
  g.a_bytes = static_cast<uint32_t>(g.rows * g.wo * kCvBK * 2);
  const int K = 9 * c;
  // the input as [n][h][w][c]; spans 2*wo-1 and 2*rows-1 with stride 2 load
  // wo columns and rows rows (and never exceed the tensor's own extent)
  const long long dims[4] = {c, w, h, n};
  const long long strides[3] = {2LL * c, 2LL * c * w, 2LL * c * w * h};
  const int box[4] = {kCvBK, 2 * g.wo - 1, 2 * g.rows - 1, 1};
  const int estr[4] = {1, 2, 2, 1};
  CUtensorMap tx, tb;
  int rc = make_tmap_nd(&tx, x, H16Traits<T>::kBf16, 4, dims, strides, box, estr, 64);
  if (rc) return rc;
  const long long bdims[2] = {K, N};
  const long long bstr[1] = {2LL * K};
  const int bbox[2] = {kCvBK, BN};
  const int bestr[2] = {1, 1};
  rc = make_tmap_nd(&tb, wt, H16Traits<T>::kBf16, 2, bdims, bstr, bbox, bestr, 64);
  if (rc) return rc;
  auto kern = conv_tma_kernel<BN, T>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::kSmem);
  if (e != cudaSuccess) return (int)e;
  const int tiles = ((N + BN - 1) / BN) * g.n_mtiles;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  e = launch_pdl(kern, dim3(grid), dim3(kGemmThreads), Cfg::kSmem, stream, tx, tb, g, N, K, ep);
  if (e != cudaSuccess) return (int)e;
  return (int)cudaGetLastError();
}

template <int BN, typename T>
int launch_pair(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                const EpiParams& ep, cudaStream_t stream) {
  // the instantiation (QKV, residual, other) and its shared memory: the
  // ring, the barriers and the epilogue warps' staging buffers
  const bool resid = ep.mode == EPI_RESID32 || ep.mode == EPI_RESID16;
  const bool qkv = BN % 128 == 0 && ep.mode == EPI_QKV_ROPE;
  const bool staged = ep.mode == EPI_STORE16 || ep.mode == EPI_SWIGLU16;
  const int stages = (qkv || resid) ? kPairStages - 1 : kPairStages;
  const size_t kPairSmem = 1024 + stages * (kPairHalf + PairCfg<BN>::kBHalf) + 256 +
                           ((qkv || resid) ? 2 : staged ? 1 : 0) * kGemmEpiWarps * kEpiStageBytes;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, H16Traits<T>::kBf16, K, M, lda, kBK, kBM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, B, H16Traits<T>::kBf16, K, N, ldb, kBK, BN / 2);
  if (rc) return rc;
  auto kern = resid ? gemm_pair_kernel<BN, T, 2> : gemm_pair_kernel<BN, T, 0>;
  if constexpr (BN % 128 == 0)
    if (qkv) kern = gemm_pair_kernel<BN, T, 1>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPairSmem);
  if (e != cudaSuccess) return (int)e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // added for the launch
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = kPairSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // persistent: as many pairs as can be resident at once (cached per device)
  static int max_pairs[64] = {0};  // per instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!max_pairs[dev]) {
    cfg.gridDim = dim3(2 * (num_sms() / 2), 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) n = num_sms() / 2;
    max_pairs[dev] = n;
  }
  const int tiles = (N / BN) * ((M + 255) / 256);
  const int pairs = tiles < max_pairs[dev] ? tiles : max_pairs[dev];
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.numAttrs = 2;  // cluster + programmatic serialization
  e = cudaLaunchKernelEx(&cfg, kern, ta, tb, M, N, K, ep);
  if (e != cudaSuccess) return (int)e;
  return (int)cudaGetLastError();
}

template <int BN, typename T>
int launch(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
           const EpiParams& ep, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  CUtensorMap ta, tb;
  // an implicit conv reads A as [M, conv_kb * 64]; K spans the taps
  const int ka = ep.conv_kb > 0 ? ep.conv_kb * kBK : K;
  int rc = make_tmap_2d(&ta, A, /*bf16=*/H16Traits<T>::kBf16, ka, M, lda, kBK, kBM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, B, H16Traits<T>::kBf16, K, N, ldb, kBK, BN);
  if (rc) return rc;
  auto kern = gemm_tc_kernel<BN, T>;
  // the residual modes add the epilogue warps' staging buffers
  const bool resid = ep.mode == EPI_RESID32 || ep.mode == EPI_RESID16;
  const size_t smem = Cfg::kSmem + (resid ? kGemmEpiWarps * kEpiStageBytes : 0);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  const int tiles = ((N + BN - 1) / BN) * ((M + kBM - 1) / kBM);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  e = launch_pdl(kern, dim3(grid), dim3(kGemmThreads), smem, stream, ta, tb, M, N, K, ep);
  if (e != cudaSuccess) return (int)e;
  return (int)cudaGetLastError();
}

}  // namespace

int device_sm_count() { return num_sms(); }

int gemm_pick_bn(int N) {
  if (N % 256 == 0) return 256;
  if (N % 240 == 0) return 240;
  if (N % 224 == 0) return 224;
  if (N % 128 == 0 && N <= 512) return 128;
  return 256;
}

int gemm_tc(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
            bool bf16, const EpiParams& ep, cudaStream_t stream, int force_bn) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(A) & 15u) || (reinterpret_cast<uintptr_t>(B) & 15u) ||
      (lda % 8) || (ldb % 8))
    return (int)cudaErrorInvalidValue;
  // an implicit conv runs on the one-CTA kernel only, with whole taps of
  // 64-column k-blocks
  if (ep.conv_kb > 0) {
    if (force_bn == -1 || K % (ep.conv_kb * kBK) || lda < ep.conv_kb * kBK)
      return (int)cudaErrorInvalidValue;
    if (force_bn == 0) force_bn = gemm_pick_bn(N);
  }
  // 256 x 256 (or 256 x 224) tiles on CTA pairs whenever N allows (force_bn 0
  // = choose, -1 = require the pair kernel, > 0 = one CTA per tile, that width)
  // folded RMSNorm: whole rows of 128-column blocks, read as float4, one
  // block per epilogue thread (256-wide tiles)
  if ((ep.ssq_in || ep.ssq_out) &&
      (ep.ssq_n % 4 || ep.ssq_n > kSsqMax || (ep.ssq_out && ep.ssq_n * kSsqCols != N) ||
       (ep.ssq_out && force_bn > 0 && force_bn != 256) ||
       ((reinterpret_cast<uintptr_t>(ep.ssq_in) | reinterpret_cast<uintptr_t>(ep.ssq_out)) & 15u)))
    return (int)cudaErrorInvalidValue;
  const bool pair224 = N % 224 == 0 && ep.mode != EPI_SWIGLU16 && ep.mode != EPI_QKV_ROPE;
  if (force_bn == -1 || (force_bn == 0 && M > 128 && (N % 256 == 0 || pair224))) {
    if (N % 256 == 0)
      return bf16 ? launch_pair<256, __nv_bfloat16>(A, lda, B, ldb, M, N, K, ep, stream)
                  : launch_pair<256, __half>(A, lda, B, ldb, M, N, K, ep, stream);
    if (pair224)
      return bf16 ? launch_pair<224, __nv_bfloat16>(A, lda, B, ldb, M, N, K, ep, stream)
                  : launch_pair<224, __half>(A, lda, B, ldb, M, N, K, ep, stream);
    return (int)cudaErrorInvalidValue;
  }
  const int bn = force_bn ? force_bn : gemm_pick_bn(N);
  if (ep.mode == EPI_SWIGLU16 && ((N % bn) || (bn % 64))) return (int)cudaErrorInvalidValue;
  if (ep.mode == EPI_QKV_ROPE && ((N % 128) || (bn % 128))) return (int)cudaErrorInvalidValue;
#define QA_GEMM_CASE(BNV)                                                               \
  case BNV:                                                                             \
    return bf16 ? launch<BNV, __nv_bfloat16>(A, lda, B, ldb, M, N, K, ep, stream)       \
                : launch<BNV, __half>(A, lda, B, ldb, M, N, K, ep, stream);
  switch (bn) {
    QA_GEMM_CASE(128)
    QA_GEMM_CASE(224)
    QA_GEMM_CASE(240)
    QA_GEMM_CASE(256)
    default:
      return (int)cudaErrorInvalidValue;
  }
#undef QA_GEMM_CASE
}

int conv3x3s2_tc(const void* x, int n, int h, int w, int c, const void* wt, int c_out,
                 bool time_major, bool bf16, const EpiParams& ep, cudaStream_t stream) {
  if (n <= 0) return 0;
  if (c % 8 || (reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(wt) & 15u))
    return (int)cudaErrorInvalidValue;
  ConvGeom g{h, w, c, (h - 1) / 2 + 1, (w - 1) / 2 + 1, time_major ? 1 : 0};
  const int M = n * g.ho * g.wo, K = 9 * c;
  const int bn = gemm_pick_bn(c_out);
  // TMA path: whole 32-channel k-blocks per tap and output rows that fit a tile
  if (c % 64 == 0 && g.wo <= kBM && c_out % 240 == 0)  // CTA pairs, 256 x 240 tiles, 64-wide k
    return bf16 ? launch_conv_pair<240, 64, __nv_bfloat16>(x, n, h, w, c, wt, c_out, time_major, ep, stream)
                : launch_conv_pair<240, 64, __half>(x, n, h, w, c, wt, c_out, time_major, ep, stream);
  if (c % kCvBK == 0 && g.wo <= kBM && c_out % 240 == 0)  // 32-wide k
    return bf16 ? launch_conv_pair<240, 32, __nv_bfloat16>(x, n, h, w, c, wt, c_out, time_major, ep, stream)
                : launch_conv_pair<240, 32, __half>(x, n, h, w, c, wt, c_out, time_major, ep, stream);
  if (c % kCvBK == 0 && g.wo <= kBM && (bn == 240 || bn == 256)) {
    if (bn == 240)
      return bf16 ? launch_conv_tma<240, __nv_bfloat16>(x, n, h, w, c, wt, c_out, time_major, ep, stream)
                  : launch_conv_tma<240, __half>(x, n, h, w, c, wt, c_out, time_major, ep, stream);
    return bf16 ? launch_conv_tma<256, __nv_bfloat16>(x, n, h, w, c, wt, c_out, time_major, ep, stream)
                : launch_conv_tma<256, __half>(x, n, h, w, c, wt, c_out, time_major, ep, stream);
  }
#define QA_CONV_CASE(BNV)                                                                 \
  case BNV:                                                                               \
    return bf16 ? launch_conv<BNV, __nv_bfloat16>(x, g, wt, M, c_out, K, ep, stream)       \
                : launch_conv<BNV, __half>(x, g, wt, M, c_out, K, ep, stream);
  switch (bn) {
    QA_CONV_CASE(240)
    QA_CONV_CASE(256)
    default:
      return (int)cudaErrorInvalidValue;
  }
#undef QA_CONV_CASE
}

}  // namespace qa
