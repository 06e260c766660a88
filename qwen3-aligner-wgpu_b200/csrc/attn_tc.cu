// (e) Causal GQA flash attention on the tcgen05 tensor cores.
//
// softmax(q·kᵀ / sqrt(128)) · v over keys 0..=pos of the same clip
// (src/cpu_decoder.rs:327-412), for the decoder prefill over the paged K/V
// cache.  A work item is one K/V head of one clip and 128 query positions
// q0..q0+127: two M=128 tiles, one per query head of the GQA pair (heads
// 2·kvh and 2·kvh+1), which share every K/V tile the item reads.  The kernel
// is persistent: one CTA per SM walks items blockIdx.x, +gridDim.x, ... of a
// list ordered longest clip first, and its pipeline runs on across item
// boundaries (the next item's Q and K/V pages load while the current one
// finishes).
//
//   warp 0      TMA: the item's two Q tiles, then its K tiles (128 keys = two
//               64-token pages, or one page for a last half tile);
//   warp 1      TMA: the V tiles (a separate ring, so K runs ahead of V);
//   warp 2      TMEM allocation and the MMAs, issued by one thread:
//                 S_h = Q_h·Kᵀ   (M=128, N=128 or 64 keys, K=128 dims) -> TMEM
//                 O_h += P_h·V   (M=128, N=128 dims, K=keys), P_h read from
//                                TMEM, V as an MN-major operand straight from
//                                the pages as TMA stored them;
//               in the order S_0(j), P_1·V(j-1), S_1(j), P_0·V(j), so that the
//               tensor cores work on one head while the other head's softmax
//               runs;
//   warps 3-10  softmax of head 0, warps 11-18 of head 1: each query row is
//               shared by two threads in two warps on the same SM sub-partition
//               (keys 0-63 and 64-127 of the tile; two warps per sub-partition
//               keep the MUFU unit busy, one alone cannot).  They exchange
//               partial row maxima through shared memory, keep the running max
//               and their partial sums in f32, write p = 2^(s·scale·log2e - m)
//               packed to 16 bits back into the first 32 columns of their own
//               half of the row's S columns (the MMA reads P there: keys 0-63
//               from columns 0-31, keys 64-127 from columns 64-95, so neither
//               half overwrites S the other has yet to read), rescale their
//               half of the O row in TMEM
//               only when the row max grew by more than 2^8 since the last
//               rescale (O / sum is exact for any reference max), and at the
//               end write their half of O / sum.
//
// TMEM (512 columns): S_0 [0,128), S_1 [128,256), O_0 [256,384), O_1 [384,512).
// tcgen05.mma instructions from one thread execute in issue order, so S_h(j+1)
// may overwrite P_h(j) once P_h(j)·V has been issued; every tcgen05.commit
// tracks all earlier MMAs, so O may be rescaled once S_h(j) is complete.
// Barriers: q_full/q_empty, k_full/k_empty, v_full/v_empty (rings), s_full[h]
// (S_h ready), p_full[h] (P_h written, O_h rescaled; 256 arrivals), o_done[h]
// (last P_h·V of the item done); named barriers 1 and 2 pair the two halves of
// each head's rows.  Every mbarrier wait is bounded (sm100.cuh), and every
// decision to leave a loop is voted on by the whole head (bar.red.and) so
// that no warp is left at a named barrier.  No cluster multicast: each CTA
// loads its own tiles.
#include <algorithm>

#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "sm100.cuh"
#include "tma_host.h"

namespace qa {

namespace {

constexpr int kHD = 128;       // head dim
constexpr int kRows = 128;     // query positions per item (one M=128 tile per head)
constexpr int kKeys = 128;     // keys per K/V tile (two 64-token pages)
constexpr int kPage = 64;
constexpr int kSoftmaxWarps = 8;                     // per head
constexpr int kThreads = (3 + 2 * kSoftmaxWarps) * 32;  // 19 warps
constexpr uint32_t kTile = kRows * kHD * 2;  // 32 KB: a Q, K or V tile
constexpr uint32_t kHalf = kTile / 2;        // 16 KB: one 64-column block of a tile
constexpr uint32_t kPageBytes = kHalf / 2;   // 8 KB: 64 rows of one block
constexpr int kKStages = 2;
constexpr int kVStages = 2;
constexpr uint32_t kXchBytes = 2 * 2 * kRows * 4;  // partial max (or sum) [head][half][row]
constexpr size_t kSmem =
    1024 + (2 + kKStages + kVStages) * kTile + 2 * kXchBytes + 256;  // Q, K, V, exchange, bars
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;  // rescale O when the row max grows by > 2^8
// Of every 8 pairs of probabilities, this many are computed with ex2_poly on
// the FMA/ALU pipes instead of the MUFU unit (which is the softmax's
// bottleneck at 16 results per clock per SM).
constexpr int kEmuPairs = 0;

struct AttnParams {
  const AttnTile* tiles;
  int n_items;  // tiles x K/V heads
  int nkv;
  const int* block_tab;
  int max_pages;
  float scale_log2;  // log2(e) / sqrt(128)
  void* out;
  long long ldo;     // out row stride (nq * 128)
  long long q_rows;  // rows of qkv and out
  int kv_pages;      // pages in each K/V pool
  unsigned* status;
};

// The shape of one work item; every role derives it the same way.
struct Item {
  AttnTile t;
  int kvh;
  int n_keys;   // keys the block attends to, rounded up to a page
  int n_tiles;  // 128-key tiles (the last may hold one page)
  bool valid;
};

__device__ __forceinline__ Item get_item(const AttnParams& ap, int i) {
  Item it;
  it.t = ap.tiles[i / ap.nkv];
  it.kvh = i % ap.nkv;
  const AttnTile& t = it.t;
  const int clip_pages = (t.len + kPage - 1) / kPage;
  it.valid = t.clip >= 0 && t.len > 0 && t.q0 >= 0 && t.q0 < t.len && t.tok0 >= 0 &&
             t.tok0 + static_cast<long long>(t.len) <= ap.q_rows && clip_pages <= ap.max_pages;
  const int q_hi = min(t.q0 + kRows, t.len);
  it.n_keys = (q_hi + kPage - 1) / kPage * kPage;
  it.n_tiles = (it.n_keys + kKeys - 1) / kKeys;
  return it;
}

__device__ __forceinline__ int tile_keys(const Item& it, int j) {
  return min(kKeys, it.n_keys - j * kKeys);
}

// 2^x for x <= 8 without the MUFU unit: x = n + f with n = rint(x) (adding
// 1.5 * 2^23 rounds to an integer held in the low mantissa bits), f in
// [-0.5, 0.5]; 2^f from a degree-3 polynomial fitted for minimax relative
// error on that interval (7.5e-5, below half an f16 ulp); 2^n is added to the
// exponent field as an integer.  x below -126 is clamped (2^-126 is zero in
// f16 and negligible in bf16 and in the row sum).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.0f);
  const float t = x + 12582912.0f;
  const float f = x - (t - 12582912.0f);
  const float p =
      fmaf(fmaf(fmaf(0.05517167f, f, 0.24261113f), f, 0.69326097f), f, 0.99992806f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// bar.red.and over a named barrier: every participating thread gets the AND
// of all threads' predicates (a synchronising, uniform vote).
__device__ __forceinline__ bool bar_and(int id, int nthreads, bool pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<int>(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// Scores i > lim of a 32-column chunk are masked to -inf (lim = the last
// visible key minus the chunk's first key); only diagonal and clip-end chunks
// (lim < 31) pay for it.
__device__ __forceinline__ void mask32(uint32_t (&u)[32], int lim) {
  if (lim < 31) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i > lim) u[i] = __float_as_uint(-INFINITY);
  }
}

// Exponentials of 32 scores against the row max, packed in pairs into w;
// their sum is added to `sum`.
template <typename T>
__device__ __forceinline__ void exp_pack32(const uint32_t (&u)[32], float scale, float neg,
                                           uint32_t (&w)[16], float& sum) {
  float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const float v0 = __uint_as_float(u[2 * e]), v1 = __uint_as_float(u[2 * e + 1]);
    const bool emu = (e & 7) < kEmuPairs;
    const float x0 = fmaf(v0, scale, neg), x1 = fmaf(v1, scale, neg);
    const float p0 = emu ? ex2_poly(x0) : ex2_approx(x0);
    const float p1 = emu ? ex2_poly(x1) : ex2_approx(x1);
    s4[e & 3] += p0 + p1;
    w[e] = pack2<T>(p0, p1);
  }
  sum += (s4[0] + s4[1]) + (s4[2] + s4[3]);
}

__device__ __forceinline__ float max32(const uint32_t (&u)[32]) {
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < 32; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(u[i]));
  return fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, AttnParams ap) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                   // [2 heads]
  uint8_t* sK = sQ + 2 * kTile;         // [kKStages]
  uint8_t* sV = sK + kKStages * kTile;  // [kVStages]
  float* xmax = reinterpret_cast<float*>(sV + kVStages * kTile);  // [head][half][row]
  float* xsum = xmax + 2 * 2 * kRows;                               // [head][half][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(xsum + 2 * 2 * kRows);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;    // [kKStages]
  uint64_t* k_empty = bars + 5;   // [kKStages]
  uint64_t* v_full = bars + 8;    // [kVStages]
  uint64_t* v_empty = bars + 10;  // [kVStages]
  uint64_t* s_full = bars + 12;   // [2 heads]
  uint64_t* p_full = bars + 14;   // [2 heads]
  uint64_t* o_done = bars + 16;   // [2 heads]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 32 * kSoftmaxWarps);
      mbar_init(&o_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 2) tmem_alloc(tslot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  auto fail = [&]() {
    *abort_flag = 1;
    if (ap.status) atomicOr(ap.status, kStatusTimeout);
  };

  if (warp <= 1) {
    // warp 0: Q and K; warp 1: V
    if (lane == 0) {
      const bool is_k = warp == 0;
      uint32_t n_it = 0, g = 0;
      bool ok = true;
      for (int i = blockIdx.x; ok && i < ap.n_items; i += gridDim.x) {
        const Item it = get_item(ap, i);
        if (!it.valid) {
          if (is_k && ap.status) atomicOr(ap.status, kStatusBadShape);
          continue;
        }
        if (is_k) {
          if (*abort_flag || !mbar_wait(q_empty, (n_it & 1) ^ 1u)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(q_full, 2 * kTile);
          const int y = it.t.tok0 + it.t.q0;
          for (int h = 0; h < 2; ++h)
            for (int half = 0; half < 2; ++half)
              tma_load_2d(&tmQ, q_full, sQ + h * kTile + half * kHalf,
                          (it.kvh * 2 + h) * kHD + half * 64, y);
        }
        const int* bt = ap.block_tab + static_cast<long long>(it.t.clip) * ap.max_pages;
        uint64_t* full = is_k ? k_full : v_full;
        uint64_t* empty = is_k ? k_empty : v_empty;
        uint8_t* ring = is_k ? sK : sV;
        const CUtensorMap* tm = is_k ? &tmK : &tmV;
        for (int j = 0; j < it.n_tiles; ++j, ++g) {
          const int st = g & 1;
          const uint32_t ph = ((g >> 1) & 1) ^ 1u;
          const int npg = tile_keys(it, j) / kPage;
          int rows[2] = {0, 0};
          for (int pg = 0; pg < npg; ++pg) {
            int page = bt[2 * j + pg];
            if (page < 0 || page >= ap.kv_pages) {
              if (ap.status) atomicOr(ap.status, kStatusBadShape);
              page = 0;
            }
            rows[pg] = (page * ap.nkv + it.kvh) * kPage;
          }
          if (*abort_flag || !mbar_wait(&empty[st], ph)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[st], npg * 2 * kPageBytes);
          for (int pg = 0; pg < npg; ++pg)
            for (int half = 0; half < 2; ++half)
              tma_load_2d(tm, &full[st], ring + st * kTile + half * kHalf + pg * kPageBytes,
                          half * 64, rows[pg]);
        }
        ++n_it;
      }
      if (!ok) fail();
    }
  } else if (warp == 2) {
    if (lane == 0) {
      const bool bf = H16Traits<T>::kBf16;
      const uint32_t idS128 = f16_instr_desc(kRows, 128, bf);
      const uint32_t idS64 = f16_instr_desc(kRows, 64, bf);
      const uint32_t idPV = f16_instr_desc(kRows, kHD, bf) | (1u << 16);  // B (V) MN-major
      const uint32_t tS[2] = {tbase, tbase + 128};
      const uint32_t tO[2] = {tbase + 256, tbase + 384};
      const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK), va = smem_u32(sV);
      auto issue_s = [&](int h, int st, int keys) {
        const uint32_t id = keys == 128 ? idS128 : idS64;
#pragma unroll
        for (int ks = 0; ks < kHD / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kHalf + (ks & 3) * 32;
          mma_f16(tS[h], sw128_kmajor_desc(qa + h * kTile + off),
                  sw128_kmajor_desc(ka + st * kTile + off), id, ks > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[h]);
      };
      auto issue_pv = [&](int h, int st, int keys, bool acc) {
        // P for keys 0-63 in S columns 0-31, for keys 64-127 in columns 64-95
        for (int ks = 0; ks < keys / 16; ++ks)
          mma_f16_ts(tO[h], tS[h] + (ks >> 2) * 64 + (ks & 3) * 8,
                     sw128_mn_desc(va + st * kTile + ks * 16 * 128, kHalf, 1024), idPV,
                     (acc || ks > 0) ? 1u : 0u);
      };
      uint32_t n_it = 0, g = 0;
      bool ok = true;
      for (int i = blockIdx.x; ok && i < ap.n_items; i += gridDim.x) {
        const Item it = get_item(ap, i);
        if (!it.valid) continue;
        if (*abort_flag || !mbar_wait(q_full, n_it & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        int prev_keys = 0;
        for (int j = 0; j < it.n_tiles; ++j, ++g) {
          const int st = g & 1, kst = st;
          const uint32_t ph = (g >> 1) & 1, kph = ph;
          const int keys = tile_keys(it, j);
          if (!mbar_wait(&k_full[kst], kph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(0, kst, keys);
          if (j > 0) {
            if (!mbar_wait(&p_full[1], (g - 1) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(1, st ^ 1, prev_keys, j > 1);
            mma_commit(&v_empty[st ^ 1]);
          }
          issue_s(1, kst, keys);
          mma_commit(&k_empty[kst]);
          if (j == it.n_tiles - 1) mma_commit(q_empty);
          if (!mbar_wait(&v_full[st], ph) || !mbar_wait(&p_full[0], g & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(0, st, keys, j > 0);
          if (j == it.n_tiles - 1) mma_commit(&o_done[0]);
          prev_keys = keys;
        }
        if (!ok) break;
        // head 1's last P·V
        if (!mbar_wait(&p_full[1], (g - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv(1, (g - 1) & 1, prev_keys, it.n_tiles > 1);
        mma_commit(&v_empty[(g - 1) & 1]);
        mma_commit(&o_done[1]);
        ++n_it;
      }
      if (!ok) fail();
    }
  } else {
    // softmax: head h, half hf of the keys (and of the O columns), row r
    const int sw = warp - 3;
    const int h = sw / kSoftmaxWarps;
    const int hf = (sw % kSoftmaxWarps) / 4;
    const int quarter = warp & 3;  // TMEM lanes 32*quarter.. are this warp's
    const int r = quarter * 32 + lane;
    const int bar_id = 1 + h;
    const int bar_n = 32 * kSoftmaxWarps;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tbase + h * 128 + lane_off;
    const uint32_t tO = tbase + 256 + h * 128 + lane_off + hf * 64;
    float* my_max = xmax + (h * 2 + hf) * kRows + r;
    const float* other_max = xmax + (h * 2 + (hf ^ 1)) * kRows + r;
    float* my_sum = xsum + (h * 2 + hf) * kRows + r;
    const float* other_sum = xsum + (h * 2 + (hf ^ 1)) * kRows + r;
    const float scale = ap.scale_log2;
    uint32_t n_it = 0, g = 0;
    bool ok = true;
    for (int i = blockIdx.x; ok && i < ap.n_items; i += gridDim.x) {
      const Item it = get_item(ap, i);
      if (!it.valid) continue;
      const int pos = it.t.q0 + r;
      const int len = it.t.len;
      float m_used = -INFINITY, l = 0.0f;
      for (int j = 0; j < it.n_tiles; ++j, ++g) {
        const int keys = tile_keys(it, j);
        const int key0 = j * kKeys + hf * 64;   // first key of this thread's half
        const bool active = hf * 64 < keys;      // a 64-key tile has no second half
        // keys key0 + i are visible for i <= lim (lim >= 63: the whole half)
        const int lim = min(pos, len - 1) - key0;
        const bool got = !*abort_flag && mbar_wait(&s_full[h], g & 1);
        tc_fence_after();
        // pass 1: partial max of this half, 32 columns at a time
        float pm = -INFINITY;
        if (got && active) {
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t u[32];
            tmem_ld_x32(tS + hf * 64 + c * 32, u);
            mask32(u, lim - c * 32);
            pm = fmaxf(pm, max32(u));
          }
        }
        *my_max = pm;
        if (!bar_and(bar_id, bar_n, got)) {  // also publishes my_max
          ok = false;
          break;
        }
        const float mx_s = fmaxf(pm, *other_max) * scale;  // scale > 0
        const bool grow = mx_s > m_used + kRescaleLog2;
        float alpha = 1.0f;
        if (grow) {
          alpha = ex2_approx(m_used - mx_s);  // 0 on the first tile (m_used = -inf)
          m_used = mx_s;
        }
        if (j > 0 && __any_sync(0xFFFFFFFFu, grow)) {
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            float o[32];
            tmem_ld32(tO + c * 32, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(tO + c * 32, o);
          }
        }
        l *= alpha;
        if (active) {
          // pass 2: P for keys [key0, key0+64) -> TMEM columns [hf*64, hf*64+32);
          // chunk c's P lands on columns chunk 0 has already been read from
          const float neg = m_used == -INFINITY ? 0.0f : -m_used;
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t u[32], w[16];
            tmem_ld_x32(tS + hf * 64 + c * 32, u);
            mask32(u, lim - c * 32);
            exp_pack32<T>(u, scale, neg, w, l);
            tmem_st_x16(tS + hf * 64 + c * 16, w);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[h]);
      }
      if (!ok) break;
      const bool got = !*abort_flag && mbar_wait(&o_done[h], n_it & 1);
      *my_sum = l;
      if (!bar_and(bar_id, bar_n, got)) {  // also publishes my_sum
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = 1.0f / (l + *other_sum);
      T* dst = static_cast<T*>(ap.out) + (static_cast<long long>(it.t.tok0) + pos) * ap.ldo +
               static_cast<long long>(it.kvh * 2 + h) * kHD + hf * 64;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float o[32];
        tmem_ld32(tO + c * 32, o);
        if (pos < len) {
          alignas(16) T ov[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = f2h<T>(o[e] * inv);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            reinterpret_cast<uint4*>(dst + c * 32)[e] = reinterpret_cast<const uint4*>(ov)[e];
        }
      }
      tc_fence_before();
      ++n_it;
    }
    if (!ok && lane == 0) fail();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace

int causal_attention_tc(const void* qkv, long long ldq, long long q_rows, int nqh, int nkvh,
                        int hd, const AttnTile* tiles, int n_tiles, const int* block_tab,
                        int max_pages, PagedKV kv, int kv_pages, void* out, bool bf16,
                        unsigned* status, cudaStream_t s) {
  if (n_tiles <= 0) return 0;
  if (hd != kHD || nqh != 2 * nkvh || kv.page_size != kPage) return (int)cudaErrorInvalidValue;
  CUtensorMap tq, tk, tv;
  const long long kv_rows = static_cast<long long>(kv_pages) * nkvh * kPage;
  int rc = make_tmap_2d(&tq, qkv, bf16, ldq, q_rows, ldq, 64, kRows);
  if (!rc) rc = make_tmap_2d(&tk, kv.k, bf16, kHD, kv_rows, kHD, 64, kPage);
  if (!rc) rc = make_tmap_2d(&tv, kv.v, bf16, kHD, kv_rows, kHD, 64, kPage);
  if (rc) return rc;
  AttnParams ap{};
  ap.tiles = tiles;
  ap.n_items = n_tiles * nkvh;
  ap.nkv = nkvh;
  ap.block_tab = block_tab;
  ap.max_pages = max_pages;
  ap.scale_log2 = (1.0f / sqrtf(128.0f)) * 1.4426950408889634f;
  ap.out = out;
  ap.ldo = static_cast<long long>(nqh) * kHD;
  ap.q_rows = q_rows;
  ap.kv_pages = kv_pages;
  ap.status = status;
  const int grid = std::min(ap.n_items, device_sm_count());
  if (bf16) {
    auto k = attn_tc_kernel<__nv_bfloat16>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
    if (e != cudaSuccess) return (int)e;
    k<<<grid, kThreads, kSmem, s>>>(tq, tk, tv, ap);
  } else {
    auto k = attn_tc_kernel<__half>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
    if (e != cudaSuccess) return (int)e;
    k<<<grid, kThreads, kSmem, s>>>(tq, tk, tv, ap);
  }
  return (int)cudaGetLastError();
}

}  // namespace qa
