// (e) Causal GQA flash attention on the tcgen05 tensor cores.
//
// softmax(q·kᵀ / sqrt(128)) · v over keys 0..=pos of the same clip
// (src/cpu_decoder.rs:327-412), for the decoder prefill over the paged K/V
// cache.  A work item is one query head of one clip and 128 query positions
// q0..q0+127 (one M=128 tile).  The kernel is persistent: one CTA per SM
// walks items blockIdx.x, +gridDim.x, ... ; items are ordered longest clip
// first with a clip's blocks adjacent and the two query heads of a K/V head
// next to each other, so the K/V pages a CTA reads were usually just read by
// its neighbour and come from L2.
//
//   warp 0       TMA: the item's Q tile (two smem buffers, so the next item's
//                Q loads early) and its K tiles (128 keys = two 64-token
//                pages, or one for a last half tile);
//   warp 1       TMA: the V tiles;
//   warp 2       TMEM allocation and the MMAs, issued by one thread:
//                  S(j) = Q·K(j)ᵀ  (M=128, N=128 or 64 keys, K=128 dims) with Q
//                                  read from TMEM, into one of two S buffers;
//                  O += P(j)·V(j)  (N=128 dims, K=keys), P read from TMEM, V
//                                  an MN-major operand straight from the pages;
//                in the order S(0), S(1), P·V(0), S(2), P·V(1), ... so that the
//                tensor cores compute S(j+1) while the softmax works on S(j);
//   warps 3-10   softmax: each query row is shared by two threads in two warps
//                on the same SM sub-partition (keys 0-63 and 64-127 of the
//                tile; two warps per sub-partition keep the MUFU unit busy).
//                They copy the item's Q from shared memory into TMEM, exchange
//                partial row maxima through shared memory, keep the running
//                max and their partial sums in f32, write P packed to 16 bits
//                over their own half of the S columns, and rescale their half
//                of the O row in TMEM only when the row max grew by more than
//                2^8 since the last rescale (O / sum is exact for any
//                reference max);
//   warps 11-14  epilogue: after the item's last P·V, O / (sum of the two
//                partial sums) row by row, then O is released for the next
//                item.
//
// TMEM (512 columns): Q [0,64) and [64,128) (16-bit, packed two per column),
// S [128,256) and [256,384), O [384,512).  tcgen05.mma instructions from one
// thread execute in issue order (S(j+1) may overwrite P(j-1) once P(j-1)·V has
// been issued), and every tcgen05.commit tracks all earlier MMAs.  Every
// mbarrier wait is bounded (sm100.cuh), and every decision to leave a loop in
// the softmax warps is voted on (bar.red.and) so that none is left at a named
// barrier.  No cluster multicast: each CTA loads its own tiles.
#include <algorithm>

#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "sm100.cuh"
#include "tma_host.h"

namespace qa {

namespace {

constexpr int kHD = 128;       // head dim
constexpr int kRows = 128;     // query positions per item (one M=128 tile)
constexpr int kKeys = 128;     // keys per K/V tile (two 64-token pages)
constexpr int kPage = 64;
constexpr int kSoftmaxWarps = 8;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (3 + kSoftmaxWarps + kEpiWarps) * 32;  // 15 warps
constexpr uint32_t kTile = kRows * kHD * 2;  // 32 KB: a Q, K or V tile
constexpr uint32_t kHalf = kTile / 2;        // 16 KB: one 64-column block of a tile
constexpr uint32_t kPageBytes = kHalf / 2;   // 8 KB: 64 rows of one block
constexpr int kKStages = 3;
constexpr int kVStages = 2;
constexpr uint32_t kXchBytes = 2 * 2 * kRows * 4;  // partial max (or sum) [buffer][half][row]
constexpr size_t kSmem =
    1024 + (1 + kKStages + kVStages) * kTile + 2 * kXchBytes + 256;  // Q, K, V, exchange, bars
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;  // rescale O when the row max grows by > 2^8

struct AttnParams {
  const AttnTile* tiles;
  int n_items;  // tiles x query heads
  int nq;
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
  int head, kvh;
  int n_keys;   // keys the block attends to, rounded up to a page
  int n_tiles;  // 128-key tiles (the last may hold one page)
  bool valid;
};

__device__ __forceinline__ Item get_item(const AttnParams& ap, int i) {
  Item it;
  it.t = ap.tiles[i / ap.nq];
  it.head = i % ap.nq;
  it.kvh = it.head / (ap.nq / ap.nkv);
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

// Scores i > lim of a thread's 64 keys are masked to -inf (lim = the last
// visible key minus the first key of the half); only diagonal and clip-end
// tiles (lim < 63) pay for it.
__device__ __forceinline__ void mask64(uint32_t (&u)[64], int lim) {
  if (lim < 63) {
#pragma unroll
    for (int i = 0; i < 64; ++i)
      if (i > lim) u[i] = __float_as_uint(-INFINITY);
  }
}

__device__ __forceinline__ float max64(const uint32_t (&u)[64]) {
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < 64; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(u[i]));
  return fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
}

// Exponentials of 64 scores against the row max, packed in pairs into w;
// their sum is added to `sum`.
template <typename T>
__device__ __forceinline__ void exp_pack64(const uint32_t (&u)[64], float scale, float neg,
                                           uint32_t (&w)[32], float& sum) {
  float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const float v0 = __uint_as_float(u[2 * e]), v1 = __uint_as_float(u[2 * e + 1]);
    const float p0 = ex2_approx(fmaf(v0, scale, neg));
    const float p1 = ex2_approx(fmaf(v1, scale, neg));
    s4[e & 3] += p0 + p1;
    w[e] = pack2<T>(p0, p1);
  }
  sum += (s4[0] + s4[1]) + (s4[2] + s4[3]);
}

// First valid item at or after i in this CTA's sequence.  Warp 0 walks every
// index of the sequence once and reports the invalid ones.
__device__ __forceinline__ int next_valid(const AttnParams& ap, int i, bool report) {
  for (; i < ap.n_items; i += gridDim.x) {
    if (get_item(ap, i).valid) break;
    if (report && ap.status) atomicOr(ap.status, kStatusBadShape);
  }
  return i;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, AttnParams ap) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                   // the next item's Q
  uint8_t* sK = sQ + kTile;             // [kKStages]
  uint8_t* sV = sK + kKStages * kTile;  // [kVStages]
  float* xmax = reinterpret_cast<float*>(sV + kVStages * kTile);  // [tile & 1][half][row]
  float* xsum = xmax + 2 * 2 * kRows;                        // [item & 1][half][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(xsum + 2 * 2 * kRows);
  uint64_t* q_full = bars + 0;    // Q tile in shared memory
  uint64_t* q_empty = bars + 1;   // Q tile copied to TMEM
  uint64_t* qt_full = bars + 2;   // [2] Q in the TMEM buffer
  uint64_t* qt_free = bars + 4;   // [2] the last S that read the TMEM buffer done
  uint64_t* k_full = bars + 6;    // [kKStages]
  uint64_t* k_empty = bars + 9;   // [kKStages]
  uint64_t* v_full = bars + 12;   // [kVStages]
  uint64_t* v_empty = bars + 14;  // [kVStages]
  uint64_t* s_full = bars + 16;   // [2] S buffer computed
  uint64_t* p_full = bars + 18;   // [2] P written over the S buffer
  uint64_t* l_full = bars + 20;   // [2] partial sums of the item in xsum
  uint64_t* o_ready = bars + 22;  // P·V of a tile complete
  uint64_t* o_done = bars + 23;   // the item's last P·V complete
  uint64_t* o_free = bars + 24;   // O of the item read by the epilogue
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 25);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kSm = 32 * kSoftmaxWarps;
  constexpr int kEpi = 32 * kEpiWarps;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, kEpi);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qt_full[i], kEpi);
      mbar_init(&qt_free[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kSm);
      mbar_init(&l_full[i], kSm);
    }
    mbar_init(o_ready, 1);
    mbar_init(o_done, 1);
    mbar_init(o_free, kEpi);
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
  const uint32_t tQ0 = tbase, tS0 = tbase + 128, tO0 = tbase + 384;
  auto fail = [&]() {
    *abort_flag = 1;
    if (ap.status) atomicOr(ap.status, kStatusTimeout);
  };

  if (warp <= 1) {
    // warp 0: Q (one item ahead) and K; warp 1: V
    if (lane == 0) {
      const bool is_k = warp == 0;
      bool ok = true;
      // Q tile of the n-th item (index i); the buffer is free once the
      // previous item's Q is in TMEM
      auto load_q = [&](int i, uint32_t n) -> bool {
        const Item it = get_item(ap, i);
        if (*abort_flag || !mbar_wait(q_empty, (n & 1) ^ 1u)) return false;
        mbar_arrive_expect_tx(q_full, kTile);
        for (int half = 0; half < 2; ++half)
          tma_load_2d(&tmQ, q_full, sQ + half * kHalf, it.head * kHD + half * 64,
                      it.t.tok0 + it.t.q0);
        return true;
      };
      const int n_st = is_k ? kKStages : kVStages;
      uint32_t n_it = 0, g = 0, st = 0, ph = 1;  // ring slot and the parity its wait takes
      int ci = next_valid(ap, blockIdx.x, is_k);
      if (is_k && ci < ap.n_items) ok = load_q(ci, 0);
      while (ok && ci < ap.n_items) {
        const Item it = get_item(ap, ci);
        const int ni = next_valid(ap, ci + gridDim.x, is_k);
        const int* bt = ap.block_tab + static_cast<long long>(it.t.clip) * ap.max_pages;
        uint64_t* full = is_k ? k_full : v_full;
        uint64_t* empty = is_k ? k_empty : v_empty;
        uint8_t* ring = is_k ? sK : sV;
        const CUtensorMap* tm = is_k ? &tmK : &tmV;
        for (int j = 0; j < it.n_tiles; ++j, ++g) {
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
          if (++st == static_cast<uint32_t>(n_st)) {
            st = 0;
            ph ^= 1u;
          }
          if (is_k && j == 0 && ni < ap.n_items && !load_q(ni, n_it + 1)) {
            ok = false;
            break;
          }
        }
        ci = ni;
        ++n_it;
      }
      if (!ok) fail();
    }
  } else if (warp == 2) {
    // the whole warp runs this role (warp-uniform values); one elected lane
    // issues each tcgen05 instruction
    auto wait = [&](uint64_t* bar, uint32_t par) -> bool {
      return __all_sync(0xFFFFFFFFu, !*abort_flag && mbar_wait(bar, par));
    };
    {
      const bool bf = H16Traits<T>::kBf16;
      const uint32_t idS128 = f16_instr_desc(kRows, 128, bf);
      const uint32_t idS64 = f16_instr_desc(kRows, 64, bf);
      const uint32_t idPV = f16_instr_desc(kRows, kHD, bf) | (1u << 16);  // B (V) MN-major
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV);
      // S(g) = Q·K(g)ᵀ into S buffer g & 1, Q from TMEM buffer qb, K from ring
      // slot g % kKStages
      auto issue_s = [&](uint32_t g, int keys, int qb) -> bool {
        const int st = g & 1;
        const uint32_t kst = g % kKStages, kph = (g / kKStages) & 1;
        if (!wait(&k_full[kst], kph)) return false;
        tc_fence_after();
        const uint32_t id = keys == 128 ? idS128 : idS64;
#pragma unroll
        for (int ks = 0; ks < kHD / 16; ++ks)
          mma_f16_ts_e(tS0 + st * 128, tQ0 + qb * 64 + ks * 8,
                       sw128_kmajor_desc(ka + kst * kTile + (ks >> 2) * kHalf + (ks & 3) * 32), id,
                       ks > 0 ? 1u : 0u);
        mma_commit_e(&s_full[st]);
        mma_commit_e(&k_empty[kst]);
        return true;
      };
      // first S of the n-th item (Q in TMEM buffer n & 1)
      auto issue_first_s = [&](const Item& it, uint32_t n, uint32_t g) -> bool {
        if (!wait(&qt_full[n & 1], (n >> 1) & 1)) return false;
        tc_fence_after();
        if (!issue_s(g, tile_keys(it, 0), n & 1)) return false;
        if (it.n_tiles == 1) mma_commit_e(&qt_free[n & 1]);
        return true;
      };
      bool ok = true;
      uint32_t cq = 0, g = 0;
      int j = 0;
      int ci = next_valid(ap, blockIdx.x, false);
      Item cur{};
      if (ci < ap.n_items) {
        cur = get_item(ap, ci);
        ok = issue_first_s(cur, 0, 0);
      }
      // Issue order: S(0), S(1), P·V(0), S(2), P·V(1), ... across items.  The
      // first S of item n+1 waits for the epilogue to have read item n-1 (its
      // partial sums share a buffer with item n+1's).
      while (ok && ci < ap.n_items) {
        const bool last = j + 1 == cur.n_tiles;
        const uint32_t o_par = (cq & 1) ^ 1u;  // o_free completion of item cq-1
        int ni = ci;
        Item nxt{};
        if (!last) {
          ok = issue_s(g + 1, tile_keys(cur, j + 1), cq & 1);
          if (ok && j + 2 == cur.n_tiles) mma_commit_e(&qt_free[cq & 1]);
        } else {
          ni = next_valid(ap, ci + gridDim.x, false);
          if (ni < ap.n_items) {
            nxt = get_item(ap, ni);
            ok = wait(o_free, o_par) && issue_first_s(nxt, cq + 1, g + 1);
          }
        }
        const int st = g & 1;
        if (!ok || !wait(&p_full[st], (g >> 1) & 1) || !wait(&v_full[st], (g >> 1) & 1) ||
            (j == 0 && !wait(o_free, o_par))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int keys = tile_keys(cur, j);
        // P for keys 0-63 in S columns 0-31, for keys 64-127 in columns 64-95
        for (int ks = 0; ks < keys / 16; ++ks)
          mma_f16_ts_e(tO0, tS0 + st * 128 + (ks >> 2) * 64 + (ks & 3) * 8,
                       sw128_mn_desc(va + st * kTile + ks * 16 * 128, kHalf, 1024), idPV,
                       (j > 0 || ks > 0) ? 1u : 0u);
        mma_commit_e(&v_empty[st]);
        mma_commit_e(o_ready);
        if (last) mma_commit_e(o_done);
        ++g;
        if (!last) {
          ++j;
        } else {
          ci = ni;
          cur = nxt;
          ++cq;
          j = 0;
        }
      }
      if (!ok && lane == 0) fail();
    }
  } else if (warp < 3 + kSoftmaxWarps) {
    // softmax: half hf of the keys (and of the O columns), row r
    const int hf = (warp - 3) / 4;
    const int quarter = warp & 3;  // TMEM lanes 32*quarter.. are this warp's
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tO = tO0 + lane_off + hf * 64;
    const float scale = ap.scale_log2;
    uint32_t n_it = 0, g = 0;
    bool ok = true;
    for (int i = next_valid(ap, blockIdx.x, false); ok && i < ap.n_items;
         i = next_valid(ap, i + gridDim.x, false), ++n_it) {
      const Item it = get_item(ap, i);
      const int pos = it.t.q0 + r;
      const int len = it.t.len;
      float m_used = -INFINITY, l = 0.0f;
      for (int j = 0; j < it.n_tiles; ++j, ++g) {
        const int st = g & 1;
        const int keys = tile_keys(it, j);
        const int key0 = j * kKeys + hf * 64;      // first key of this thread's half
        const bool active = hf * 64 < keys;         // a 64-key tile has no second half
        const int lim = min(pos, len - 1) - key0;  // keys key0 + i visible for i <= lim
        const uint32_t tS = tS0 + st * 128 + lane_off + hf * 64;
        const bool got = !*abort_flag && mbar_wait(&s_full[st], (g >> 1) & 1);
        tc_fence_after();
        float pm = -INFINITY;
        uint32_t u[64];  // this half's 64 scores, kept in registers across the exchange
        if (got && active) {
          tmem_ld_x64(tS, u);
          mask64(u, lim);
          pm = max64(u);
        }
        xmax[(st * 2 + hf) * kRows + r] = pm;
        if (!bar_and(1, kSm, got)) {  // also publishes xmax
          ok = false;
          break;
        }
        const float mx_s = fmaxf(pm, xmax[(st * 2 + (hf ^ 1)) * kRows + r]) * scale;  // scale > 0
        const bool grow = mx_s > m_used + kRescaleLog2;
        float alpha = 1.0f;
        if (grow) {
          alpha = ex2_approx(m_used - mx_s);  // 0 on the first tile (m_used = -inf)
          m_used = mx_s;
        }
        if (j > 0 && __any_sync(0xFFFFFFFFu, grow)) {
          // the previous tile's P·V must be complete before O is rescaled
          if (!__all_sync(0xFFFFFFFFu, mbar_wait(o_ready, (g - 1) & 1))) {
            if (lane == 0) fail();
          } else {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
              float o[32];
              tmem_ld32(tO + c * 32, o);
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] *= alpha;
              tmem_st32(tO + c * 32, o);
            }
          }
        }
        l *= alpha;
        if (active) {
          // P for keys [key0, key0+64) -> TMEM columns [0, 32) of this half of
          // the S buffer
          const float neg = m_used == -INFINITY ? 0.0f : -m_used;
          uint32_t w[32];
          exp_pack64<T>(u, scale, neg, w, l);
          tmem_st_x32(tS, w);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[st]);
      }
      if (!ok) break;
      xsum[((n_it & 1) * 2 + hf) * kRows + r] = l;
      mbar_arrive(&l_full[n_it & 1]);  // release: the epilogue reads xsum after its wait
    }
    if (!ok && lane == 0) fail();
  } else {
    // epilogue: row r of Q (into TMEM, one item ahead) and of O (to memory)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tO = tO0 + lane_off;
    // Q of the n-th item: shared memory (TMA, 128-byte swizzle) -> TMEM buffer n & 1
    auto copy_q = [&](uint32_t n) -> bool {
      const int b = n & 1;
      const bool got = !*abort_flag && mbar_wait(q_full, n & 1) &&
                       mbar_wait(&qt_free[b], ((n >> 1) & 1) ^ 1u);
      if (!__all_sync(0xFFFFFFFFu, got)) return false;
      tc_fence_after();
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        const uint8_t* qrow = sQ + half * kHalf + r * 128;
        uint32_t w[32];
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint4 v = *reinterpret_cast<const uint4*>(qrow + ((ch ^ (r & 7)) << 4));
          w[4 * ch] = v.x;
          w[4 * ch + 1] = v.y;
          w[4 * ch + 2] = v.z;
          w[4 * ch + 3] = v.w;
        }
        tmem_st32(tQ0 + b * 64 + lane_off + half * 32, w);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(q_empty);
      mbar_arrive(&qt_full[b]);
      return true;
    };
    bool ok = true;
    uint32_t n_it = 0;
    int ci = next_valid(ap, blockIdx.x, false);
    if (ci < ap.n_items) ok = copy_q(0);
    while (ok && ci < ap.n_items) {
      const Item it = get_item(ap, ci);
      const int ni = next_valid(ap, ci + gridDim.x, false);
      if (ni < ap.n_items && !copy_q(n_it + 1)) {
        ok = false;
        break;
      }
      const bool got = !*abort_flag && mbar_wait(o_done, n_it & 1) &&
                       mbar_wait(&l_full[n_it & 1], (n_it >> 1) & 1);
      if (!__all_sync(0xFFFFFFFFu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int pos = it.t.q0 + r;
      const float* ls = xsum + (n_it & 1) * 2 * kRows;
      const float inv = 1.0f / (ls[r] + ls[kRows + r]);
      T* dst = static_cast<T*>(ap.out) + (static_cast<long long>(it.t.tok0) + pos) * ap.ldo +
               static_cast<long long>(it.head) * kHD;
#pragma unroll 1
      for (int c = 0; c < kHD / 32; ++c) {
        float o[32];
        tmem_ld32(tO + c * 32, o);
        if (pos < it.t.len) {
          alignas(16) T ov[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = f2h<T>(o[e] * inv);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            reinterpret_cast<uint4*>(dst + c * 32)[e] = reinterpret_cast<const uint4*>(ov)[e];
        }
      }
      tc_fence_before();
      mbar_arrive(o_free);
      ci = ni;
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
  if (hd != kHD || nkvh <= 0 || nqh % nkvh || kv.page_size != kPage) return (int)cudaErrorInvalidValue;
  CUtensorMap tq, tk, tv;
  const long long kv_rows = static_cast<long long>(kv_pages) * nkvh * kPage;
  int rc = make_tmap_2d(&tq, qkv, bf16, ldq, q_rows, ldq, 64, kRows);
  if (!rc) rc = make_tmap_2d(&tk, kv.k, bf16, kHD, kv_rows, kHD, 64, kPage);
  if (!rc) rc = make_tmap_2d(&tv, kv.v, bf16, kHD, kv_rows, kHD, 64, kPage);
  if (rc) return rc;
  AttnParams ap{};
  ap.tiles = tiles;
  ap.n_items = n_tiles * nqh;
  ap.nq = nqh;
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
