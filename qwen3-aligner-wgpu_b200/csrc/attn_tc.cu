// (e) Causal GQA flash attention on the tcgen05 tensor cores.
//
// softmax(q·kᵀ / sqrt(128)) · v over keys 0..=pos of the same clip
// (src/cpu_decoder.rs:327-412), for the decoder prefill over the paged K/V
// cache.  A work item is one K/V head of one clip and 128 query positions
// q0..q0+127: the two query heads A and B of that K/V head (GQA group of two),
// one M=128 tile each, sharing every K/V tile.  The kernel is persistent: one
// CTA per SM walks items blockIdx.x, +gridDim.x, ...; items are ordered longest
// clip first with a clip's blocks adjacent, so the K/V pages a CTA reads were
// usually just read by a neighbour and come from L2.
//
//   warp 0       TMA: Q of heads A and B (one shared-memory tile each) and the
//                K tiles (128 keys = two 64-token pages, or one for a last half
//                tile);
//   warp 1       TMA: the V tiles;
//   warp 2       TMEM allocation and the MMAs (the whole warp, one elected lane
//                issuing):
//                  S_h(j) = Q_h·K(j)ᵀ  (M=128, N=128 or 64 keys, K=128 dims),
//                                     both operands from shared memory;
//                  O_h += P_h(j)·V(j) (N=128 dims, K=keys), P_h read from TMEM,
//                                     V an MN-major operand straight from the
//                                     pages;
//                in the order P·V_A(j), S_A(j+1), P·V_B(j), S_B(j+1), ... so
//                that one head's MMAs run while the other head's softmax does;
//   warps 3-6    softmax of head A, warps 7-10 of head B: one query row per
//                thread (TMEM lane = row).  Each SM sub-partition thus runs one
//                softmax warp of each head, on independent tiles.  A thread
//                keeps the running max and sum in f32, writes P packed to 16
//                bits over its S columns (keys 0-63 at columns 0-31, keys
//                64-127 at 64-95), and rescales its O row in TMEM only when the
//                row max grew by more than 2^8 since the last rescale (O / sum
//                is exact for any reference max);
//   warps 11-14  epilogue: after an item's last P·V of each head, O / sum row by
//                row into the output, then O is released for the next item.
//
// TMEM (512 columns): S_A [0,128), S_B [128,256), O_A [256,384), O_B
// [384,512).  tcgen05.mma instructions from one thread execute in issue order
// (S_h(j+1) may overwrite P_h(j) once P_h(j)·V has been issued), and every
// tcgen05.commit tracks all earlier MMAs.  Every mbarrier wait is bounded
// (sm100.cuh) and warp-uniform.  No cluster multicast: each CTA loads its own
// tiles.
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
constexpr int kSoftmaxWarps = 8;  // 4 per head
constexpr int kEpiWarps = 4;
constexpr int kThreads = (3 + kSoftmaxWarps + kEpiWarps) * 32;  // 15 warps
constexpr uint32_t kTile = kRows * kHD * 2;  // 32 KB: a Q, K or V tile
constexpr uint32_t kHalf = kTile / 2;        // 16 KB: one 64-column block of a tile
constexpr uint32_t kPageBytes = kHalf / 2;   // 8 KB: 64 rows of one block
constexpr int kStages = 2;                   // K and V ring depth
constexpr uint32_t kSumBytes = 2 * 2 * kRows * 4;  // row sums [item parity][head][row]
constexpr int kMaxStaged = 128;  // work items of one CTA whose descriptors sit in shared memory
constexpr uint32_t kOutStage = 4096;  // per epilogue warp: 32 rows x 64 output columns
constexpr size_t kSmem =
    1024 + (2 + 2 * kStages) * kTile + kSumBytes + 256 + kMaxStaged * 32 + kEpiWarps * kOutStage;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;  // rescale O when the row max grows by > 2^8

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
  int kvh;      // K/V head; query heads 2 kvh (A) and 2 kvh + 1 (B)
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

// The CTA's items i = blockIdx.x + k * gridDim.x are derived once, at the
// start, into shared memory (`staged`, index k), so no role waits on a global
// load at an item boundary.
__device__ __forceinline__ const Item& staged_item(const Item* staged, int i) {
  return staged[(i - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x)];
}

// First valid item at or after i in this CTA's sequence.
__device__ __forceinline__ int next_valid(const AttnParams& ap, const Item* staged, int i) {
  for (; i < ap.n_items; i += gridDim.x)
    if (staged_item(staged, i).valid) break;
  return i;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, AttnParams ap) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                 // [head]
  uint8_t* sK = sQ + 2 * kTile;       // [kStages]
  uint8_t* sV = sK + kStages * kTile;  // [kStages]
  float* xsum = reinterpret_cast<float*>(sV + kStages * kTile);  // [item & 1][head][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(xsum + 2 * 2 * kRows);
  uint64_t* q_full = bars + 0;    // [head] Q tile in shared memory
  uint64_t* q_free = bars + 2;    // [head] the item's last S of the head done
  uint64_t* k_full = bars + 4;    // [kStages]
  uint64_t* k_empty = bars + 6;   // [kStages]
  uint64_t* v_full = bars + 8;    // [kStages]
  uint64_t* v_empty = bars + 10;  // [kStages]
  uint64_t* s_full = bars + 12;   // [head] S computed
  uint64_t* p_full = bars + 14;   // [head] P written over S
  uint64_t* o_ready = bars + 16;  // [head] P·V of a tile complete
  uint64_t* o_done = bars + 18;   // [head] the item's last P·V complete
  uint64_t* o_free = bars + 20;   // [head] O read by the epilogue
  uint64_t* l_full = bars + 22;   // [item & 1][head] row sums in xsum
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 26);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  Item* staged = reinterpret_cast<Item*>(bars + 32);  // [kMaxStaged]
  static_assert(sizeof(Item) <= 32, "staged item size");
  uint8_t* ostage = reinterpret_cast<uint8_t*>(bars + 32) + kMaxStaged * 32;  // [kEpiWarps]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kSmHead = 32 * kSoftmaxWarps / 2;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_free[i], 1);
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kSmHead);
      mbar_init(&o_ready[i], 1);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_free[i], 32 * kEpiWarps);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&l_full[i], kSmHead);
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
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();
  {  // this CTA's item descriptors (at most kMaxStaged: the launcher sizes the grid)
    const int n_seq = static_cast<int>(blockIdx.x) < ap.n_items
                          ? (ap.n_items - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                          : 0;
    for (int k = threadIdx.x; k < n_seq; k += blockDim.x) {
      const Item it = get_item(ap, static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x));
      staged[k] = it;
      if (!it.valid && ap.status) atomicOr(ap.status, kStatusBadShape);
    }
    __syncthreads();
  }
  const uint32_t tS0 = tbase, tO0 = tbase + 256;  // S_h at tS0 + 128 h, O_h at tO0 + 128 h
  auto fail = [&]() {
    *abort_flag = 1;
    if (ap.status) atomicOr(ap.status, kStatusTimeout);
  };
  // bounded wait taken by a whole warp, warp-uniform result
  auto wait = [&](uint64_t* bar, uint32_t par) -> bool {
    return __all_sync(0xFFFFFFFFu, !*abort_flag && mbar_wait(bar, par));
  };

  if (warp <= 1) {
    // warp 0: Q of both heads and K; warp 1: V
    if (lane == 0) {
      const bool is_k = warp == 0;
      bool ok = true;
      uint32_t n_it = 0, g = 0;
      for (int ci = next_valid(ap, staged, blockIdx.x); ok && ci < ap.n_items;
           ci = next_valid(ap, staged, ci + gridDim.x), ++n_it) {
        const Item it = staged_item(staged, ci);
        if (is_k) {
          // Q_h of this item once the previous item's last S_h is done
          for (int h = 0; h < 2 && ok; ++h) {
            if (*abort_flag || !mbar_wait(&q_free[h], (n_it & 1) ^ 1u)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&q_full[h], kTile);
            for (int half = 0; half < 2; ++half)
              tma_load_2d(&tmQ, &q_full[h], sQ + h * kTile + half * kHalf,
                          (2 * it.kvh + h) * kHD + half * 64, it.t.tok0 + it.t.q0);
          }
          if (!ok) break;
        }
        const int* bt = ap.block_tab + static_cast<long long>(it.t.clip) * ap.max_pages;
        uint64_t* full = is_k ? k_full : v_full;
        uint64_t* empty = is_k ? k_empty : v_empty;
        uint8_t* ring = is_k ? sK : sV;
        const CUtensorMap* tm = is_k ? &tmK : &tmV;
        // page ids are read one tile ahead: the next tile's load is in flight
        // while this one waits for its ring slot
        int nxt[2] = {bt[0], tile_keys(it, 0) > kPage ? bt[1] : 0};
        for (int j = 0; j < it.n_tiles; ++j, ++g) {
          const int st = g & 1;
          const int npg = tile_keys(it, j) / kPage;
          const int cur[2] = {nxt[0], nxt[1]};
          if (j + 1 < it.n_tiles) {
            nxt[0] = bt[2 * (j + 1)];
            nxt[1] = tile_keys(it, j + 1) > kPage ? bt[2 * (j + 1) + 1] : 0;
          }
          int rows[2] = {0, 0};
          for (int pg = 0; pg < npg; ++pg) {
            int page = cur[pg];
            if (page < 0 || page >= ap.kv_pages) {
              if (ap.status) atomicOr(ap.status, kStatusBadShape);
              page = 0;
            }
            rows[pg] = (page * ap.nkv + it.kvh) * kPage;
          }
          if (*abort_flag || !mbar_wait(&empty[st], ((g >> 1) & 1) ^ 1u)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[st], npg * 2 * kPageBytes);
          for (int pg = 0; pg < npg; ++pg)
            for (int half = 0; half < 2; ++half)
              tma_load_2d(tm, &full[st], ring + st * kTile + half * kHalf + pg * kPageBytes,
                          half * 64, rows[pg]);
        }
      }
      if (!ok) fail();
    }
  } else if (warp == 2) {
    // the whole warp runs this role; one elected lane issues each tcgen05 op
    const bool bf = H16Traits<T>::kBf16;
    const uint32_t idS128 = f16_instr_desc(kRows, 128, bf);
    const uint32_t idS64 = f16_instr_desc(kRows, 64, bf);
    const uint32_t idPV = f16_instr_desc(kRows, kHD, bf) | (1u << 16);  // B (V) MN-major
    const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK), va = smem_u32(sV);
    // S_h = Q_h·K(g)ᵀ into S_h; K in ring slot g & 1
    auto issue_s = [&](int h, uint32_t g, int keys) {
      const uint32_t id = keys == kKeys ? idS128 : idS64;
      const uint64_t dq = sw128_kmajor_desc(qa + h * kTile);
      const uint64_t dk = sw128_kmajor_desc(ka + (g & 1) * kTile);
#pragma unroll
      for (int ks = 0; ks < kHD / 16; ++ks) {
        const uint32_t off = (ks >> 2) * (kHalf >> 4) + (ks & 3) * 2;  // 16-byte units
        mma_f16_e(tS0 + h * 128, dq + off, dk + off, id, ks > 0 ? 1u : 0u);
      }
      mma_commit_e(&s_full[h]);
    };
    bool ok = true;
    uint32_t n_it = 0, g = 0;
    int ci = next_valid(ap, staged, blockIdx.x);
    Item cur{};
    if (ci < ap.n_items) {
      cur = staged_item(staged, ci);
      ok = wait(&q_full[0], 0) && wait(&q_full[1], 0) && wait(&k_full[0], 0);
      if (ok) {
        tc_fence_after();
        for (int h = 0; h < 2; ++h) {
          issue_s(h, 0, tile_keys(cur, 0));
          if (cur.n_tiles == 1) mma_commit_e(&q_free[h]);
        }
        mma_commit_e(&k_empty[0]);
      }
    }
    int j = 0;
    while (ok && ci < ap.n_items) {
      const bool last = j + 1 == cur.n_tiles;
      int ni = ci;
      Item nxt{};
      if (last) {
        ni = next_valid(ap, staged, ci + gridDim.x);
        if (ni < ap.n_items) nxt = staged_item(staged, ni);
      }
      const bool has_next = !last || ni < ap.n_items;
      const Item& sit = last ? nxt : cur;  // owner of the next S
      const int sj = last ? 0 : j + 1;
      const uint32_t sn = last ? n_it + 1 : n_it;  // its item count
      const int st = g & 1;
      for (int h = 0; h < 2 && ok; ++h) {
        // the previous item's O_h read by the epilogue (its sums, too) before
        // this item's first P·V_h and before the next item's first S_h
        if ((j == 0 || (last && has_next)) && n_it > 0 && !wait(&o_free[h], (n_it - 1) & 1)) {
          ok = false;
          break;
        }
        if (!wait(&p_full[h], g & 1) || (h == 0 && !wait(&v_full[st], (g >> 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // P_h for keys 0-63 in S_h columns 0-31, for keys 64-127 in columns 64-95
        const uint32_t tp = tS0 + h * 128;
        const uint64_t dv = sw128_mn_desc(va + st * kTile, kHalf, 1024);  // + 128 per 16 keys
        const int keys = tile_keys(cur, j);
        for (int ks = 0; ks < keys / 16; ++ks)
          mma_f16_ts_e(tO0 + h * 128, tp + (ks >> 2) * 64 + (ks & 3) * 8, dv + ks * 128, idPV,
                       (j > 0 || ks > 0) ? 1u : 0u);
        mma_commit_e(&o_ready[h]);
        if (last) mma_commit_e(&o_done[h]);
        if (h == 1) mma_commit_e(&v_empty[st]);
        if (has_next) {
          // the next S_h (this item's tile j+1 or the next item's first tile)
          if ((last && !wait(&q_full[h], sn & 1)) ||
              (h == 0 && !wait(&k_full[(g + 1) & 1], ((g + 1) >> 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(h, g + 1, tile_keys(sit, sj));
          if (sj + 1 == sit.n_tiles) mma_commit_e(&q_free[h]);
          if (h == 1) mma_commit_e(&k_empty[(g + 1) & 1]);
        }
      }
      ++g;
      if (!last) {
        ++j;
      } else {
        ci = ni;
        cur = nxt;
        ++n_it;
        j = 0;
      }
    }
    if (!ok && lane == 0) fail();
  } else if (warp < 3 + kSoftmaxWarps) {
    // softmax: head h, row r (one per thread), all keys of each tile
    const int h = (warp - 3) / 4;
    const int quarter = warp & 3;  // TMEM lanes 32*quarter.. are this warp's
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tS0 + h * 128 + lane_off;
    const uint32_t tO = tO0 + h * 128 + lane_off;
    const float scale = ap.scale_log2;
    uint32_t n_it = 0, g = 0;
    bool ok = true;
    for (int i = next_valid(ap, staged, blockIdx.x); ok && i < ap.n_items;
         i = next_valid(ap, staged, i + gridDim.x), ++n_it) {
      const Item it = staged_item(staged, i);
      const int pos = it.t.q0 + r;
      const int len = it.t.len;
      float m_used = -INFINITY, l = 0.0f;
      for (int j = 0; j < it.n_tiles; ++j, ++g) {
        const int nch = tile_keys(it, j) / 64;      // 64-key chunks in this tile
        const int lim = min(pos, len - 1) - j * kKeys;  // keys j*128 + i visible for i <= lim
        if (!wait(&s_full[h], g & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // max pass; the last chunk's scores stay in registers
        uint32_t u[64];
        float pm = -INFINITY;
        for (int c = 0; c < nch; ++c) {
          tmem_ld_x64(tS + c * 64, u);
          mask64(u, lim - c * 64);
          pm = fmaxf(pm, max64(u));
        }
        const float mx_s = pm * scale;  // scale > 0
        const bool grow = mx_s > m_used + kRescaleLog2;
        float alpha = 1.0f;
        if (grow) {
          alpha = ex2_approx(m_used - mx_s);  // 0 on the first tile (m_used = -inf)
          m_used = mx_s;
        }
        if (j > 0 && __any_sync(0xFFFFFFFFu, grow)) {
          // the previous tile's P·V must be complete before O is rescaled
          if (!wait(&o_ready[h], (g - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < kHD / 32; ++c) {
            float o[32];
            tmem_ld32(tO + c * 32, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(tO + c * 32, o);
          }
        }
        l *= alpha;
        // exponentials, last chunk first (its scores are in u); chunk c's P
        // goes to columns 64c .. 64c + 31, which only chunk c's scores held
        const float neg = m_used == -INFINITY ? 0.0f : -m_used;
        for (int c = nch - 1; c >= 0; --c) {
          if (c != nch - 1) {
            tmem_ld_x64(tS + c * 64, u);
            mask64(u, lim - c * 64);
          }
          uint32_t w[32];
          exp_pack64<T>(u, scale, neg, w, l);
          tmem_st_x32(tS + c * 64, w);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[h]);
      }
      if (!ok) break;
      xsum[((n_it & 1) * 2 + h) * kRows + r] = l;
      mbar_arrive(&l_full[(n_it & 1) * 2 + h]);  // release: the epilogue reads xsum after its wait
    }
    if (!ok && lane == 0) fail();
  } else {
    // epilogue: row r of O_A and O_B
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t n_it = 0;
    bool ok = true;
    for (int i = next_valid(ap, staged, blockIdx.x); ok && i < ap.n_items;
         i = next_valid(ap, staged, i + gridDim.x), ++n_it) {
      const Item it = staged_item(staged, i);
      const int pos = it.t.q0 + r;
      for (int h = 0; h < 2; ++h) {
        if (!wait(&o_done[h], n_it & 1) || !wait(&l_full[(n_it & 1) * 2 + h], (n_it >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float inv = 1.0f / xsum[((n_it & 1) * 2 + h) * kRows + r];
        T* dst = static_cast<T*>(ap.out) + (static_cast<long long>(it.t.tok0) + pos) * ap.ldo +
                 static_cast<long long>(2 * it.kvh + h) * kHD;
        const uint32_t tO = tO0 + h * 128 + lane_off;
        // the row's 128 values, scaled and packed, then O_h goes back to the
        // MMA warp before any of them is stored
        uint32_t w[kHD / 2];
#pragma unroll
        for (int c = 0; c < kHD / 32; ++c) {
          float o[32];
          tmem_ld32(tO + c * 32, o);
#pragma unroll
          for (int e = 0; e < 16; ++e) w[c * 16 + e] = cvt2_rn<T>(make_float2(o[2 * e] * inv, o[2 * e + 1] * inv));
        }
        tc_fence_before();
        mbar_arrive(&o_free[h]);
        // 64 columns per staged block, stored four whole row segments at a time
        uint8_t* st = ostage + quarter * kOutStage;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            stage_unit(st, u, make_uint4(w[b * 32 + 4 * u], w[b * 32 + 4 * u + 1], w[b * 32 + 4 * u + 2],
                                         w[b * 32 + 4 * u + 3]));
          flush_rows<T>(st, pos < it.t.len ? dst : nullptr, b * 64, b * 64 + 32);
        }
      }
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
  // two query heads per K/V head (the model's GQA group), 128-dim heads, 64-token pages
  if (hd != kHD || nkvh <= 0 || nqh != 2 * nkvh || kv.page_size != kPage)
    return (int)cudaErrorInvalidValue;
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
  // persistent, one CTA per SM; more CTAs (queued) only when an SM's share of
  // items would exceed what its shared memory stages
  const int grid = std::max(std::min(ap.n_items, device_sm_count()),
                            (ap.n_items + kMaxStaged - 1) / kMaxStaged);
  if (bf16) {
    auto k = attn_tc_kernel<__nv_bfloat16>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
    if (e != cudaSuccess) return (int)e;
    e = launch_pdl(k, dim3(grid), dim3(kThreads), kSmem, s, tq, tk, tv, ap);
    if (e != cudaSuccess) return (int)e;
  } else {
    auto k = attn_tc_kernel<__half>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
    if (e != cudaSuccess) return (int)e;
    e = launch_pdl(k, dim3(grid), dim3(kThreads), kSmem, s, tq, tk, tv, ap);
    if (e != cudaSuccess) return (int)e;
  }
  return (int)cudaGetLastError();
}

}  // namespace qa
