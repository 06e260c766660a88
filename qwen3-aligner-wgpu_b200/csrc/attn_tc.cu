// (e) Causal GQA flash attention on the tcgen05 tensor cores.
//
// softmax(q·kᵀ / sqrt(128)) · v over keys 0..=pos of the same clip
// (src/cpu_decoder.rs:327-412), for the decoder prefill over the paged K/V
// cache.  A work item is one K/V head of one clip and 128 query positions
// q0..q0+127: two M=128 tiles, one per query head of the GQA pair (heads
// 2·kvh and 2·kvh+1), which share every K/V tile the item reads.  The kernel
// is persistent: one CTA per SM walks items blockIdx.x, +gridDim.x, ... of a
// list sorted longest first, and its pipeline runs on across item boundaries
// (the next item's Q and K/V pages load while the current one finishes).
//
//   warp 0     TMA: the item's two Q tiles, then its K and V tiles (128 keys =
//              two 64-token pages, or one page for a last half tile) into a
//              two-stage ring with separate K and V barriers;
//   warp 1     TMEM allocation and the MMAs, issued by one thread:
//                S_h = Q_h·Kᵀ   (M=128, N=128 or 64 keys, K=128 dims) -> TMEM
//                O_h += P_h·V   (M=128, N=128 dims, K=keys), P_h read from
//                               TMEM, V as an MN-major operand straight from
//                               the pages as TMA stored them;
//              in the order S_0(j), P_1·V(j-1), S_1(j), P_0·V(j), so that the
//              tensor cores work on one head while the other head's softmax
//              runs;
//   warps 2-5  softmax of head 0, warps 6-9 of head 1, one thread per query
//              row: the row of S from TMEM, causal/length mask, running max
//              and sum in f32, p = 2^(s·scale·log2e - m), P packed to 16 bits
//              back into the first half of the row's S columns (the MMA
//              reads it there), O rescaled in TMEM only when the row max grew
//              by more than 2^8 since the last rescale (the final O / sum is
//              exact for any reference max), O / sum written out at the end.
//
// TMEM (512 columns): S_0 [0,128), S_1 [128,256), O_0 [256,384), O_1 [384,512).
// tcgen05.mma instructions from one thread execute in issue order, so S_h(j+1)
// may overwrite P_h(j) once P_h(j)·V has been issued; every tcgen05.commit
// tracks all earlier MMAs, so a row's O may be rescaled once S_h(j) is
// complete.  Barriers: q_full/q_empty, k_full/k_empty, v_full/v_empty (ring),
// s_full[h] (S_h ready), p_full[h] (P_h written, O_h rescaled; 128 arrivals),
// o_done[h] (last P_h·V of the item done).  Every wait is bounded (sm100.cuh).
// No cluster multicast: each CTA loads its own tiles.
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
constexpr int kThreads = 320;  // 10 warps
constexpr uint32_t kTile = kRows * kHD * 2;  // 32 KB: a Q, K or V tile
constexpr uint32_t kHalf = kTile / 2;        // 16 KB: one 64-column block of a tile
constexpr uint32_t kPageBytes = kHalf / 2;   // 8 KB: 64 rows of one block
constexpr size_t kSmem = 1024 + 6 * kTile + 256;  // 2x Q, 2x K, 2x V, barriers
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

// One key tile of one query row (this thread's TMEM lane): read S, mask,
// update the running max / sum, rescale O if needed, write P over S.
template <typename T, int NK>
__device__ __forceinline__ void softmax_tile(uint32_t tS, uint32_t tO, int key0, int pos, int len,
                                             bool need_mask, float scale, bool first,
                                             float& m_used, float& l) {
  float s[NK];
#pragma unroll
  for (int c = 0; c < NK / 32; ++c)
    tmem_ld32(tS + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
  if (need_mask) {
#pragma unroll
    for (int i = 0; i < NK; ++i) {
      const int key = key0 + i;
      if (key > pos || key >= len) s[i] = -INFINITY;
    }
  }
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < NK; ++i) mx = fmaxf(mx, s[i]);
  const float mx_s = mx * scale;  // scale > 0: the max of the scaled row
  const bool grow = mx_s > m_used + kRescaleLog2;
  float alpha = 1.0f;
  if (grow) {
    alpha = ex2_approx(m_used - mx_s);  // 0 on the first tile (m_used = -inf)
    m_used = mx_s;
  }
  if (!first && __any_sync(0xFFFFFFFFu, grow)) {
#pragma unroll 1
    for (int c = 0; c < kHD / 32; ++c) {
      float o[32];
      tmem_ld32(tO + c * 32, o);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] *= alpha;
      tmem_st32(tO + c * 32, o);
    }
  }
  const float neg = m_used == -INFINITY ? 0.0f : -m_used;
  float sum = 0.0f;
#pragma unroll
  for (int c = 0; c < NK / 64; ++c) {
    uint32_t w[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const float p0 = ex2_approx(fmaf(s[c * 64 + 2 * e], scale, neg));
      const float p1 = ex2_approx(fmaf(s[c * 64 + 2 * e + 1], scale, neg));
      sum += p0 + p1;
      w[e] = pack2<T>(p0, p1);
    }
    tmem_st32(tS + c * 32, w);
  }
  l = l * alpha + sum;
  tmem_wait_st();
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, AttnParams ap) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;            // [2 heads]
  uint8_t* sK = sQ + 2 * kTile;  // [2 stages]
  uint8_t* sV = sK + 2 * kTile;  // [2 stages]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * kTile);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;   // [2 stages]
  uint64_t* k_empty = bars + 4;  // [2 stages]
  uint64_t* v_full = bars + 6;   // [2 stages]
  uint64_t* v_empty = bars + 8;  // [2 stages]
  uint64_t* s_full = bars + 10;  // [2 heads]
  uint64_t* p_full = bars + 12;  // [2 heads]
  uint64_t* o_done = bars + 14;  // [2 heads]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
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
  if (warp == 1) tmem_alloc(tslot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  auto fail = [&]() {
    *abort_flag = 1;
    if (ap.status) atomicOr(ap.status, kStatusTimeout);
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t n_it = 0, g = 0;
      bool ok = true;
      for (int i = blockIdx.x; ok && i < ap.n_items; i += gridDim.x) {
        const Item it = get_item(ap, i);
        if (!it.valid) {
          if (ap.status) atomicOr(ap.status, kStatusBadShape);
          continue;
        }
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
        const int* bt = ap.block_tab + static_cast<long long>(it.t.clip) * ap.max_pages;
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
          if (!mbar_wait(&k_empty[st], ph)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[st], npg * 2 * kPageBytes);
          for (int pg = 0; pg < npg; ++pg)
            for (int half = 0; half < 2; ++half)
              tma_load_2d(&tmK, &k_full[st], sK + st * kTile + half * kHalf + pg * kPageBytes,
                          half * 64, rows[pg]);
          if (!mbar_wait(&v_empty[st], ph)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[st], npg * 2 * kPageBytes);
          for (int pg = 0; pg < npg; ++pg)
            for (int half = 0; half < 2; ++half)
              tma_load_2d(&tmV, &v_full[st], sV + st * kTile + half * kHalf + pg * kPageBytes,
                          half * 64, rows[pg]);
        }
        ++n_it;
      }
      if (!ok) fail();
    }
  } else if (warp == 1) {
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
        for (int ks = 0; ks < keys / 16; ++ks)
          mma_f16_ts(tO[h], tS[h] + ks * 8,
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
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          const int keys = tile_keys(it, j);
          if (!mbar_wait(&k_full[st], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(0, st, keys);
          if (j > 0) {
            if (!mbar_wait(&p_full[1], (g - 1) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(1, st ^ 1, prev_keys, j > 1);
            mma_commit(&v_empty[st ^ 1]);
          }
          issue_s(1, st, keys);
          mma_commit(&k_empty[st]);
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
    const int h = (warp - 2) >> 2;  // query head of the pair
    const int quarter = warp & 3;   // TMEM lanes 32*quarter.. are this warp's
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tbase + h * 128 + lane_off;
    const uint32_t tO = tbase + 256 + h * 128 + lane_off;
    uint32_t n_it = 0, g = 0;
    bool ok = true;
    for (int i = blockIdx.x; ok && i < ap.n_items; i += gridDim.x) {
      const Item it = get_item(ap, i);
      if (!it.valid) continue;
      const int pos = it.t.q0 + r;
      float m_used = -INFINITY, l = 0.0f;
      for (int j = 0; j < it.n_tiles; ++j, ++g) {
        const int keys = tile_keys(it, j);
        const int key0 = j * kKeys;
        // warp-uniform: tcgen05.ld/st and the vote inside are warp-collective
        const bool got = !*abort_flag && mbar_wait(&s_full[h], g & 1);
        if (!__all_sync(0xFFFFFFFFu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const bool need_mask = key0 + keys - 1 > it.t.q0 || key0 + keys > it.t.len;
        if (keys == kKeys)
          softmax_tile<T, kKeys>(tS, tO, key0, pos, it.t.len, need_mask, ap.scale_log2, j == 0,
                                 m_used, l);
        else
          softmax_tile<T, kPage>(tS, tO, key0, pos, it.t.len, need_mask, ap.scale_log2, j == 0,
                                 m_used, l);
        tc_fence_before();
        mbar_arrive(&p_full[h]);
      }
      if (!ok) break;
      const bool got = !*abort_flag && mbar_wait(&o_done[h], n_it & 1);
      if (!__all_sync(0xFFFFFFFFu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = 1.0f / l;
      T* dst = static_cast<T*>(ap.out) + (static_cast<long long>(it.t.tok0) + pos) * ap.ldo +
               static_cast<long long>(it.kvh * 2 + h) * kHD;
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
      ++n_it;
    }
    if (!ok && lane == 0) fail();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
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
