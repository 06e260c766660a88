// (e) Attention kernels of the alignment path.
//
// causal_attention: the decoder's causal GQA prefill attention
//   softmax(q·kᵀ / sqrt(128)) · v over keys 0..=pos of the same clip
//   (src/cpu_decoder.rs:327-412; GPU flat/slabbed paths src/decoder.rs:1373-1600),
//   flash-style: one CTA owns 64 query positions of one clip for the `rep` (= 2)
//   query heads that share a K/V head, streams 64-key pages of the paged cache
//   through a double-buffered cp.async pipeline and keeps the softmax online
//   (running max / sum per row, warp-shuffle reductions inside each quad).
//   Pages are the cache's own 64-token pages, so one K/V tile = one page.
// window_attention: the audio tower's windowed attention, every query of a
//   104-token window attending to the whole window (src/audio_encoder.rs:574-627);
//   one CTA per (window, head) holds the window in shared memory.
//
// Both use mma.sync m16n8k16 (f16/bf16 in, f32 accumulate) with ldmatrix from
// XOR-swizzled shared memory.  Rows past a clip's or window's end are
// zero-filled on load (0·NaN from stale cache rows would otherwise poison the
// P·V product) and masked to -inf in the scores.
#include <algorithm>

#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace qa {

namespace {

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t s = smem_u32(smem);
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                 uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of 16-byte chunk `c` of row `r` in a tile whose rows hold
// CPR chunks, XOR-swizzled so that 8 consecutive rows hit 8 distinct chunks.
template <int CPR>
__device__ __forceinline__ int swz(int r, int c) {
  return (r * CPR + (c ^ (r & 7))) * 16;
}

constexpr float kLog2e = 1.4426950408889634f;

// ======================================================================
// Decoder: causal GQA over the paged cache, HD = 128, 64 queries x rep heads.
// ======================================================================
template <typename T, int REP>
__global__ void __launch_bounds__(128 * REP)
    causal_attn_kernel(const T* __restrict__ qkv, long long ldq, int nqh, int nkvh,
                       const AttnTile* __restrict__ tiles, const int* __restrict__ block_tab,
                       int max_pages, PagedKV kv, T* __restrict__ out, float scale_log2) {
  constexpr int HD = 128, BQ = 64, BK = 64, CPR = HD * 2 / 16;  // 16 chunks per row
  constexpr int NT = 128 * REP;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;                         // [REP*BQ][HD]
  uint8_t* sK = sQ + REP * BQ * HD * 2;       // [2][BK][HD]
  uint8_t* sV = sK + 2 * BK * HD * 2;         // [2][BK][HD]

  const AttnTile tl = tiles[blockIdx.x];
  const int kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hsel = warp / 4;            // which query head of the group
  const int head = kvh * REP + hsel;
  const int wrow = (warp % 4) * 16;     // first row of this warp inside the tile
  const int len = tl.len;
  const int q_hi = min(tl.q0 + BQ, len);  // queries q0 .. q_hi-1 are real
  const int n_tiles = (q_hi + BK - 1) / BK;
  const int* bt = block_tab + static_cast<long long>(tl.clip) * max_pages;

  // ---- Q tile (all REP heads), zero past the clip end
  for (int i = threadIdx.x; i < REP * BQ * CPR; i += NT) {
    const int c = i % CPR, rr = i / CPR;
    const int hs = rr / BQ, r = rr % BQ;
    const int q = tl.q0 + r;
    const bool ok = q < len;
    const T* src = qkv + (static_cast<long long>(tl.tok0) + (ok ? q : 0)) * ldq +
                   static_cast<long long>(kvh * REP + hs) * HD + c * 8;
    cp_async16(sQ + hs * BQ * HD * 2 + swz<CPR>(r, c), src, ok);
  }
  auto load_kv = [&](int j, int stage) {
    const int page = bt[j];
    const long long base = (static_cast<long long>(page) * nkvh + kvh) * kv.page_size * HD;
    const T* kp = static_cast<const T*>(kv.k) + base;
    const T* vp = static_cast<const T*>(kv.v) + base;
    uint8_t* dk = sK + stage * BK * HD * 2;
    uint8_t* dv = sV + stage * BK * HD * 2;
    for (int i = threadIdx.x; i < BK * CPR; i += NT) {
      const int c = i % CPR, r = i / CPR;
      const bool ok = j * BK + r < len;
      cp_async16(dk + swz<CPR>(r, c), kp + (ok ? r : 0) * HD + c * 8, ok);
      cp_async16(dv + swz<CPR>(r, c), vp + (ok ? r : 0) * HD + c * 8, ok);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  uint32_t qf[HD / 16][4];
  const int g = lane >> 2, tq = lane & 3;
  const int qrow0 = tl.q0 + wrow + g;  // query position of rows g and g+8

  for (int j = 0; j < n_tiles; ++j) {
    const int stage = j & 1;
    if (j + 1 < n_tiles) load_kv(j + 1, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
      const uint8_t* qb = sQ + hsel * BQ * HD * 2;
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks) {
        const int r = wrow + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(qf[ks], qb + swz<CPR>(r, c));
      }
    }
    const uint8_t* kb = sK + stage * BK * HD * 2;
    const uint8_t* vb = sV + stage * BK * HD * 2;
    // ---- S = Q Kᵀ (16 rows x 64 keys per warp)
    float s[BK / 8][4];
#pragma unroll
    for (int i = 0; i < BK / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
      for (int np = 0; np < BK / 16; ++np) {
        uint32_t b[4];
        const int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(b, kb + swz<CPR>(r, c));
        mma16816<T>(s[2 * np], qf[ks], b[0], b[1]);
        mma16816<T>(s[2 * np + 1], qf[ks], b[2], b[3]);
      }
    }
    // ---- scale, mask, online softmax
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < BK / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = j * BK + nt * 8 + 2 * tq + (e & 1);
        const int qp = qrow0 + (e >> 1) * 8;
        float v = s[nt][e] * scale_log2;
        if (key > qp || key >= len) v = -INFINITY;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xFFFFFFFFu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xFFFFFFFFu, mx[h], 2));
      const float mnew = fmaxf(m_r[h], mx[h]);
      const float base = mnew == -INFINITY ? 0.f : mnew;
      alpha[h] = exp2f(m_r[h] - base);
      m_r[h] = mnew;
      mx[h] = base;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < BK / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(s[nt][e] - mx[e >> 1]);
        s[nt][e] = p;
        rs[e >> 1] += p;
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rs[h] += __shfl_xor_sync(0xFFFFFFFFu, rs[h], 1);
      rs[h] += __shfl_xor_sync(0xFFFFFFFFu, rs[h], 2);
      l_r[h] = l_r[h] * alpha[h] + rs[h];
    }
#pragma unroll
    for (int dt = 0; dt < HD / 8; ++dt) {
      o[dt][0] *= alpha[0];
      o[dt][1] *= alpha[0];
      o[dt][2] *= alpha[1];
      o[dt][3] *= alpha[1];
    }
    // ---- O += P V
#pragma unroll
    for (int ks = 0; ks < BK / 16; ++ks) {
      uint32_t a[4];
      a[0] = pack2<T>(s[2 * ks][0], s[2 * ks][1]);
      a[1] = pack2<T>(s[2 * ks][2], s[2 * ks][3]);
      a[2] = pack2<T>(s[2 * ks + 1][0], s[2 * ks + 1][1]);
      a[3] = pack2<T>(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        uint32_t b[4];
        const int r = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dp * 2 + (lane >> 4);
        ldsm_x4_t(b, vb + swz<CPR>(r, c));
        mma16816<T>(o[2 * dp], a, b[0], b[1]);
        mma16816<T>(o[2 * dp + 1], a, b[2], b[3]);
      }
    }
    __syncthreads();  // the next iteration's prefetch overwrites this stage
  }

  // ---- normalise and store
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int qp = qrow0 + h * 8;
    if (qp >= len) continue;
    const float inv = 1.0f / l_r[h];
    T* dst = out + (static_cast<long long>(tl.tok0) + qp) * (static_cast<long long>(nqh) * HD) +
             static_cast<long long>(head) * HD;
#pragma unroll
    for (int dt = 0; dt < HD / 8; ++dt) {
      const uint32_t pk = pack2<T>(o[dt][2 * h] * inv, o[dt][2 * h + 1] * inv);
      *reinterpret_cast<uint32_t*>(dst + dt * 8 + 2 * tq) = pk;
    }
  }
}

// ======================================================================
// Audio tower: windowed attention, HD = 64, window <= 128.  Persistent: each
// CTA (8 warps x 16 query rows) walks items (window, head) = blockIdx.x,
// +gridDim.x, ... with the next item's Q, K and V prefetched by cp.async into
// the other of two shared-memory stages while the current item computes.
// ======================================================================
constexpr int kWinHD = 64, kWinW = 128, kWinCPR = kWinHD * 2 / 16;  // 8 chunks per row
constexpr int kWinStage = 3 * kWinW * kWinHD * 2;                  // Q, K, V: 48 KB
constexpr int kWinSmem = 2 * kWinStage;

template <typename T>
__device__ __forceinline__ void window_load(const T* __restrict__ qkv, int dm, int2 win, int head,
                                            uint8_t* st) {
  const long long ld = 3LL * dm;
  uint8_t* sQ = st;
  uint8_t* sK = st + kWinW * kWinHD * 2;
  uint8_t* sV = sK + kWinW * kWinHD * 2;
  for (int i = threadIdx.x; i < kWinW * kWinCPR; i += 256) {
    const int c = i % kWinCPR, r = i / kWinCPR;
    const bool ok = r < win.y;
    const T* row = qkv + (static_cast<long long>(win.x) + (ok ? r : 0)) * ld + head * kWinHD + c * 8;
    cp_async16(sQ + swz<kWinCPR>(r, c), row, ok);
    cp_async16(sK + swz<kWinCPR>(r, c), row + dm, ok);
    cp_async16(sV + swz<kWinCPR>(r, c), row + 2 * dm, ok);
  }
}

// One item: this warp's 16 query rows against the window's keys.
template <typename T>
__device__ __forceinline__ void window_item(const uint8_t* st, int2 win, int head, int dm,
                                            T* __restrict__ out, float scale_log2) {
  constexpr int HD = kWinHD, W = kWinW, CPR = kWinCPR;
  const uint8_t* sQ = st;
  const uint8_t* sK = st + W * HD * 2;
  const uint8_t* sV = sK + W * HD * 2;
  const int len = win.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wrow = warp * 16;
  if (wrow >= len) return;
  const int g = lane >> 2, tq = lane & 3;
  uint32_t qf[HD / 16][4];
#pragma unroll
  for (int ks = 0; ks < HD / 16; ++ks) {
    const int r = wrow + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int c = ks * 2 + (lane >> 4);
    ldsm_x4(qf[ks], sQ + swz<CPR>(r, c));
  }
  float s[W / 8][4];
#pragma unroll
  for (int i = 0; i < W / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < HD / 16; ++ks)
#pragma unroll
    for (int np = 0; np < W / 16; ++np) {
      uint32_t b[4];
      const int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
      const int c = ks * 2 + ((lane >> 3) & 1);
      ldsm_x4(b, sK + swz<CPR>(r, c));
      mma16816<T>(s[2 * np], qf[ks], b[0], b[1]);
      mma16816<T>(s[2 * np + 1], qf[ks], b[2], b[3]);
    }
  // raw scores: masked keys (past the window) at -inf, row max over the rest
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int nt = 0; nt < W / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int key = nt * 8 + 2 * tq + (e & 1);
      if (key >= len) s[nt][e] = -INFINITY;
      mx[e >> 1] = fmaxf(mx[e >> 1], s[nt][e]);
    }
  float rs[2] = {0.f, 0.f};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xFFFFFFFFu, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xFFFFFFFFu, mx[h], 2));
  }
  // 2^((s - max) * scale_log2) = e^((s - max) / sqrt(64)), one FMA + ex2 each
  const float neg[2] = {-mx[0] * scale_log2, -mx[1] * scale_log2};
#pragma unroll
  for (int nt = 0; nt < W / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float p = ex2_approx(fmaf(s[nt][e], scale_log2, neg[e >> 1]));
      s[nt][e] = p;
      rs[e >> 1] += p;
    }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    rs[h] += __shfl_xor_sync(0xFFFFFFFFu, rs[h], 1);
    rs[h] += __shfl_xor_sync(0xFFFFFFFFu, rs[h], 2);
  }
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < W / 16; ++ks) {
    uint32_t a[4];
    a[0] = pack2<T>(s[2 * ks][0], s[2 * ks][1]);
    a[1] = pack2<T>(s[2 * ks][2], s[2 * ks][3]);
    a[2] = pack2<T>(s[2 * ks + 1][0], s[2 * ks + 1][1]);
    a[3] = pack2<T>(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
    for (int dp = 0; dp < HD / 16; ++dp) {
      uint32_t b[4];
      const int r = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = dp * 2 + (lane >> 4);
      ldsm_x4_t(b, sV + swz<CPR>(r, c));
      mma16816<T>(o[2 * dp], a, b[0], b[1]);
      mma16816<T>(o[2 * dp + 1], a, b[2], b[3]);
    }
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = wrow + g + h * 8;
    if (r >= len) continue;
    const float inv = 1.0f / rs[h];
    T* dst = out + (static_cast<long long>(win.x) + r) * dm + head * HD;
#pragma unroll
    for (int dt = 0; dt < HD / 8; ++dt)
      *reinterpret_cast<uint32_t*>(dst + dt * 8 + 2 * tq) =
          pack2<T>(o[dt][2 * h] * inv, o[dt][2 * h + 1] * inv);
  }
}

template <typename T>
__global__ void __launch_bounds__(256, 2)
    window_attn_kernel(const T* __restrict__ qkv, int dm, int nh, const int2* __restrict__ windows,
                       int n_items, T* __restrict__ out, float scale_log2) {
  extern __shared__ __align__(128) uint8_t wsm[];
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();
  int i = blockIdx.x;
  if (i >= n_items) return;
  window_load<T>(qkv, dm, windows[i / nh], i % nh, wsm);
  cp_async_commit();
  for (int k = 0; i < n_items; i += gridDim.x, ++k) {
    uint8_t* cur = wsm + (k & 1) * kWinStage;
    const int nx = i + gridDim.x;
    if (nx < n_items) {  // the other stage was last read by item k-1 (behind the barrier below)
      window_load<T>(qkv, dm, windows[nx / nh], nx % nh, wsm + ((k + 1) & 1) * kWinStage);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    window_item<T>(cur, windows[i / nh], i % nh, dm, out, scale_log2);
    __syncthreads();  // the next prefetch overwrites this stage
  }
}

}  // namespace

int causal_attention(const void* qkv, long long ldq, int nqh, int nkvh, int hd,
                     const AttnTile* tiles, int n_tiles, const int* block_tab, int max_pages,
                     PagedKV kv, void* out, bool bf16, cudaStream_t s) {
  if (n_tiles <= 0) return 0;
  if (hd != 128 || nqh != 2 * nkvh || kv.page_size != 64) return (int)cudaErrorInvalidValue;
  constexpr int REP = 2;
  const size_t smem = (REP * 64 + 4 * 64) * 128 * 2;  // Q + 2x(K, V)
  const float sl2 = (1.0f / sqrtf(128.0f)) * kLog2e;
  dim3 grid(n_tiles, nkvh);
  if (bf16) {
    auto k = causal_attn_kernel<__nv_bfloat16, REP>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, 128 * REP, smem, s>>>(static_cast<const __nv_bfloat16*>(qkv), ldq, nqh, nkvh, tiles,
                                    block_tab, max_pages, kv, static_cast<__nv_bfloat16*>(out), sl2);
  } else {
    auto k = causal_attn_kernel<__half, REP>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, 128 * REP, smem, s>>>(static_cast<const __half*>(qkv), ldq, nqh, nkvh, tiles,
                                    block_tab, max_pages, kv, static_cast<__half*>(out), sl2);
  }
  return (int)cudaGetLastError();
}

int window_attention(const void* qkv, int dm, int nh, int hd, const int2* windows, int n_windows,
                     void* out, bool bf16, cudaStream_t s) {
  if (n_windows <= 0) return 0;
  if (hd != 64 || dm != nh * hd) return (int)cudaErrorInvalidValue;
  const float sl2 = (1.0f / sqrtf(64.0f)) * kLog2e;
  const int n_items = n_windows * nh;
  const int grid = std::min(n_items, 2 * device_sm_count());  // two CTAs (96 KB each) per SM
  if (bf16) {
    auto k = window_attn_kernel<__nv_bfloat16>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kWinSmem);
    if (e != cudaSuccess) return (int)e;
    e = launch_pdl(k, dim3(grid), dim3(256), kWinSmem, s, static_cast<const __nv_bfloat16*>(qkv), dm,
                   nh, windows, n_items, static_cast<__nv_bfloat16*>(out), sl2);
    if (e != cudaSuccess) return (int)e;
  } else {
    auto k = window_attn_kernel<__half>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kWinSmem);
    if (e != cudaSuccess) return (int)e;
    e = launch_pdl(k, dim3(grid), dim3(256), kWinSmem, s, static_cast<const __half*>(qkv), dm, nh,
                   windows, n_items, static_cast<__half*>(out), sl2);
    if (e != cudaSuccess) return (int)e;
  }
  return (int)cudaGetLastError();
}

}  // namespace qa
