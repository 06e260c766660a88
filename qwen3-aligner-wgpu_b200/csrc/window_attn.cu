// (b) The audio tower's windowed self-attention on the tcgen05 tensor cores.
//
// Every query of a window attends to every key of the same window, full
// softmax, no mask inside the window (src/audio_encoder.rs:574-627; the
// reference's GPU tower, src/audio_encoder_gpu.rs:1497-1547).  Windows are
// runs of at most 128 packed audio tokens (104 for the checkpoint's
// n_window_infer = 800); head dim 64.
//
// A work item is one (window, head).  One CTA of four warps runs items one
// after another, and three CTAs share an SM, so one CTA's softmax overlaps
// another's loads and MMAs.  Per item:
//   - TMA brings Q (128 rows from the window's first token), K and V (NK rows)
//     of the head into shared memory as 128-byte swizzled K-major tiles.  The
//     rows past the window belong to the next window (or read as zero past the
//     last token); their keys are masked and their query rows never stored;
//   - warp 0 issues S = Q·Kᵀ (M=128, N=NK, K=64) into TMEM columns [0, NK);
//   - each thread owns one query row (TMEM lane = row): it reads its NK
//     scores with one TMEM load, masks the keys past the window to -inf,
//     takes the row max, the exponentials 2^((s - max)·log2(e)/8) and their
//     f32 sum, and writes P packed to 16 bits over columns [0, NK/2);
//   - warp 0 issues O = P·V (M=128, N=64, K=NK; P from TMEM, V an MN-major
//     operand) into columns [64, 128), which only the scores (already in
//     registers) used;
//   - every thread stores its row of O / sum as 16 bits.
// Q and K of the next item are loaded as soon as this item's S is complete,
// V as soon as its O is.
//
// Every mbarrier wait is bounded (sm100.cuh): a wait that runs out sets the
// timeout bit of the status word and an abort flag, the CTA leaves its loop
// at the next item boundary, waits (bounded) for its own loads in flight and
// frees its TMEM.  No TMA load uses cluster multicast.
#include <algorithm>

#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "sm100.cuh"
#include "tma_host.h"

namespace qa {

namespace {

constexpr int kWHD = 64;         // head dim
constexpr int kWRows = 128;      // query rows per item (one M=128 tile)
constexpr int kWThreads = 128;   // four warps, one TMEM lane quarter each
constexpr int kWCtasPerSm = 3;   // 3 x 128 TMEM columns, 3 x ~46 KB shared memory
constexpr uint32_t kWTmemCols = 128;
constexpr uint32_t kWRowBytes = kWHD * 2;  // 128 B: one swizzle row per token
constexpr float kWLog2e = 1.4426950408889634f;

__host__ __device__ constexpr uint32_t w_q_bytes() { return kWRows * kWRowBytes; }
__host__ __device__ constexpr uint32_t w_kv_bytes(int nk) { return nk * kWRowBytes; }
__host__ __device__ constexpr size_t w_smem(int nk) {
  return 1024 + w_q_bytes() + 2 * w_kv_bytes(nk) + 128;
}

// One TMEM load of 112 consecutive 32-bit columns of this warp's lanes (x64 +
// x32 + x16 behind one wait, so no use of r is scheduled before the data).
__device__ __forceinline__ void tmem_ld_x112(uint32_t taddr, uint32_t (&r)[112]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%112];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95}, [%113];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111}, [%114];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111])
      : "r"(taddr + 0u), "r"(taddr + 64u), "r"(taddr + 96u)
      : "memory");
}

// Store 56 consecutive 32-bit columns of this warp's lanes (x32 + x16 + x8; no wait).
__device__ __forceinline__ void tmem_st_x56(uint32_t taddr, const uint32_t (&w)[56]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34};\n\t"
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%1], {%35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50};\n\t"
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%2], {%51, %52, %53, %54, %55, %56, %57, %58};\n\t"
      :
      : "r"(taddr + 0u), "r"(taddr + 32u), "r"(taddr + 48u), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7]), "r"(w[8]), "r"(w[9]), "r"(w[10]), "r"(w[11]), "r"(w[12]), "r"(w[13]), "r"(w[14]), "r"(w[15]), "r"(w[16]), "r"(w[17]), "r"(w[18]), "r"(w[19]), "r"(w[20]), "r"(w[21]), "r"(w[22]), "r"(w[23]), "r"(w[24]), "r"(w[25]), "r"(w[26]), "r"(w[27]), "r"(w[28]), "r"(w[29]), "r"(w[30]), "r"(w[31]), "r"(w[32]), "r"(w[33]), "r"(w[34]), "r"(w[35]), "r"(w[36]), "r"(w[37]), "r"(w[38]), "r"(w[39]), "r"(w[40]), "r"(w[41]), "r"(w[42]), "r"(w[43]), "r"(w[44]), "r"(w[45]), "r"(w[46]), "r"(w[47]), "r"(w[48]), "r"(w[49]), "r"(w[50]), "r"(w[51]), "r"(w[52]), "r"(w[53]), "r"(w[54]), "r"(w[55])
      : "memory");
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

struct WinParams {
  const int2* windows;  // (first packed token, length) per window
  int n_items;          // windows x heads
  int nh;
  int dm;               // model width: q at column h*64, k at dm + h*64, v at 2*dm + h*64
  void* out;            // [T][dm]
  float scale_log2;     // log2(e) / sqrt(64)
  unsigned* status;
};

template <typename T, int NK>
__global__ void __launch_bounds__(kWThreads, kWCtasPerSm)
    window_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                     WinParams wp) {
  static_assert(NK == 112 || NK == 128, "keys per window tile");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + w_q_bytes();
  uint8_t* sV = sK + w_kv_bytes(NK);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + w_kv_bytes(NK));
  uint64_t* bar_qk = bars + 0;  // Q and K of an item in shared memory
  uint64_t* bar_v = bars + 1;   // V of an item in shared memory
  uint64_t* bar_s = bars + 2;   // S = Q·Kᵀ complete
  uint64_t* bar_o = bars + 3;   // O = P·V complete
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKV);
  }
  if (warp == 0) tmem_alloc(tslot, kWTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_wait();  // the previous kernel's results are visible from here
  pdl_trigger();

  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const int r = warp * 32 + lane;  // this thread's query row within the item
  const bool bf = H16Traits<T>::kBf16;
  const uint32_t idS = f16_instr_desc(kWRows, NK, bf);
  const uint32_t idPV = f16_instr_desc(kWRows, kWHD, bf) | (1u << 16);  // B (V) MN-major
  const uint64_t dq = sw128_kmajor_desc(smem_u32(sQ));
  const uint64_t dk = sw128_kmajor_desc(smem_u32(sK));
  const uint64_t dv = sw128_mn_desc(smem_u32(sV), w_kv_bytes(NK), 1024);  // + 128 per 16 keys
  auto fail = [&]() {
    *abort_flag = 1;
    if (wp.status) atomicOr(wp.status, kStatusTimeout);
  };
  // a bounded wait taken by a whole warp; skipped once the CTA has aborted
  auto wait = [&](uint64_t* bar, uint32_t par) -> bool {
    const bool ok = __all_sync(0xFFFFFFFFu, !*abort_flag && mbar_wait(bar, par));
    if (!ok && lane == 0) fail();
    return ok;
  };
  // loads issued by thread 0 (counted so that an abort can wait for them)
  uint32_t qk_issued = 0, v_issued = 0;
  auto load_qk = [&](int item) {
    const int2 win = wp.windows[item / wp.nh];
    const int h = item % wp.nh;
    mbar_arrive_expect_tx(bar_qk, w_q_bytes() + w_kv_bytes(NK));
    tma_load_2d(&tmQ, bar_qk, sQ, h * kWHD, win.x);
    tma_load_2d(&tmKV, bar_qk, sK, wp.dm + h * kWHD, win.x);
    ++qk_issued;
  };
  auto load_v = [&](int item) {
    const int2 win = wp.windows[item / wp.nh];
    const int h = item % wp.nh;
    mbar_arrive_expect_tx(bar_v, w_kv_bytes(NK));
    tma_load_2d(&tmKV, bar_v, sV, 2 * wp.dm + h * kWHD, win.x);
    ++v_issued;
  };
  if (threadIdx.x == 0 && static_cast<int>(blockIdx.x) < wp.n_items) {
    load_qk(blockIdx.x);
    load_v(blockIdx.x);
  }

  uint32_t k = 0;  // items done by this CTA
  for (int item = blockIdx.x; item < wp.n_items; item += gridDim.x, ++k) {
    const int2 win = wp.windows[item / wp.nh];
    const int h = item % wp.nh;
    const int len = win.y;
    const int next = item + static_cast<int>(gridDim.x);
    const uint32_t ph = k & 1;
    // S = Q·Kᵀ into columns [0, NK)
    if (warp == 0 && wait(bar_qk, ph)) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < kWHD / 16; ++ks)
        mma_f16_e(tbase, dq + ks * 2, dk + ks * 2, idS, ks > 0 ? 1u : 0u);
      mma_commit_e(bar_s);
    }
    bool ok = wait(bar_s, ph);
    tc_fence_after();
    // Q and K are free: the next item's go in now
    if (ok && threadIdx.x == 0 && next < wp.n_items) load_qk(next);
    // softmax of row r over the window's keys
    float sum = 0.0f;
    {
      uint32_t u[NK];
      if constexpr (NK == 112) {
        tmem_ld_x112(tbase + lane_off, u);
      } else {
        tmem_ld_x128(tbase + lane_off, u);
      }
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < NK; ++j) {
        if (j >= len) u[j] = __float_as_uint(-INFINITY);
        m4[j & 3] = fmaxf(m4[j & 3], __uint_as_float(u[j]));
      }
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      // 2^((s - max) * log2(e) / 8) = e^((s - max) / sqrt(64)): one FMA + ex2 each
      const float neg = -mx * wp.scale_log2;
      float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      uint32_t w[NK / 2];
#pragma unroll
      for (int e = 0; e < NK / 2; ++e) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(u[2 * e]), wp.scale_log2, neg));
        const float p1 = ex2_approx(fmaf(__uint_as_float(u[2 * e + 1]), wp.scale_log2, neg));
        s4[e & 3] += p0 + p1;
        w[e] = pack2<T>(p0, p1);
      }
      sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      if constexpr (NK == 112) {
        tmem_st_x56(tbase + lane_off, w);
      } else {
        tmem_st_x64(tbase + lane_off, w);
      }
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();  // P of all 128 rows is in TMEM
    tc_fence_after();
    // O = P·V into columns [64, 128)
    if (warp == 0 && wait(bar_v, ph)) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < NK / 16; ++ks)
        mma_f16_ts_e(tbase + 64, tbase + ks * 8, dv + ks * 128, idPV, ks > 0 ? 1u : 0u);
      mma_commit_e(bar_o);
    }
    ok = wait(bar_o, ph);
    tc_fence_after();
    if (ok && threadIdx.x == 0 && next < wp.n_items) load_v(next);
    // this row of O / sum
    {
      uint32_t o[64];
      tmem_ld_x64(tbase + lane_off + 64, o);
      if (ok && r < len) {
        const float inv = 1.0f / sum;
        T* dst = static_cast<T*>(wp.out) + (static_cast<long long>(win.x) + r) * wp.dm + h * kWHD;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 v;
          v.x = pack2<T>(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
          v.y = pack2<T>(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
          v.z = pack2<T>(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
          v.w = pack2<T>(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
          reinterpret_cast<uint4*>(dst)[c] = v;
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // O read by every row before the next S overwrites its columns
    tc_fence_after();
    if (*abort_flag) break;
  }
  // after an abort, wait (bounded) for this CTA's own loads still in flight
  // (the last load issued on a barrier completes after every earlier one)
  if (threadIdx.x == 0 && *abort_flag) {
    if (qk_issued) mbar_wait(bar_qk, (qk_issued - 1) & 1);
    if (v_issued) mbar_wait(bar_v, (v_issued - 1) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, kWTmemCols);
  }
}

template <typename T, int NK>
int launch_window(const CUtensorMap& tq, const CUtensorMap& tkv, const WinParams& wp,
                  cudaStream_t s) {
  auto kern = window_tc_kernel<T, NK>;
  const size_t smem = w_smem(NK);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  const int grid = std::min(wp.n_items, kWCtasPerSm * device_sm_count());
  e = launch_pdl(kern, dim3(grid), dim3(kWThreads), smem, s, tq, tkv, wp);
  return (int)e;
}

}  // namespace

int window_attention(const void* qkv, long long T, int dm, int nh, int hd, const int2* windows,
                     int n_windows, int max_window, void* out, bool bf16, unsigned* status,
                     cudaStream_t s) {
  if (n_windows <= 0) return 0;
  if (hd != kWHD || dm != nh * hd || max_window <= 0 || max_window > 128 || T <= 0)
    return (int)cudaErrorInvalidValue;
  const int nk = max_window <= 112 ? 112 : 128;
  CUtensorMap tq, tkv;
  int rc = make_tmap_2d(&tq, qkv, bf16, 3LL * dm, T, 3LL * dm, 64, kWRows);
  if (!rc) rc = make_tmap_2d(&tkv, qkv, bf16, 3LL * dm, T, 3LL * dm, 64, nk);
  if (rc) return rc;
  WinParams wp{};
  wp.windows = windows;
  wp.n_items = n_windows * nh;
  wp.nh = nh;
  wp.dm = dm;
  wp.out = out;
  wp.scale_log2 = (1.0f / sqrtf(static_cast<float>(hd))) * kWLog2e;
  wp.status = status;
  if (bf16)
    return nk == 112 ? launch_window<__nv_bfloat16, 112>(tq, tkv, wp, s)
                     : launch_window<__nv_bfloat16, 128>(tq, tkv, wp, s);
  return nk == 112 ? launch_window<__half, 112>(tq, tkv, wp, s)
                   : launch_window<__half, 128>(tq, tkv, wp, s);
}

}  // namespace qa
