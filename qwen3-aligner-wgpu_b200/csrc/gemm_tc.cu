// tcgen05 / TMEM / TMA GEMM with fused epilogues (see gemm_tc.cuh).
//
// One CTA computes a 128 x BN tile.  Warp roles (192 threads):
//   warp 0      TMA producer: streams 128x64 A and BNx64 B tiles (128B swizzle)
//               into a STAGES-deep shared-memory ring, one mbarrier per slot;
//   warp 1      allocates the TMEM accumulator and issues tcgen05.mma
//               (M=128, N=BN, K=16) from one thread; tcgen05.commit frees a
//               ring slot when the MMAs reading it retire;
//   warps 2..5  epilogue: tcgen05.ld 32x32b pulls one accumulator row per
//               thread (warp w reads TMEM lanes 32*(w%4) .. +31), applies the
//               fused epilogue and stores to global memory.
// Nothing here uses cluster multicast: each CTA loads its own tiles.
#include "gemm_tc.cuh"
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

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int col) {
  uint32_t u = __float_as_uint(v);
  uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(ord) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(col));
}

template <typename T>
__device__ __forceinline__ void store16_row(T* dst, const float (&v)[32], int ncols) {
  if (ncols == 32 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    alignas(16) T tmp[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) tmp[i] = f2h<T>(v[i]);
    const uint4* s = reinterpret_cast<const uint4*>(tmp);
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = s[i];
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

template <int BN, typename T>
__device__ __forceinline__ void epilogue(const EpiParams& ep, uint32_t tmem_row, int row, int M,
                                         int n0, int N) {
  if (ep.mode == EPI_SWIGLU16) {
    // gate in columns [0, BN/2), up in [BN/2, BN) of this tile
    constexpr int H = BN / 2;
    T* out = static_cast<T*>(ep.out);
#pragma unroll 1
    for (int c0 = 0; c0 < H; c0 += 32) {
      float g[32], u[32];
      tmem_ld32(tmem_row + c0, g);
      tmem_ld32(tmem_row + H + c0, u);
      if (row < M) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float gh = round16<T>(g[i]);
          const float uh = round16<T>(u[i]);
          const float silu = gh / (1.0f + expf(-gh));
          g[i] = silu * uh;
        }
        const int oc = n0 / 2 + c0;
        const int nc = min(32, N / 2 - oc);
        if (nc > 0) store16_row<T>(out + (long long)row * ep.ldo + oc, g, nc);
      }
    }
    return;
  }

  if (ep.mode == EPI_ARGMAX) {
    unsigned long long best = 0ull;
    float* out = static_cast<float*>(ep.out);
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      float v[32];
      tmem_ld32(tmem_row + c0, v);
      if (row < M) {
        const int nc = min(min(32, BN - c0), N - (n0 + c0));
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (i >= nc) break;
          const float x = v[i];
          if (out) out[(long long)row * ep.ldo + n0 + c0 + i] = x;
          if (x == x) {  // NaN never wins, as in a strict `>` scan
            const unsigned long long k = argmax_key(x, n0 + c0 + i);
            best = k > best ? k : best;
          }
        }
      }
    }
    if (row < M && best != 0ull) atomicMax(ep.keys + row, best);
    return;
  }

#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    float v[32];
    tmem_ld32(tmem_row + c0, v);
    if (row >= M) continue;
    const int col = n0 + c0;
    const int nc = min(min(32, BN - c0), N - col);  // BN need not be a multiple of 32
    if (nc <= 0) continue;
    if (ep.bias) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nc) v[i] += ep.bias[col + i];
    }
    switch (ep.mode) {
      case EPI_STORE16: {
        if (ep.act == ACT_GELU) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
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
        break;
      }
      case EPI_RESID32: {
        float* dst = static_cast<float*>(ep.out) + (long long)row * ep.ldo + col;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < nc) dst[i] += v[i];
        break;
      }
      case EPI_STORE32: {
        int orow = row;
        if (ep.row_map) orow = ep.row_map[row];
        if (orow < 0) break;
        if (ep.pe) {
          const float* pe = ep.pe + (long long)(row % ep.pe_period) * N + col;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < nc) v[i] += pe[i];
        }
        float* dst = static_cast<float*>(ep.out) + (long long)orow * ep.ldo + col;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < nc) dst[i] = v[i];
        break;
      }
      default:
        break;
    }
  }
}

template <int BN, typename T>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   int M, int N, int K, EpiParams ep) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes);
  uint64_t* empty = full + S;
  uint64_t* accb = empty + S;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accb + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM;
  const int n0 = blockIdx.x * BN;
  const int nkb = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(accb, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tslot, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1u)) {
          if (ep.status) atomicOr(ep.status, kStatusTimeout);
          break;
        }
        mbar_arrive_expect_tx(&full[s], Cfg::kABytes + Cfg::kBBytes);
        tma_load_2d(&tmA, &full[s], sA + s * Cfg::kABytes, kb * kBK, m0);
        tma_load_2d(&tmB, &full[s], sB + s * Cfg::kBBytes, kb * kBK, n0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = f16_instr_desc(kBM, BN, H16Traits<T>::kBf16);
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        if (!mbar_wait(&full[s], ph)) {
          if (ep.status) atomicOr(ep.status, kStatusTimeout);
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
          mma_f16(tbase, da, db, idesc, (kb > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&empty[s]);
      }
      if (ok) mma_commit(accb);
    }
  } else {
    const int q = warp & 3;
    const bool ok = mbar_wait(accb, 0);
    tc_fence_after();
    if (ok) {
      const int row = m0 + q * 32 + lane;
      const uint32_t trow = tbase + (static_cast<uint32_t>(q * 32) << 16);
      epilogue<BN, T>(ep, trow, row, M, n0, N);
    } else if (lane == 0 && ep.status) {
      atomicOr(ep.status, kStatusTimeout);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, Cfg::kTmemCols);
  }
}

template <int BN, typename T>
int launch(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
           const EpiParams& ep, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, /*bf16=*/H16Traits<T>::kBf16, K, M, lda, kBK, kBM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, B, H16Traits<T>::kBf16, K, N, ldb, kBK, BN);
  if (rc) return rc;
  auto kern = gemm_tc_kernel<BN, T>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::kSmem);
  if (e != cudaSuccess) return (int)e;
  dim3 grid((N + BN - 1) / BN, (M + kBM - 1) / kBM);
  kern<<<grid, 192, Cfg::kSmem, stream>>>(ta, tb, M, N, K, ep);
  return (int)cudaGetLastError();
}

}  // namespace

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
  const int bn = force_bn ? force_bn : gemm_pick_bn(N);
  if (ep.mode == EPI_SWIGLU16 && ((N % bn) || (bn % 64))) return (int)cudaErrorInvalidValue;
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

}  // namespace qa
