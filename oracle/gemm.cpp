// TEST INFRASTRUCTURE (parity oracle / CPU baseline).
//
// f32 GEMM C = A · Bᵀ (+C), standing in for the `gemm` crate 0.18.2 the
// reference calls for every CPU projection (src/cpu_decoder.rs:583-610,
// src/cpu_tensor.rs:85-107, src/audio_encoder.rs:416-426).  The crate is a
// packed, register-blocked f32 FMA GEMM parallelised over all cores; this is a
// restatement of that algorithm family (pack A row panels and Bᵀ column
// panels, 6x16 register micro-tile, OpenMP over output tiles).  Summation order
// differs from the crate, which the reference itself allows
// (src/cpu_decoder.rs:8-12).
#include <omp.h>

#include <algorithm>

#include "common.h"

namespace orc {

namespace {

typedef float v8f __attribute__((vector_size(32)));

constexpr int MR = 6;
constexpr int NR = 16;
constexpr int MC = 96;
constexpr int NC = 256;
constexpr int KC = 256;

inline v8f load8(const float* p) {
  v8f v;
  std::memcpy(&v, p, 32);
  return v;
}
inline void store8(float* p, v8f v) { std::memcpy(p, &v, 32); }

// acc[MR][NR] = Σ_k Ap[k][r] * Bp[k][c]
inline void micro(const float* Ap, const float* Bp, int kc, float* out /* MR*NR */) {
  v8f c[MR][2];
  for (int r = 0; r < MR; ++r) c[r][0] = c[r][1] = v8f{0, 0, 0, 0, 0, 0, 0, 0};
  for (int k = 0; k < kc; ++k) {
    const v8f b0 = load8(Bp + k * NR);
    const v8f b1 = load8(Bp + k * NR + 8);
    const float* a = Ap + k * MR;
    for (int r = 0; r < MR; ++r) {
      const v8f av = v8f{a[r], a[r], a[r], a[r], a[r], a[r], a[r], a[r]};
      c[r][0] += av * b0;
      c[r][1] += av * b1;
    }
  }
  for (int r = 0; r < MR; ++r) {
    store8(out + r * NR, c[r][0]);
    store8(out + r * NR + 8, c[r][1]);
  }
}

}  // namespace

void gemm(const float* A, int lda, const float* B, int ldb, float* C, int ldc, int M, int N, int K,
          bool accumulate) {
  if (M <= 0 || N <= 0) return;
  const int mblocks = (M + MC - 1) / MC;
  const int nblocks = (N + NC - 1) / NC;
#pragma omp parallel
  {
    std::vector<float> Ap(static_cast<size_t>(MC + MR) * KC);
    std::vector<float> Bp(static_cast<size_t>(NC + NR) * KC);
    std::vector<float> acc(static_cast<size_t>(MC) * NC);
    float tile[MR * NR];
#pragma omp for collapse(2) schedule(dynamic)
    for (int mb = 0; mb < mblocks; ++mb) {
      for (int nb = 0; nb < nblocks; ++nb) {
        const int m0 = mb * MC, n0 = nb * NC;
        const int mc = std::min(MC, M - m0), nc = std::min(NC, N - n0);
        const int mp = (mc + MR - 1) / MR, np = (nc + NR - 1) / NR;
        std::fill(acc.begin(), acc.end(), 0.0f);
        for (int k0 = 0; k0 < K; k0 += KC) {
          const int kc = std::min(KC, K - k0);
          // pack A rows into MR-row panels: Ap[p][k][r]
          for (int p = 0; p < mp; ++p)
            for (int k = 0; k < kc; ++k)
              for (int r = 0; r < MR; ++r) {
                const int m = p * MR + r;
                Ap[(static_cast<size_t>(p) * KC + k) * MR + r] =
                    m < mc ? A[static_cast<size_t>(m0 + m) * lda + k0 + k] : 0.0f;
              }
          // pack B rows (output columns) into NR-wide panels: Bp[q][k][c]
          for (int q = 0; q < np; ++q)
            for (int c = 0; c < NR; ++c) {
              const int n = q * NR + c;
              const float* src = B + static_cast<size_t>(n0 + n) * ldb + k0;
              float* dst = &Bp[static_cast<size_t>(q) * KC * NR + c];
              if (n < nc) {
                for (int k = 0; k < kc; ++k) dst[k * NR] = src[k];
              } else {
                for (int k = 0; k < kc; ++k) dst[k * NR] = 0.0f;
              }
            }
          for (int p = 0; p < mp; ++p)
            for (int q = 0; q < np; ++q) {
              micro(&Ap[static_cast<size_t>(p) * KC * MR], &Bp[static_cast<size_t>(q) * KC * NR],
                    kc, tile);
              for (int r = 0; r < MR; ++r) {
                const int m = p * MR + r;
                if (m >= mc) break;
                float* a = &acc[static_cast<size_t>(m) * NC + q * NR];
                for (int c = 0; c < NR; ++c) a[c] += tile[r * NR + c];
              }
            }
        }
        for (int m = 0; m < mc; ++m) {
          float* dst = C + static_cast<size_t>(m0 + m) * ldc + n0;
          const float* a = &acc[static_cast<size_t>(m) * NC];
          if (accumulate)
            for (int n = 0; n < nc; ++n) dst[n] += a[n];
          else
            for (int n = 0; n < nc; ++n) dst[n] = a[n];
        }
      }
    }
  }
}

// ------------------------------------------------------------ 16-bit carriers

uint16_t f32_to_f16(float x) {
  // IEEE binary16 round-to-nearest-even with subnormals, inf and NaN, as the
  // `half` crate's f16::from_f32 (half16.rs:40-43 calls it).
  uint32_t u;
  std::memcpy(&u, &x, 4);
  const uint32_t sign = (u >> 16) & 0x8000u;
  const uint32_t a = u & 0x7FFFFFFFu;
  if (a >= 0x7F800000u) {  // inf / NaN
    if (a == 0x7F800000u) return static_cast<uint16_t>(sign | 0x7C00u);
    return static_cast<uint16_t>(sign | 0x7E00u | ((a >> 13) & 0x3FFu));
  }
  if (a >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);  // rounds to inf
  if (a < 0x38800000u) {                                             // f16 subnormal / zero
    if (a < 0x33000000u) return static_cast<uint16_t>(sign);         // < 2^-25: to zero
    const uint32_t e = a >> 23;                                      // 102..112
    const uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
    const uint32_t shift = 126 - e;  // bits to drop so that the unit is 2^-24
    uint32_t r = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (r & 1u))) ++r;
    return static_cast<uint16_t>(sign | r);
  }
  // normal: rebias exponent 127 -> 15, keep 10 mantissa bits, RNE on 13
  uint32_t r = ((a >> 13) - ((127u - 15u) << 10));
  const uint32_t rem = a & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;  // may carry into inf: correct
  return static_cast<uint16_t>(sign | r);
}

float f16_to_f32(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu;
  uint32_t u;
  if (e == 0) {
    if (m == 0) {
      u = sign;
    } else {  // subnormal: normalise
      int ee = -1;
      do {
        ++ee;
        m <<= 1;
      } while ((m & 0x400u) == 0);
      u = sign | ((127u - 15u - ee) << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    u = sign | 0x7F800000u | (m << 13);
  } else {
    u = sign | ((e + 127u - 15u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

uint16_t f32_to_bf16(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);  // NaN
  return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

}  // namespace orc

extern "C" {
uint16_t or_f32_to_f16(float x) { return orc::f32_to_f16(x); }
float or_f16_to_f32(uint16_t h) { return orc::f16_to_f32(h); }
uint16_t or_f32_to_bf16(float x) { return orc::f32_to_bf16(x); }
float or_bf16_to_f32(uint16_t h) { return orc::bf16_to_f32(h); }
void or_gemm(const float* A, int lda, const float* B, int ldb, float* C, int ldc, int M, int N,
             int K, int accumulate) {
  orc::gemm(A, lda, B, ldb, C, ldc, M, N, K, accumulate != 0);
}
void or_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}
}
