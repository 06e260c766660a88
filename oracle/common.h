// TEST INFRASTRUCTURE (parity oracle) — shared helpers of the CPU restatement.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "oracle.h"

namespace orc {

// f16 round-to-nearest-even, the `half` crate's f16::from_f32 (half 2.7.1),
// which the reference uses at every CPU rounding point (src/cpu_decoder.rs).
uint16_t f32_to_f16(float x);
float f16_to_f32(uint16_t h);
inline float r16(float x) { return f16_to_f32(f32_to_f16(x)); }

// bf16 round-to-nearest-even (src/shaders.rs:74-80, `u + 0x7FFF + lsb`).
uint16_t f32_to_bf16(float x);
inline float bf16_to_f32(uint16_t h) {
  uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// C[M,N] (+)= A[M,K] · B[N,K]^T, f32, OpenMP-parallel blocked GEMM (the
// reference's `gemm` crate call sites: src/cpu_decoder.rs:583-610,
// src/cpu_tensor.rs:85-107, src/audio_encoder.rs:416-426).
void gemm(const float* A, int lda, const float* B, int ldb, float* C, int ldc, int M, int N, int K,
          bool accumulate);

inline float gelu_erf(float x) {
  // src/audio_encoder.rs:195-198: 0.5 x (1 + erf(x / sqrt 2)), erf from libm
  return 0.5f * x * (1.0f + std::erf(x * static_cast<float>(M_SQRT1_2)));
}

}  // namespace orc
