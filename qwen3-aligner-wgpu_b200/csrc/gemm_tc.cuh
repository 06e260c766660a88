// Tensor-core GEMM for sm_100a: D = A · Bᵀ with A [M, K] and B [N, K], both
// K-major 16-bit (f16 or bf16), f32 accumulation in TMEM, and a fused
// epilogue.  This is the one GEMM core behind every dense projection of the
// aligner: the decoder's QKV / O / gate-up / down, the audio tower's conv
// stem, QKV, out_proj, fc1/fc2, conv_out and projector, and the timestamp head.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace qa {

// Epilogue modes (what happens to each f32 accumulator element acc[r, c]).
enum EpiMode : int {
  // out16[r, c] = h16(act(acc + bias[c]))
  EPI_STORE16 = 0,
  // out16[r, c] = h16(f32(out16[r, c]) + acc)            (decoder residual)
  EPI_RESID16 = 1,
  // out32[r, c] += acc + bias[c]                          (audio-tower residual)
  EPI_RESID32 = 2,
  // columns [0, BN/2) of a tile are gate, [BN/2, BN) up, for the same outputs:
  // out16[r, j] = h16(silu(h16(g)) * h16(u))             (SwiGLU, out width N/2)
  EPI_SWIGLU16 = 3,
  // out32[map(r), c] = acc + bias[c] + pe[(r % pe_period), c]
  EPI_STORE32 = 4,
  // optional out32[r, c] = acc; keys[r] = max over c of (ordered(acc), ~c)
  EPI_ARGMAX = 5,
  // decoder QKV projection with (d) fused: every 128-column head of the row is
  // rounded to 16 bits, q/k heads get RMSNorm + rotate-half RoPE (Q written to
  // out at the head's columns, K appended to the paged cache), v heads are
  // appended as they are.  Tiles must be 256 wide (two heads).
  EPI_QKV_ROPE = 6,
  // v = act(acc + bias[c]) as an f32-accurate pair of 16-bit values
  // hi = h16(v), lo = h16(v - hi), stored as three N-wide parts of the output
  // row, out16[o, c] = hi, out16[o, N + c] = lo, out16[o, 2N + c] = hi (the A
  // operand of the next three-term product, [hi | lo | hi] . [w_hi | w_hi |
  // w_lo]); optional out2 f32[o, c] = v.  Output row o from the row period
  // fields below (or row_map, or the row itself).
  EPI_SPLIT3 = 7,
};

// Operands of EPI_QKV_ROPE (norm_rope_head, src/cpu_decoder.rs:305-321).
struct RopeKV {
  const int* pos_of = nullptr;     // [M] position of the row within its clip
  const int* clip_of = nullptr;    // [M] clip of the row
  const int* block_tab = nullptr;  // [clips][max_pages] page ids
  int max_pages = 0;
  int page_size = 64;
  void* kc = nullptr;              // this layer's K pages [page][nkv][page_size][128]
  void* vc = nullptr;
  const void* cos_t = nullptr;     // [max_seq][64] in the storage format
  const void* sin_t = nullptr;
  const float* qn = nullptr;       // [128] q_norm gain (rounded to the storage format)
  const float* kn = nullptr;
  float eps = 1e-6f;
  int nq = 16, nkv = 8;
};

enum EpiAct : int { ACT_NONE = 0, ACT_GELU = 1 };

struct EpiParams {
  int mode = EPI_STORE16;
  int act = ACT_NONE;
  void* out = nullptr;          // output base (16-bit or f32 per mode)
  long long ldo = 0;            // output row stride in elements
  const float* bias = nullptr;  // [N] f32, optional
  const int* row_map = nullptr; // optional output row per A row; < 0 skips the row
  const float* pe = nullptr;    // optional [pe_period, N] f32 added by row % pe_period
  int pe_period = 1;
  unsigned long long* keys = nullptr;  // EPI_ARGMAX: [M] packed (value, index) keys
  unsigned* status = nullptr;   // device status word (timeouts)
  RopeKV rk;                    // EPI_QKV_ROPE only
  // EPI_SPLIT3 second output (f32) and its row stride
  float* out2 = nullptr;
  long long ldo2 = 0;
  // Periodic row layout (EPI_SPLIT3 / EPI_STORE32 when row_period > 0): row r
  // with r % row_period >= row_valid is skipped, the others go to output row
  // (r / row_period) * row_out_period + row_out_off + r % row_period.
  int row_period = 0, row_valid = 0, row_out_period = 0, row_out_off = 0;
  // RMSNorm folded into the decoder GEMMs (rms_norm_row, src/cpu_decoder.rs:
  // 289-300).  EPI_RESID16 with ssq_out: for every 128-column block of a row
  // it also writes the sum of squares of the row's new 16-bit values, in
  // column order, ssq_out[r * ssq_n + col / 128] (ssq_n = N / 128, 4 or 8).
  // EPI_QKV_ROPE / EPI_SWIGLU16 with ssq_in: the accumulator of row r is
  // multiplied by 1 / sqrt(sum_j ssq_in[r * ssq_n + j] / rms_d + rms_eps)
  // (sum in j order) before its 16-bit rounding; the norm gain is folded
  // into the B operand's columns.
  float* ssq_out = nullptr;
  const float* ssq_in = nullptr;
  int ssq_n = 0;
  float rms_d = 1.0f, rms_eps = 0.0f;
  // Implicit 1-D convolution along the rows of A (0 = plain GEMM): A is
  // [M, conv_kb * 64] and k-block kb reads the 64 columns (kb % conv_kb) * 64
  // of rows shifted down by kb / conv_kb, so K = taps * conv_kb * 64 covers
  // rows m .. m + taps - 1 of A for output row m (rows past M read as zeros).
  int conv_kb = 0;
};

// Launch D = A·Bᵀ.  A: [M, K] rows lda elements apart; B: [N, K] rows ldb
// apart.  Both pointers 16-byte aligned, lda/ldb multiples of 8.  K tails and
// M/N tails are zero-filled by TMA and masked in the epilogue.
// Returns 0 or a cudaError_t value.
int gemm_tc(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
            bool bf16, const EpiParams& ep, cudaStream_t stream, int force_bn = 0);

// Tile width the launcher picks for N (exposed for SwiGLU weight packing).
int gemm_pick_bn(int N);

// Implicit-GEMM conv2d (3x3, stride 2, pad 1) on the tensor cores: x is NHWC
// [n][h][w][c] 16-bit, wt is [c_out][9c] with k = (kh*3 + kw)*c + ic; output
// rows are positions (oh, ow) per image, or (ow, oh) when time_major, written
// by the epilogue `ep` as an [n*ho*wo, c_out] matrix.  No im2col buffer.
int conv3x3s2_tc(const void* x, int n, int h, int w, int c, const void* wt, int c_out,
                 bool time_major, bool bf16, const EpiParams& ep, cudaStream_t stream);

// SMs of the current device (cached per device), for persistent grids.
int device_sm_count();

}  // namespace qa
