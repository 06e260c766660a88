/*
 * Kernel-level entry points of the B200 alignment backend.
 *
 * These take DEVICE pointers (already resident in HBM) and a CUDA stream, and
 * run one hot-path kernel each.  They exist so that each kernel can be
 * parity-tested and timed on its own; the reference has no counterpart at this
 * granularity (its kernels are WGSL dispatches inside src/decoder.rs and
 * src/audio_encoder_gpu.rs), so each declaration names the reference stage it
 * computes instead.
 *
 * All functions return 0 on success or a QA_ERR_* code (see qa_b200.h).
 * 16-bit element buffers are f16 when `bf16 == 0`, bf16 otherwise.
 */
#ifndef QA_B200_KERNELS_H
#define QA_B200_KERNELS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Epilogue selectors for qa_k_gemm (values match the library's EpiMode). */
#define QA_EPI_STORE16 0
#define QA_EPI_RESID16 1
#define QA_EPI_RESID32 2
#define QA_EPI_SWIGLU16 3
#define QA_EPI_STORE32 4
#define QA_EPI_ARGMAX 5

/*
 * D = A · Bᵀ on the tcgen05 tensor cores (TMEM accumulator, TMA-fed).
 * A [M, K] (row stride lda), B [N, K] (row stride ldb), 16-bit.
 * `mode`/`act`/`bias`/`out`/`ldo`/`row_map`/`pe`/`keys` select the fused
 * epilogue.  Stands in for every `prefill_gemm*` dispatch of the reference
 * (src/shaders.rs:1817-2077; src/decoder.rs:1321-1657) and for the host
 * projections of src/audio_encoder.rs and src/align_inference.rs:789-790.
 * `status` (device, may be NULL) receives timeout bits.  `force_bn`: 0 = the
 * library's tile choice, -1 = 256-row tiles on CTA pairs, > 0 = one CTA per
 * 128-row tile of that width (128, 224, 240 or 256).
 */
int qa_k_gemm(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
              int bf16, int mode, int act, void* out, long long ldo, const float* bias,
              const int* row_map, const float* pe, int pe_period, unsigned long long* keys,
              unsigned* status, int force_bn, void* stream);

/*
 * The decoder's fused QKV projection: qkv = A · Bᵀ (B = [q|k|v] rows), with
 * the epilogue of cpu_decoder.rs:305-321 per 128-column head: q and k heads
 * are rounded, RMS-normalised (gains qn / kn), rotated by RoPE at the row's
 * position (cos_t / sin_t [max_seq][64] in the storage format); q is written
 * to q_out (row stride ldo), k and v are appended to the paged caches kc / vc
 * [page][nkv][64][128] at (block_tab[clip_of[row]][pos / 64], pos % 64) with
 * pos = pos_of[row].  N = (nq + 2 nkv) * 128.
 */
int qa_k_gemm_qkv_rope(const void* A, long long lda, const void* B, long long ldb, int M, int N,
                       int K, int bf16, void* q_out, long long ldo, const int* pos_of,
                       const int* clip_of, const int* block_tab, int max_pages, void* kc, void* vc,
                       const void* cos_t, const void* sin_t, const float* qn, const float* kn,
                       float eps, int nq, int nkv, unsigned* status, int force_bn, void* stream);

/*
 * Implicit-GEMM conv2d, 3x3 / stride 2 / pad 1, on the tcgen05 tensor cores:
 * x NHWC [n][h][w][c] 16-bit, wt [c_out][9c] (k = (kh*3 + kw)*c + ic),
 * output [n*ho*wo][c_out] through the same epilogues as qa_k_gemm (rows in
 * (oh, ow) order, or (ow, oh) when time_major).  Stands in for the conv2 /
 * conv3 levels of CpuConvStem::conv_block_stages (src/audio_encoder.rs:361-447)
 * and the GPU tower's im2col + GEMM (src/audio_encoder_gpu.rs:1714-1795).
 */
int qa_k_conv3x3s2(const void* x, int n, int h, int w, int c, const void* wt, int c_out,
                   int time_major, int bf16, int mode, int act, void* out, long long ldo,
                   const float* bias, unsigned* status, void* stream);

/*
 * First conv level of the audio tower: conv2d(1 -> c_out, 3x3, stride 2,
 * pad 1) + bias + erf-GELU over mel chunks [n][h][w] (f32), output NHWC
 * [n][ho][wo][c_out] 16-bit (CpuConvStem::conv_block_stages level 1,
 * src/audio_encoder.rs:361-447).  wt [c_out][9] f32, bias [c_out] f32.
 * c_out a multiple of 32 (up to 512) runs on the tensor cores with split f16
 * operands (f32-grade products); other channel counts on CUDA cores.
 */
int qa_k_conv1(const float* mel, int n, int h, int w, const float* wt, const float* bias,
               int c_out, void* out, int bf16, void* stream);

/*
 * Causal GQA attention of the decoder prefill over the paged K/V cache
 * (src/cpu_decoder.rs:327-412; the reference GPU path's
 * prefill_attention_paged dispatch, src/decoder.rs:1463-1520), on the
 * persistent tcgen05/TMEM kernel the pipeline runs.
 * qkv [q_rows][ldq] 16-bit with query head h at column h*128; kpool/vpool
 * [kv_pages][nkvh][64][128]; tiles [n_tiles][4] = (clip, q0, tok0, len), one
 * per 128 query positions of a clip; block_tab [clips][max_pages] page ids;
 * out [q_rows][nqh*128].  GQA groups of two (nqh == 2 * nkvh, the model's
 * geometry); other head counts give QA_ERR_CUDA.
 */
int qa_k_causal_attention(const void* qkv, long long ldq, long long q_rows, int nqh, int nkvh,
                          const int* tiles, int n_tiles, const int* block_tab, int max_pages,
                          const void* kpool, const void* vpool, int kv_pages, void* out, int bf16,
                          unsigned* status, void* stream);

/*
 * The audio tower's windowed self-attention (src/audio_encoder.rs:574-627;
 * the reference GPU tower's window attention, src/audio_encoder_gpu.rs:
 * 1497-1547) on the tcgen05 tensor cores: every query of a window attends to
 * every key of the same window.  qkv [T][3*dm] 16-bit (q | k | v, head h at
 * columns h*64 of each), out [T][dm] with dm = 64 * nh; windows [n_windows][2]
 * = (first token, length), 1 <= length <= max_window <= 128, inside [0, T).
 * A pipeline wait that runs out sets bit 1 of *status (may be NULL).
 */
int qa_k_window_attention(const void* qkv, long long T, int dm, int nh, const int* windows,
                          int n_windows, int max_window, void* out, int bf16, unsigned* status,
                          void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QA_B200_KERNELS_H */
