/*
 * TEST INFRASTRUCTURE — not part of the product.
 *
 * A CPU restatement (C++17 + OpenMP) of the reference crate's `--device cpu`
 * alignment path, used only as the parity checker by tests/, by
 * __graft_entry__.smoke() and as bench.py's cpu_baseline / --impl reference
 * arm.  Nothing in the qwen3-aligner-wgpu_b200 package links or calls it.
 *
 * Each function cites the reference file:line it restates (paths inside the
 * eclipse005/qwen3-aligner-wgpu project).  Parity status: the reference is Rust
 * and cannot be built in this environment (no cargo/rustc), and its model-level
 * golden data is not in its tree, so this restatement is pinned against the
 * reference's own known-answer tests (tests/golden/kat.json, built from the
 * test sources) and cross-checked against an independent PyTorch forward; the
 * model-level numbers themselves are "parity unpinned" against the Rust binary.
 */
#ifndef QA_ORACLE_H
#define QA_ORACLE_H

#include <stdint.h>

#include "../include/qa_b200.h" /* qa_tensor, qa_cfg */

#ifdef __cplusplus
extern "C" {
#endif

typedef struct or_model or_model;

/* --- numeric carriers (src/half16.rs, src/shaders.rs:74-80) --- */
uint16_t or_f32_to_f16(float x);
float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_bf16(float x);
float or_bf16_to_f32(uint16_t h);

/* --- bookkeeping (src/align_input.rs:49-87, src/audio_encoder.rs:693-696) --- */
int64_t or_conv3_length(int64_t len);
int64_t or_audio_token_count(int64_t valid_mel_frames, int64_t n_window);
int64_t or_padded_mel_frames(int64_t valid_mel_frames, int64_t n_window);
int64_t or_valid_mel_frames(int64_t n_samples);

/* --- mel (src/mel.rs:15-242) --- */
/* out [128, n/160] row-major; returns frames via *n_frames; 0 on success. */
int or_mel(const float* samples, int64_t n, float* out, int64_t out_len, int* n_frames);
/* helpers exposed for the reference's own unit tests (src/mel.rs:249-289) */
void or_hann_window(int n, float* out);
int or_reflection_pad(const float* x, int n, int pad, float* out);
void or_mel_filterbank(int num_mels, int n_fft, int sr, float* out /* [num_mels, n_fft/2+1] */);

/* --- rope tables (src/mrope.rs:55-89, src/align_inference.rs:320-328) --- */
void or_rope_tables(int positions, int head_dim, double theta, float* cos_out, float* sin_out);

/* --- model --- */
or_model* or_load(const qa_tensor* tensors, int n, const qa_cfg* cfg, char* err, int err_len);
void or_free(or_model* m);
void or_set_threads(int n);

/* CpuAudioEncoder::forward (src/audio_encoder.rs:754-832): mel [n_mels, valid]
 * -> out [n_audio_tokens, output_dim] f32 (before the f16 narrowing of
 * src/align_inference.rs:124-131). */
int or_audio_embeds(or_model* m, const float* mel, int valid_frames, float* out, int64_t out_len);

/* Host gather + scatter (src/align_inference.rs:685-715) in f16:
 * ids [seq] -> emb [seq, hidden] f16 bits. audio [n_audio, hidden] f16 bits. */
int or_gather(or_model* m, const uint32_t* ids, int seq, const uint16_t* audio, int n_audio,
              uint16_t* emb);

/* CpuTextDecoder::prefill_hidden (src/cpu_decoder.rs:416-547): emb [seq,
 * hidden] f16 -> [seq, hidden] f16 after `n_layers` layers (-1 = all). */
int or_text_hidden(or_model* m, const uint16_t* emb, int seq, int n_layers, uint16_t* out);

/* Final norm + timestamp head + argmax (src/align_inference.rs:737-805).
 * hidden [seq, hidden] f32.  raw_ms [n_rows]; logits [n_rows, labels],
 * normed [n_rows, hidden] (unfolded norm), margin [n_rows] (top1 - top2 logit)
 * are optional. */
int or_head(or_model* m, const float* hidden, int seq, const int* rows, int n_rows,
            int64_t* raw_ms, float* logits, float* normed, float* margin);

/* --- post-processing (src/postprocess.rs:33-113) --- */
void or_fix_timestamps(const int64_t* data, int n, int64_t* out);

/* --- Local Head refinement (src/local_head.rs) --- */
typedef struct or_local_head or_local_head;
/* The package's F32 tensors (src/local_head.rs:810-916) and the [91]
 * normalizer; NULL with a message in err on a missing or mis-shaped tensor. */
or_local_head* or_lh_load(const qa_tensor* tensors, int n, const float* mean, const float* std_,
                          char* err, int err_len);
void or_lh_free(or_local_head* h);
void or_lh_hann(int n, float* out);                         /* src/local_head.rs:917-925 */
void or_lh_mel_bank(float* out /* [80][257] */);            /* src/local_head.rs:927-973 */
void or_lh_band_edges(int bins, int* out /* [5] */);        /* src/local_head.rs:975-982 */
int64_t or_lh_valid_class_count(double duration_ms, int64_t class_count); /* :1066-1069 */
void or_lh_remove_overlaps(double* intervals /* [n][2] */, int n);        /* :1084-1100 */
void or_lh_bound_to_duration(double* intervals, int n, double duration_ms); /* :1102-1130 */
/* [41][91] normalised window centred on center_ms (src/local_head.rs:359-507). */
void or_lh_features_one(const or_local_head* h, const float* samples, int64_t n,
                        int64_t center_ms, float* out);
/* One endpoint's offset in ms (src/local_head.rs:509-611); ctx [4][1024]. */
float or_lh_endpoint_offset(const or_local_head* h, const float* feat, const float* ctx,
                            const float* mask4, int is_end);
/* LocalHead::refine (src/local_head.rs:179-307): out [W][2] seconds; the fixed
 * centres [2W] and offsets [2W] too when non-NULL.  Returns 0, or 1 on bad
 * arguments. */
int or_lh_refine(const or_local_head* h, const float* samples, int64_t n, int W,
                 const float* logits, int n_labels, const float* hidden, int hidden_size,
                 double* out, int64_t* fixed_out, float* offsets_out);

/* --- building blocks, for unit tests --- */
void or_gemm(const float* A, int lda, const float* B, int ldb, float* C, int ldc, int M, int N,
             int K, int accumulate);

#ifdef __cplusplus
}
#endif

#endif
