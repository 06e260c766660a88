/*
 * qa_b200 — C ABI of the B200 (sm_100a) backend for the Qwen3-ForcedAligner
 * single-forward alignment path.
 *
 * This is the drop-in boundary.  In the reference crate the towers sit behind
 * a private enum (src/align_inference.rs:82-181, `enum Backend { Gpu, Cpu }`)
 * with four methods; a `Backend::Cuda { ctx }` arm binds the functions below
 * one for one, through an `extern "C"` block whose Rust types follow the C
 * types here (int -> c_int, int64_t -> i64, pointers -> *const / *mut, the
 * structs #[repr(C)] with the same field order):
 *
 *   Backend::half()                 -> qa_half
 *   Backend::audio_embeds(mel, v)   -> qa_audio_embeds
 *   Backend::ensure_capacity(need)  -> qa_ensure_capacity
 *   Backend::text_hidden(bytes, s)  -> qa_text_hidden
 *
 * plus the stages the reference runs on the host that this backend moves onto
 * the GPU: the log-mel (src/mel.rs:15-242 -> qa_mel) and the final norm +
 * timestamp head + argmax (src/align_inference.rs:737-805 -> qa_head), and a
 * batched, device-resident whole-path call (qa_align_batch) that runs
 * samples -> raw_ms for many clips with one upload and one readback.
 *
 * Conventions (mirroring the reference's anyhow::Result contract):
 *  - every function returns an int status, QA_OK (0) on success; nothing
 *    aborts; qa_last_error(ctx) gives the message of the last failure;
 *  - the context owns all device memory; the caller owns every host buffer
 *    (inputs are borrowed for the call, outputs are caller-allocated);
 *  - one context is single-threaded (the reference's `align` takes &mut self);
 *    distinct contexts on distinct devices may run concurrently;
 *  - 16-bit element buffers are little-endian f16 or bf16 per the context's
 *    storage format (qa_half).
 */
#ifndef QA_B200_H
#define QA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define QA_OK 0
#define QA_ERR_SHAPE 1   /* a size or shape does not match (reference: ensure!/bail!) */
#define QA_ERR_CAP 2     /* seq > max_seq (8192) or audio tokens > 16384 */
#define QA_ERR_CUDA 3    /* a CUDA runtime call failed */
#define QA_ERR_OOM 4     /* device allocation failed */
#define QA_ERR_TIMEOUT 5 /* a bounded device wait ran out */
#define QA_ERR_STATE 6   /* call out of order, or a conflicting storage format */
#define QA_ERR_WEIGHTS 7 /* a weight is missing or mis-shaped */
#define QA_ERR_ARG 8     /* a NULL or otherwise invalid argument */

/* 16-bit storage formats (src/shaders.rs:108-160, `Half`). */
#define QA_HALF_F16 0
#define QA_HALF_BF16 1

/* Tensor element types for qa_load (safetensors dtypes). */
#define QA_DTYPE_F32 0
#define QA_DTYPE_F16 1
#define QA_DTYPE_BF16 2

typedef struct qa_ctx qa_ctx;

/* One host tensor, borrowed for the duration of qa_load (e.g. a pointer into
 * an mmap'd safetensors shard).  Names are the checkpoint's own, in either
 * layout: the `-hf` names (model.audio_tower.*, model.language_model.*,
 * model.multi_modal_projector.linear_{1,2}.*, score.weight) are remapped the
 * way src/weights.rs:231-265 does. */
typedef struct {
  const char* name;
  int dtype;
  int ndim;
  int64_t shape[4];
  const void* data;
} qa_tensor;

/* Model geometry, as parsed from config.json (src/config.rs:81-137,186-236). */
typedef struct {
  /* audio tower */
  int d_model, encoder_layers, encoder_heads, encoder_ffn_dim, num_mel_bins;
  int downsample_hidden, max_source_positions, n_window, n_window_infer, output_dim;
  /* text decoder */
  int vocab_size, hidden_size, intermediate_size, num_layers, num_heads, num_kv_heads, head_dim;
  double rms_norm_eps, rope_theta;
  /* forced-aligner head */
  int num_labels, timestamp_token_id, audio_token_id;
  double timestamp_segment_time_ms;
  int max_seq; /* 8192 (src/align_inference.rs:70) */
} qa_cfg;

/* Per-phase device times of the last batched call, in ms (CUDA events on the
 * context's stream; the phases of src/align_inference.rs:230-251). */
typedef struct {
  double h2d_ms, mel_ms, enc_ms, gather_ms, prefill_ms, head_ms, d2h_ms, total_ms;
  int64_t gpu_launches; /* kernels this library launched in the call */
  int64_t h2d_bytes;    /* host->device bytes the call copied */
  int64_t d2h_bytes;    /* device->host bytes the call copied */
  double local_ms;      /* the Local Head's refinement (Timings::local_ms); 0 when it did not run */
} qa_timings;

/* Live per-kernel statistics (qa_set_profile): CUDA-event time of every launch
 * of a kernel class on the launching stream, and the class's algorithmic work. */
typedef struct {
  char name[32];
  int64_t launches;
  double total_ms;
  double flops; /* algorithmic FLOPs of all launches (0 for memory-bound kernels) */
  double bytes; /* algorithmic HBM bytes of all launches */
} qa_kernel_stat;

/* ---------------------------------------------------------------- lifetime */

/* Open a context on CUDA device `device` storing 16-bit values in `half`
 * (Aligner::load_backend_with_dtype, src/align_inference.rs:287-292). */
int qa_open(int device, int half, qa_ctx** out);
/* Upload the weights (src/align_inference.rs:294-453). */
int qa_load(qa_ctx* ctx, const qa_tensor* tensors, int n, const qa_cfg* cfg);
int qa_close(qa_ctx* ctx);
const char* qa_last_error(const qa_ctx* ctx);
/* Bound on every host-side wait for the device (default 60000 ms). */
int qa_set_timeout_ms(qa_ctx* ctx, int ms);
/* Backend::half (src/align_inference.rs:103-108). */
int qa_half(const qa_ctx* ctx);
int qa_get_timings(const qa_ctx* ctx, qa_timings* out);
/* Launch on the caller's CUDA stream (a cudaStream_t; NULL restores the
 * context's own non-blocking stream, so the legacy default stream cannot be
 * selected: pass a created stream to order the library's work with other work
 * on it).  No reference counterpart: wgpu owns its queue. */
int qa_set_stream(qa_ctx* ctx, void* stream);
/* Record CUDA events around every kernel launch (on = 1) and accumulate them
 * per kernel class; qa_get_profile returns up to `max` classes.  No reference
 * counterpart (the reference profiles with host timers, src/load_trace.rs). */
int qa_set_profile(qa_ctx* ctx, int on);
int qa_get_profile(qa_ctx* ctx, qa_kernel_stat* stats, int max, int* n);

/* ---------------------------------------------------------------- stages */

/* Log-mel of 16 kHz mono samples (mel::mel_features, src/mel.rs:15-242):
 * out is [num_mel_bins, n_frames] row-major f32 with n_frames = n / 160.
 * *n_frames receives the frame count; out_len is out's capacity in floats. */
int qa_mel(qa_ctx* ctx, const float* samples, int64_t n, float* out, int64_t out_len,
           int* n_frames);

/* Backend::audio_embeds (src/align_inference.rs:118-133): mel [n_mels,
 * valid_frames] row-major f32 -> [n_audio_tokens, output_dim] 16-bit.
 * out_len is out's capacity in elements; the produced count must equal
 * n_audio_tokens * output_dim. */
int qa_audio_embeds(qa_ctx* ctx, const float* mel, int n_mels, int valid_frames, uint16_t* out,
                    int64_t out_len);

/* Backend::ensure_capacity (src/align_inference.rs:137-142): make the K/V
 * cache hold `need` positions (grow-only, capped at max_seq). */
int qa_ensure_capacity(qa_ctx* ctx, int need, int* cap);

/* Backend::text_hidden (src/align_inference.rs:150-173): [seq, hidden] 16-bit
 * input embeddings -> [seq, hidden] f32 hidden states after the last layer. */
int qa_text_hidden(qa_ctx* ctx, const uint16_t* emb, int seq, float* out);

/* Final RMSNorm + timestamp head + argmax on the given rows of `hidden`
 * (src/align_inference.rs:737-805).  hidden [seq, hidden_size] f32; rows the
 * timestamp positions.  raw_ms [n_rows] receives (argmax * segment_ms) as
 * i64.  logits [n_rows, num_labels] and normed [n_rows, hidden_size] (the
 * unfolded norm the Local Head reads) are optional (NULL to skip). */
int qa_head(qa_ctx* ctx, const float* hidden, int seq, const int* rows, int n_rows,
            int64_t* raw_ms, float* logits, float* normed);

/* Timestamp repair (src/postprocess.rs:33-113, `fix_timestamps`): the
 * longest non-decreasing subsequence with the reference's earliest-index ties
 * (its O(n^2) DP, :39-48, found here in O(n log n)); runs of <= 2 outliers
 * snap to the nearer neighbour by index distance, longer runs are
 * interpolated in f64 and truncated toward zero.  out may alias data. */
int qa_fix_timestamps(const int64_t* data, int n, int64_t* out);

/* ---------------------------------------------------------------- audio input */

/* mel::load_audio_wav's decode + downmix (src/mel.rs:347-465) over a WAV
 * file's bytes: 16-bit PCM by the reference's own reader (i16 / 32768.0f,
 * channels summed in order and divided by their count), 8/24/32-bit PCM,
 * 32-bit float and the extensible header as the `hound` crate decodes them.
 * out [out_cap] receives the mono samples at the file's rate; with out NULL
 * the call only reports n_out, sample_rate and channels (a size query).
 * QA_ERR_SHAPE: not RIFF/WAVE, no fmt or data chunk, no samples, or a format
 * neither reader takes; also when out_cap < n_out. */
int qa_decode_wav(const uint8_t* bytes, int64_t n_bytes, float* out, int64_t out_cap,
                  int64_t* n_out, int* sample_rate, int* channels);
/* The length after resampling (librosa fix_length after soxr in
 * src/mel.rs:537-715): ceil(n * sr_out / sr_in); -1 on bad arguments. */
int64_t qa_resampled_length(int64_t n, int sr_in, int sr_out);
/* Mono sample-rate conversion for sources that are not 16 kHz (the soxr HQ
 * call of src/mel.rs:537-715): a linear-phase Kaiser-windowed sinc low-pass
 * with soxr HQ's band edges (pass band to 0.913 of the lower Nyquist
 * frequency, stop band from it, 125 dB), output sample k at input time
 * k * sr_in / sr_out.  out_len must be qa_resampled_length(n, sr_in, sr_out)
 * (QA_ERR_SHAPE otherwise).  Same band edges and length as soxr, not the same
 * bits. */
int qa_resample(const float* in, int64_t n, int sr_in, int sr_out, float* out, int64_t out_len);

/* The failure path of a bounded device wait, on purpose (no counterpart in
 * the reference, which reports a lost device after each submit,
 * src/decoder.rs:1670-1672).  Launches one CTA that waits, for at most
 * limit_ms (1..10000), on a pipeline barrier that nothing completes -- the
 * state a lost TMA copy or MMA commit leaves a tensor-core kernel in.  The
 * wait runs out, the kernel sets the timeout bit of the context's status
 * word and returns, and the call returns QA_ERR_TIMEOUT; the context stays
 * usable (nothing is left in flight).  QA_ERR_ARG for a limit out of range. */
int qa_probe_timeout(qa_ctx* ctx, int limit_ms);

/* Timestamp head without any device allocation.  No counterpart in the
 * reference; it is the qa_head computation for callers that cannot allocate
 * device memory: a host that has given the whole GPU to its own memory pool,
 * or a latency-bound caller (a live audio pipeline) that must not stall on
 * cudaMalloc/cudaFree.  hidden [seq, hidden_size] f32, rows [n_rows] int32,
 * raw_ms [n_rows] int64 and the optional logits [n_rows, num_labels] f32 are
 * DEVICE pointers the caller owns.  The scratch is one fixed array inside the
 * library (about 8.4 MB, held by every GPU that loads it until exit), so
 * n_rows <= QA_NOALLOC_HEAD_MAX_ROWS and hidden_size <= 1024, else
 * QA_ERR_CAP.  A row index outside [0, seq) is never read: the call returns
 * QA_ERR_SHAPE (as qa_head does) and leaves the context usable.  The first call
 * on a device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * Work runs on the context's stream and the call waits (bounded) for it.
 * Every call shares the one array, so calls that overlap on the GPU (other
 * threads or contexts on the same device) race; serialise them. */
#define QA_NOALLOC_HEAD_MAX_ROWS 2048
int qa_head_noalloc(qa_ctx* ctx, const float* hidden, int seq, const int* rows, int n_rows,
                    int64_t* raw_ms, float* logits);

/* ---------------------------------------------------------------- Local Head */

/* The optional +-60 ms refinement a checkpoint ships in local_head/
 * (src/local_head.rs).  qa_local_head_load uploads its model.safetensors
 * tensors (all F32, the names and shapes of src/local_head.rs:810-916) and
 * the [91] normalizer mean / std of normalizer.json; the host validates
 * config.json (src/local_head.rs:661-715) before calling it.  Loading enables
 * it (the reference turns it on whenever the package is present,
 * src/align_inference.rs:449).  QA_ERR_WEIGHTS on a missing or mis-shaped
 * tensor, QA_ERR_STATE if one is already loaded. */
int qa_local_head_load(qa_ctx* ctx, const qa_tensor* tensors, int n, const float* mean,
                       const float* std_);
/* Aligner::set_local_head_enabled (src/align_inference.rs:584-593): enabling
 * a context without a loaded Local Head is QA_ERR_STATE. */
int qa_set_local_head_enabled(qa_ctx* ctx, int enabled);
/* Aligner::local_head_enabled: 1 when loaded and enabled. */
int qa_local_head_enabled(const qa_ctx* ctx);

/* LocalHead::refine (src/local_head.rs:179-307) for one clip, on the device:
 * samples [n] 16 kHz mono; logits [2 * n_words][n_labels], the timestamp
 * head's pre-argmax output; hidden [2 * n_words][hidden_size] the unfolded
 * final-norm rows at the timestamp slots.  intervals [n_words][2] receives
 * (start, end) in seconds.  Optional (NULL to skip): fixed_ms [2 * n_words]
 * the repaired coarse centres, offsets_ms [2 * n_words] the head's offsets,
 * features [2 * n_words][41][91] the normalised acoustic windows.
 * QA_ERR_SHAPE when hidden_size is not the head's 1024 context width or the
 * audio is empty; QA_ERR_STATE without a loaded Local Head. */
int qa_local_head_refine(qa_ctx* ctx, const float* samples, int64_t n, int n_words,
                         const float* logits, int n_labels, const float* hidden, int hidden_size,
                         double* intervals, int64_t* fixed_ms, float* offsets_ms,
                         float* features);

/* ---------------------------------------------------------------- batched path */

typedef struct {
  const float* samples; /* 16 kHz mono */
  int64_t n_samples;
  const uint32_t* input_ids; /* InputBuilder::build output (src/align_input.rs:190-262) */
  int seq_len;
} qa_clip;

typedef struct {
  int64_t* raw_ms; /* [n_ts] caller-allocated: one value per <timestamp> token */
  int n_ts;        /* number of <timestamp> tokens in the clip's input_ids */
  float* logits;   /* optional [n_ts, num_labels] */
  float* normed;   /* optional [n_ts, hidden_size] unfolded-norm rows */
  double* intervals; /* optional [n_ts / 2][2] (start, end) seconds per word from
                        the Local Head (LocalHead::refine); needs it enabled */
} qa_result;

/* Align a batch of independent clips in one device-resident pass:
 * samples -> mel -> audio tower -> embedding gather + audio scatter -> causal
 * prefill over a paged K/V cache -> timestamp head -> argmax -> raw_ms.
 * Equivalent, clip by clip, to Aligner::align_raw_rows
 * (src/align_inference.rs:656-834) fed by mel::mel_features. */
int qa_align_batch(qa_ctx* ctx, const qa_clip* clips, int n, qa_result* results);

/* qa_align_batch in three parts, for callers that keep inputs resident or
 * overlap phases (no reference counterpart; the reference is one blocking
 * call per clip):
 *   qa_batch_stage  validates and plans the batch and copies its inputs to
 *                   the device (results give the n_ts per clip and which
 *                   optional outputs to produce);
 *   qa_batch_run    enqueues the device pass over the oldest staged batch on
 *                   the context's stream, followed by the copy of its results
 *                   to pinned host memory, and returns without waiting; with
 *                   no batch staged it runs the last batch again;
 *   qa_batch_fetch  waits (bounded) for the oldest batch that was run and
 *                   copies its results into `results`.
 * Up to two batches may be between stage and fetch, so the next batch can be
 * staged (host copies, uploads queued behind the running kernels) while the
 * previous one runs: stage(1) run(1) stage(2) run(2) fetch(1) stage(3) ... */
int qa_batch_stage(qa_ctx* ctx, const qa_clip* clips, int n, const qa_result* results);
int qa_batch_run(qa_ctx* ctx);
int qa_batch_fetch(qa_ctx* ctx, qa_result* results);

#ifdef __cplusplus
}
#endif

#endif /* QA_B200_H */
