// Launchers of the non-GEMM kernels on the alignment path.  Every launcher
// returns 0 or a cudaError_t value; `bf16` selects the 16-bit storage type
// (f16 when false).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace qa {



// ---------------------------------------------------------------- (a) mel
// Per-clip geometry of a batched mel pass.
struct MelClip {
  long long sample_off;  // first sample of the clip in the sample buffer
  int n_samples;
  int frame_off;         // first frame of the clip in the frame-major scratch
  int n_frames;          // n_samples / 160
  int chunk_off;         // first 100-frame chunk of the clip in the chunked output
};

// Filterbank in compact form: for mel m, weights w[start[m] .. start[m]+len[m]).
struct MelBank {
  const int* start;
  const int* len;
  const int* woff;  // offset of mel m's weights in w
  const float* w;
};

// Pass 1: log10 mel power of every frame -> scratch [total_frames][128] and
// per-clip running max (ordered-uint encoding) in maxkey[clip], on the tensor
// cores: every frame's 400 reflected samples, scaled by
// 2^12 and split into f16 hi + lo, are one row of A = [hi | lo | hi]
// (kMelDftK columns) in frames_ws; dft_hilo is B = [w_hi | w_hi | w_lo] over
// the Hann-windowed DFT rows (cos for bins [0, 201) at rows [0, 201), -sin at
// rows [224, 425)), so one GEMM gives re / im of every bin with the three
// products hi*hi + lo*hi + hi*lo (relative error about 2^-21 per product) into
// spec_ws [total_frames][kMelDftRows] f32.  Power, filterbank, log10 and the
// per-clip max then follow the reference's operation order.
constexpr int kMelDftK = 1200;
constexpr int kMelDftRows = 448;
constexpr int kMelImRow = 224;
int mel_logpower_tc(const float* samples, const MelClip* clips, int n_clips, int max_frames,
                    int total_frames, const void* dft_hilo, MelBank bank, float log10_factor,
                    void* frames_ws, float* spec_ws, float* scratch, unsigned* maxkey,
                    unsigned* status, cudaStream_t s);
// Host construction of dft_hilo (f16 bits, [kMelDftRows][kMelDftK]) from the
// f32 periodic Hann window.
void mel_dft_hilo(const float* window400, uint16_t* out);
// Pass 2a: clamp at max - 8 and (x + 4) / 4 into the chunked encoder input
// [chunk][128][chunk_frames] (tail zero padded).
int mel_finalize_chunked(const float* scratch, const MelClip* clips, const int* chunk_clip,
                         int total_chunks, int chunk_frames, const unsigned* maxkey, float* chunked,
                         cudaStream_t s);
// Pass 2b: the same values in the reference's [128][frames] layout (one clip).
int mel_finalize_rows(const float* scratch, int n_frames, const unsigned* maxkey, float* out,
                      cudaStream_t s);

// ---------------------------------------------------------------- (b) audio tower
// conv1: chunked mel [n][h][w] f32 (c_in = 1) -> NHWC [n][ho][wo][c_out] 16-bit,
// gelu(w·x + b).  w [c_out][9] f32 (k = kh*3 + kw).  On the tensor cores (split
// f16 operands, f32-grade products) when c_out is a multiple of 32 up to 512
// and the output rows are 16-byte aligned; a bounded wait that runs out sets
// kStatusTimeout in *status.
int conv1_direct(const float* mel, int n, int h, int w, const float* wt, const float* bias,
                 int c_out, int ldc, void* out, bool bf16, unsigned* status, cudaStream_t s);

// Channels per pixel of the conv activations that feed the implicit GEMMs:
// c rounded up to 64 (the pad channels hold zeros), so that a 64-channel
// (128-byte) k-block of the TMA im2col boxes never straddles two taps.
inline int conv_channels_padded(int c) { return (c + 63) / 64 * 64; }
// LayerNorm (eps) over rows of f32 x [rows][d] -> 16-bit out.
int layernorm_rows(const float* x, int rows, int d, const float* g, const float* b, float eps,
                   void* out, bool bf16, cudaStream_t s);
// Windowed self-attention over packed audio tokens on the tcgen05 tensor
// cores.  qkv [T][3*dm] 16-bit (q | k | v, head h at columns h*64), out
// [T][dm].  Windows are (start, len) pairs, 1 <= len <= max_window <= 128,
// lying inside [0, T); hd must be 64.  A pipeline wait that runs out sets
// kStatusTimeout in *status.
int window_attention(const void* qkv, long long T, int dm, int nh, int hd, const int2* windows,
                     int n_windows, int max_window, void* out, bool bf16, unsigned* status,
                     cudaStream_t s);

// ---------------------------------------------------------------- decoder
// RMSNorm over rows of 16-bit x [rows][d] -> 16-bit out, f16(x*inv*w).
int rmsnorm_rows(const void* x, int rows, int d, const float* w, float eps, void* out, bool bf16,
                 cudaStream_t s);

// Geometry of the paged K/V cache of one layer: [pages][nkv][page][hd].
struct PagedKV {
  void* k;
  void* v;
  int page_size;  // tokens per page (64)
};

// Per-token position bookkeeping for packed variable-length clips.
struct TokenMap {
  const int* clip_of;   // [T] clip index
  const int* pos_of;    // [T] position within the clip
  const int* block_tab; // [clips][max_pages] page ids
  int max_pages;
};

// (e) causal GQA flash attention on the tcgen05 tensor cores.  Q rows in qkv
// (row stride ldq, head h at column h*hd), K/V from the paged cache, out
// [T][nqh*hd].  Work items are (clip, q0) tiles of 128 query positions (q0 a
// multiple of 128 is not required); K/V pages are read by TMA from the
// layer's pool of `kv_pages` pages; the qkv buffer has `q_rows` rows.
// Persistent: one CTA per SM.  Malformed tiles and out-of-pool page ids set
// status bit 2.
struct AttnTile {
  int clip;
  int q0;       // first query position of the tile within the clip
  int tok0;     // packed token index of position 0 of the clip
  int len;      // clip length
};
int causal_attention_tc(const void* qkv, long long ldq, long long q_rows, int nqh, int nkvh,
                        int hd, const AttnTile* tiles, int n_tiles, const int* block_tab,
                        int max_pages, PagedKV kv, int kv_pages, void* out, bool bf16,
                        unsigned* status, cudaStream_t s);

// Block sums of squares of 16-bit rows [rows][d] (d % 512 == 0):
// out[r * (d/128) + j] = sum of the squares of block j's 128 values, in order
// (the first decoder RMSNorm's statistics, EpiParams::ssq_in).
int row_ssq(const void* x, int rows, int d, float* out, bool bf16, cudaStream_t s);

// Embedding gather: rows of the device table for every non-audio token.
int embed_gather(const uint32_t* ids, int T, const void* table, int vocab, int d, int audio_id,
                 void* out, int* bad, cudaStream_t s);

// Bits of the device flag word `bad` that the gather kernels raise on input
// they reject (the host turns them into QA_ERR_SHAPE).
constexpr int kBadTokenId = 1;  // a token id outside the vocabulary
constexpr int kBadHeadRow = 2;  // a timestamp row outside [0, n_hidden)

// (f) timestamp rows: folded final RMSNorm -> [hi | lo] bf16 split (A operand
// of the head GEMM); optional unfolded norm rows (f32).
// hidden_kind: 0 = f16, 1 = bf16, 2 = f32 rows.  `hidden` holds n_hidden rows;
// a row index outside [0, n_hidden) is not read: its operand row is zeroed
// and kBadHeadRow is or-ed into *bad.
int head_gather_norm(const void* hidden, int hidden_kind, int n_hidden, const int* rows,
                     int n_rows, int d, const float* w, float eps, void* a_hilo, float* unfolded,
                     int* bad, cudaStream_t s);
// keys -> raw_ms = (int64)(argmax * segment_ms)
int argmax_finalize(const unsigned long long* keys, int n, double segment_ms, long long* raw_ms,
                    cudaStream_t s);

// ---------------------------------------------------------------- Local Head
// (src/local_head.rs).  Endpoints are the timestamp slots of the batch, clip
// by clip (2 per word); E counts them.
constexpr int kLhFrames = 41, kLhFrameLen = 400, kLhNfft = 512, kLhBins = 257;
constexpr int kLhMels = 80, kLhBands = 4, kLhFeat = 91;
constexpr int kLhRows = 45;        // rows of an endpoint's conv operand block: 2 + 41 + 2
constexpr int kLhCh = 128;         // channels per part (91 features zero-padded; 128 hidden)
constexpr int kLhXw = 3 * kLhCh;   // a conv operand row: [hi | lo | hi]

struct LhClip {
  long long sample_off;  // first sample of the clip in the batch's sample buffer
  int n_samples;
  int ep_off;            // first endpoint (even: clips hold whole words)
  int n_words;
  int valid;             // classes inside the audio, clamp(floor(ms / 80) + 1, 1, labels)
};
struct LhFeatConst {
  const float* hann;         // [400] symmetric Hann
  const float* bank;         // [80][257] unit-sum mel bank
  const int2* bank_range;    // [80] nonzero bins [x, y) of each bank row
  const float* mean;         // [91] normalizer
  const float* stdv;
  const double2* twiddle;    // [256] exp(-2 pi i k / 512)
};
struct LhTailW {
  const float *cq, *ck, *cv, *co, *aq, *ao;  // [128 in][128 out] (transposed)
  const float *cbq, *cbk, *cbv, *co_b, *abq, *ao_b;
  const float *ctx_b, *role, *endpoint;      // [128], [4][128], [2][128]
  const float *qn_w, *qn_b, *an_w, *an_b, *act_w, *bnd_w, *prior;
  float act_b, bnd_b, derivative_scale;
};
// raw[e] = (first argmax of logits[e][0 .. valid)) * 80, one warp per row.
int lh_masked_argmax(const float* logits, int E, int n_labels, const LhClip* clips,
                     const int* ep_clip, long long* raw, cudaStream_t s);
// fix_timestamps of each clip's raw slots (max_slots bounds 2 * n_words).
int lh_fix(const long long* raw, const LhClip* clips, int n_clips, int max_slots, long long* fixed,
           cudaStream_t s);
// Features of every endpoint -> the first conv's A rows x1 [E * 45][384]
// bf16 (and the padding rows of the second conv's x2); feat_out optional
// [E][41][91] f32.
int lh_features(const float* samples, const LhClip* clips, const int* ep_clip,
                const long long* fixed, int E, const LhFeatConst& kc, uint16_t* x1, uint16_t* x2,
                float* feat_out, cudaStream_t s);
// Context rows [E + E/2][3H] bf16 ([hi | lo | hi]) from the unfolded norm rows.
int lh_ctx_pack(const float* normed, int E, int H, uint16_t* out, cudaStream_t s);
// Offsets (ms) of every endpoint from the projected context rows P
// [E + E/2][128], the audio K/V kv [E * 41][256] and the audio rows
// audio [E * 41][128].
int lh_tail(const float* P, const float* kv, const float* audio, const LhClip* clips,
            const int* ep_clip, int E, const LhTailW& w, float* offsets, cudaStream_t s);
// Refined intervals [E/2][2] in seconds.
int lh_repair(const long long* fixed, const float* offsets, const LhClip* clips, int n_clips,
              double* intervals, cudaStream_t s);

// 16-bit [rows][d] -> f32 widening (text_hidden readback).
int widen16(const void* x, long long n, float* out, bool bf16, cudaStream_t s);

}  // namespace qa
