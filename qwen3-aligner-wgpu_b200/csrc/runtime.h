// Host runtime of the B200 alignment backend: the qa_ctx behind the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <map>
#include <memory>
#include <vector>

#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "qa_b200.h"

namespace qa {

// Grow-only device buffer (the reference's capacities are grow-only too,
// src/decoder.rs:657-688).
struct DevBuf {
  void* p = nullptr;
  size_t cap = 0;
  template <typename T = void>
  T* as() const {
    return static_cast<T*>(p);
  }
};

struct PinBuf {
  void* p = nullptr;
  size_t cap = 0;
};

struct EncLayerW {
  float *ln1_g, *ln1_b, *ln2_g, *ln2_b;
  void* qkv_w;  // [3*dm][dm]
  float* qkv_b; // [3*dm]
  void* o_w;
  float* o_b;
  void* fc1_w;
  float* fc1_b;
  void* fc2_w;
  float* fc2_b;
};

struct DecLayerW {
  float *iln, *pln, *qn, *kn;  // rounded to the run's 16-bit format, held as f32
  void* qkv_w;                 // [(nqh + 2 nkv) hd][H]
  void* o_w;                   // [H][nqh hd]
  void* gu_w;                  // [2I][H], gate/up interleaved in blocks of 128 rows
  void* down_w;                // [H][I]
};

struct Weights {
  // mel constants
  void* mel_dft;     // [kMelDftRows][kMelDftK] f16: windowed DFT rows as [hi | hi | lo]
  int *fb_start, *fb_len, *fb_woff;
  float* fb_w;
  // conv stem
  float* c1_w;  // [c1][9]
  float* c1_b;
  void* c2_w;   // [c][9c] permuted
  float* c2_b;
  void* c3_w;
  float* c3_b;
  void* co_w;   // [dm][f3*c] permuted
  float* co_b;
  float* pe;    // [13][dm]
  std::vector<EncLayerW> enc;
  float *lnp_g, *lnp_b;
  void* p1_w;
  float* p1_b;
  void* p2_w;
  float* p2_b;
  // decoder
  void* embed;  // [vocab][H]
  std::vector<DecLayerW> dec;
  float* final_norm;
  void* head_w2;  // [labels][2H] bf16: [score | score]
  void *rope_cos, *rope_sin;  // [max_seq][hd/2] in the storage format
};

// Host-side bookkeeping for one batch of clips (all indices into packed
// device buffers).  Built once per call, uploaded as one int buffer.
struct Plan {
  int n = 0;
  // mel
  std::vector<MelClip> mel;
  std::vector<int> chunk_clip;
  int total_frames = 0, total_chunks = 0, max_frames = 0;
  // audio tower
  std::vector<int> atok0, n_audio;
  int T_a = 0;
  std::vector<int> co_map;     // [total_chunks*13] -> packed audio row or -1
  std::vector<int2> windows;   // encoder windows
  int max_window = 0;          // longest window (tokens)
  // decoder
  std::vector<int> tok0, seq;
  int T_d = 0;
  std::vector<int> p2_map;     // [T_a] -> packed decoder row
  std::vector<int> clip_of, pos_of;
  std::vector<int> block_tab;  // [n][max_pages]
  int max_pages = 0, total_pages = 0;
  std::vector<AttnTile> tiles;
  // head
  std::vector<int> ts_rows;    // packed decoder rows of <timestamp> tokens
  std::vector<int> ts_off;     // per clip offset into ts_rows
};

// Device copies of the plan's arrays inside ctx->idx_dev.
struct PlanDev {
  MelClip* mel;
  int* chunk_clip;
  int* co_map;
  int2* windows;
  int* p2_map;
  int* clip_of;
  int* pos_of;
  int* block_tab;
  AttnTile* tiles;
  int* ts_rows;
  uint32_t* ids;
};


// The Local Head (src/local_head.rs) on the device: weights in the layouts
// the kernels and GEMMs read, and the grow-only workspace of one pass.
struct LocalHeadDev {
  void* conv1_w = nullptr;  // [128][5 * 384] bf16: per tap [w_hi | w_hi | w_lo] (91 -> 128 ch)
  void* conv2_w = nullptr;  // [128][5 * 384]
  float *conv1_b = nullptr, *conv2_b = nullptr;
  void* kv_w = nullptr;     // [256][384]: audio attention k rows, then v rows
  float* kv_b = nullptr;    // [256]
  void* ctx_w = nullptr;    // [128][3 * 1024]
  float* ctx_b = nullptr;
  LhTailW tail{};
  LhFeatConst feat{};
  // one pass
  DevBuf raw, fixed, x1, x2, audio, asplit, kv, ctxa, proj, off, iv;
  // qa_local_head_refine's own inputs and outputs
  DevBuf samples, logits, normed, plan, feat_out;
};

// A batch staged by qa_batch_stage, kept until the next stage call.
// One batch between qa_batch_stage and qa_batch_fetch.  A context holds two,
// so that the next batch can be staged while the previous one runs: each has
// its own pinned staging and result buffers and its own events; the device
// workspaces are shared (every write to them is ordered on the stream after
// the previous batch's kernels).
struct Staged {
  enum State { kFree = 0, kStaged = 1, kRunning = 2 };
  Plan P;
  PlanDev D;
  std::vector<int> n_ts;
  int R = 0;
  bool want_logits = false, want_normed = false;
  bool want_intervals = false;  // the Local Head runs on this batch
  std::vector<LhClip> lh_clips;
  std::vector<int> lh_ep_clip;
  int lh_max_slots = 0;
  PinBuf pin_lh;
  DevBuf lh_plan;
  long long h2d_bytes = 0;
  int state = kFree;
  unsigned long long seq = 0;       // staging order
  int launches = 0;
  PinBuf pin_samples, pin_plan, pin_res;
  DevBuf samples, plan;  // this batch's device inputs (uploaded on the copy stream)
  // 0/1 around the uploads (copy stream), 2..7 phases of the run, 8/9 around
  // the result copy, 10 after the Local Head
  cudaEvent_t ev[11] = {};
};

// One profiled launch: CUDA events around it on the launching stream.
struct ProfRec {
  int cls;
  int ev0, ev1;
  double flops, bytes;
};

// Bounded wait for everything queued on the context's stream (the context's
// timeout), then the device status words: QA_ERR_TIMEOUT for a tensor-core
// pipeline wait that ran out, QA_ERR_SHAPE for an input a kernel rejected.
int wait_stream(qa_ctx* ctx);
int check_status(qa_ctx* ctx);

}  // namespace qa

struct qa_ctx {
  int device = 0;
  int half = QA_HALF_F16;
  bool bf16 = false;
  cudaStream_t stream = nullptr;
  int timeout_ms = 60000;
  std::string err;
  bool loaded = false;
  qa_cfg cfg{};
  int f3 = 0;  // conv3 frequency rows (16)
  qa::Weights w{};
  std::vector<void*> allocations;  // weights, freed at close
  // workspace (grow-only)
  qa::DevBuf samples, mel_scratch, mel_chunked, maxkey, clips_dev, idx_dev;
  qa::DevBuf mel_frames, mel_spec;  // tensor-core mel: A rows, re / im
  qa::DevBuf act1, cols, act2, act3, xenc, h16a, qkv_enc, attn_enc, ffn_enc, proj1;
  qa::DevBuf emb_out, hid, qkv, attn, mlp, kcache, vcache;
  qa::DevBuf ssq_attn, ssq_mlp;  // folded RMSNorm: block sums of squares [T][H/128]
  qa::DevBuf head_a, head_keys, head_raw, head_logits, head_normed, hidden_f32, status, badflag;
  qa::PinBuf pin_in, pin_out, pin_res;  // plan staging, sample staging, results
  int kv_pages = 0;     // pages per layer the cache holds
  int kv_cap_tokens = 0;
  cudaEvent_t ev[12] = {};
  cudaStream_t own_stream = nullptr;  // the context's stream (stream may be the caller's)
  cudaStream_t copy_stream = nullptr;  // batch uploads, overlapping the previous batch's pass
  std::unique_ptr<qa::Staged> slots[2];  // batches between stage and fetch
  unsigned long long batch_seq = 0;
  // live profile (qa_set_profile)
  bool profile = false;
  std::vector<cudaEvent_t> prof_pool;
  int prof_next = 0;
  std::vector<qa::ProfRec> prof_recs;
  std::vector<std::string> prof_names;
  std::vector<qa_kernel_stat> prof_stats;
  qa_timings timings{};
  long long launches = 0;
  // Local Head (qa_local_head_load); runs when lh_on
  std::unique_ptr<qa::LocalHeadDev> lh;
  bool lh_on = false;
};
