// qa_head_noalloc: the timestamp head (final RMSNorm + [hidden x labels]
// projection + argmax) for callers that cannot allocate device memory.
//
// Who needs it: a host that has handed the whole GPU to its own memory pool
// at start-up (a serving framework that reserves device memory up front and
// lets no other component call cudaMalloc), and latency-bound callers such as
// a live audio pipeline that must not stall on cudaMalloc / cudaFree, which
// take driver locks and synchronise the device.  They own their input and
// output buffers and pass them in; this call needs nothing else.
//
// Its scratch (the [rows][2*hidden] bf16 hi/lo operand of the head GEMM and
// the per-row argmax keys) lives in one file-scope __device__ array of fixed
// size, which every GPU that loads this library holds until the process exits.
#include <mutex>
#include <string>

#include "runtime.h"
#include "sm100.cuh"

namespace {

constexpr int kNoAllocMaxRows = QA_NOALLOC_HEAD_MAX_ROWS;
constexpr int kNoAllocMaxHidden = 1024;
constexpr size_t kOperandBytes = static_cast<size_t>(kNoAllocMaxRows) * 2 * kNoAllocMaxHidden * 2;
constexpr size_t kKeyBytes = static_cast<size_t>(kNoAllocMaxRows) * 8;

// Host code may not use this name as a device address: it resolves on the
// host to a stand-in.  The device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_head_scratch[kOperandBytes + kKeyBytes];

std::mutex g_setup_mu;
void* g_scratch_addr[256] = {};  // per device ordinal, filled on first use

// Once per device, with that device current: look up the array's device
// address.  Allocates nothing.
int scratch_address(int device, void** out) {
  if (device < 0 || device >= 256) return QA_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_head_scratch);
    if (e != cudaSuccess || !p) return QA_ERR_CUDA;
    g_scratch_addr[device] = p;
  }
  *out = g_scratch_addr[device];
  return QA_OK;
}

}  // namespace

extern "C" int qa_head_noalloc(qa_ctx* ctx, const float* hidden, int seq, const int* rows,
                               int n_rows, int64_t* raw_ms, float* logits) {
  if (!ctx) return QA_ERR_ARG;
  if (!ctx->loaded) {
    ctx->err = "qa_load has not succeeded on this context";
    return QA_ERR_STATE;
  }
  if (!hidden || !rows || !raw_ms || seq <= 0) {
    ctx->err = "qa_head_noalloc: null buffer or empty sequence";
    return QA_ERR_ARG;
  }
  if (n_rows <= 0) return QA_OK;
  const qa_cfg& c = ctx->cfg;
  const int H = c.hidden_size;
  if (n_rows > kNoAllocMaxRows || H > kNoAllocMaxHidden) {
    ctx->err = "qa_head_noalloc: " + std::to_string(n_rows) + " rows of width " +
               std::to_string(H) + " exceed its fixed scratch (" +
               std::to_string(kNoAllocMaxRows) + " rows of width " +
               std::to_string(kNoAllocMaxHidden) + "); use qa_head";
    return QA_ERR_CAP;
  }
  if (cudaSetDevice(ctx->device) != cudaSuccess) return QA_ERR_CUDA;
  void* scratch = nullptr;
  int rc = scratch_address(ctx->device, &scratch);
  if (rc) {
    ctx->err = "qa_head_noalloc: cudaGetSymbolAddress failed";
    return rc;
  }
  void* a_hilo = scratch;
  auto* keys = reinterpret_cast<unsigned long long*>(static_cast<unsigned char*>(scratch) + kOperandBytes);
  cudaStream_t s = ctx->stream;
  // The scratch keeps the previous call's contents: the argmax keys must
  // start at zero.  (The operand rows are fully rewritten below.)
  if (cudaMemsetAsync(keys, 0, static_cast<size_t>(n_rows) * 8, s) != cudaSuccess) {
    ctx->err = "qa_head_noalloc: cudaMemsetAsync failed";
    return QA_ERR_CUDA;
  }
  if (cudaMemsetAsync(ctx->status.p, 0, 4, s) != cudaSuccess ||
      cudaMemsetAsync(ctx->badflag.p, 0, 4, s) != cudaSuccess) {
    ctx->err = "qa_head_noalloc: cudaMemsetAsync failed";
    return QA_ERR_CUDA;
  }
  // Row indices outside [0, seq) are never read: the gather zeroes their
  // operand rows and raises a flag, and the call returns QA_ERR_SHAPE.
  rc = qa::head_gather_norm(hidden, 2, seq, rows, n_rows, H, ctx->w.final_norm,
                            static_cast<float>(c.rms_norm_eps), a_hilo, nullptr,
                            ctx->badflag.as<int>(), s);
  if (!rc) {
    qa::EpiParams ep;
    ep.status = ctx->status.as<unsigned>();
    ep.mode = qa::EPI_ARGMAX;
    ep.out = logits;
    ep.ldo = c.num_labels;
    ep.keys = keys;
    rc = qa::gemm_tc(a_hilo, 2 * H, ctx->w.head_w2, 2 * H, n_rows, c.num_labels, 2 * H, true, ep, s);
  }
  if (!rc)
    rc = qa::argmax_finalize(keys, n_rows, c.timestamp_segment_time_ms,
                             reinterpret_cast<long long*>(raw_ms), s);
  if (rc) {
    ctx->err = std::string("qa_head_noalloc: launch failed: ") +
               cudaGetErrorString(static_cast<cudaError_t>(rc));
    return QA_ERR_CUDA;
  }
  // Bounded wait (the context's timeout), then the device status words: a
  // tensor-core wait that ran out gives QA_ERR_TIMEOUT, a rejected row
  // QA_ERR_SHAPE.
  rc = qa::wait_stream(ctx);
  if (rc) return rc;
  return qa::check_status(ctx);
}
