// Host runtime behind include/qa_b200.h: context lifetime, weight upload
// (with the layout transforms the kernels want), grow-only workspaces, the
// single-clip stage calls that mirror the reference's tower boundary, and the
// batched device-resident alignment path.
#include "runtime.h"
#include "sm100.cuh"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <numeric>
#include <thread>

using namespace qa;

namespace {

// ------------------------------------------------------------ errors

int fail(qa_ctx* ctx, int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (ctx) ctx->err = buf;
  return code;
}

#define CK(expr)                                                                              \
  do {                                                                                        \
    cudaError_t e_ = (expr);                                                                  \
    if (e_ != cudaSuccess)                                                                    \
      return fail(ctx, e_ == cudaErrorMemoryAllocation ? QA_ERR_OOM : QA_ERR_CUDA,            \
                  "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, __LINE__);       \
  } while (0)

// QA_ERR_SHAPE for the bits of the device flag word the gather kernels raise.
int flag_error(qa_ctx* ctx, int bad) {
  if (bad & kBadTokenId) return fail(ctx, QA_ERR_SHAPE, "a token id is outside the vocabulary");
  return fail(ctx, QA_ERR_SHAPE, "a timestamp row is outside the hidden rows");
}

// Launch a kernel (expr returns a cudaError_t value), count it, and when
// profiling is on bracket it with CUDA events tagged with its kernel class and
// algorithmic FLOPs / HBM bytes.
#define KL(tag, flops, bytes, expr)                                                           \
  do {                                                                                        \
    ProfScope ps_(ctx, tag, static_cast<double>(flops), static_cast<double>(bytes));          \
    int e_ = (expr);                                                                          \
    ++ctx->launches;                                                                          \
    if (e_)                                                                                   \
      return fail(ctx, QA_ERR_CUDA, "%s: %s (%s:%d)", #expr,                                  \
                  cudaGetErrorString(static_cast<cudaError_t>(e_)), __FILE__, __LINE__);      \
  } while (0)

int prof_class(qa_ctx* ctx, const char* name) {
  for (size_t i = 0; i < ctx->prof_names.size(); ++i)
    if (ctx->prof_names[i] == name) return static_cast<int>(i);
  ctx->prof_names.push_back(name);
  qa_kernel_stat st{};
  std::snprintf(st.name, sizeof st.name, "%s", name);
  ctx->prof_stats.push_back(st);
  return static_cast<int>(ctx->prof_names.size() - 1);
}

cudaEvent_t prof_event(qa_ctx* ctx, int* idx) {
  if (ctx->prof_next >= static_cast<int>(ctx->prof_pool.size())) {
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    ctx->prof_pool.push_back(e);
  }
  *idx = ctx->prof_next++;
  return ctx->prof_pool[*idx];
}

struct ProfScope {
  qa_ctx* ctx;
  int rec = -1;
  ProfScope(qa_ctx* c, const char* name, double fl, double by) : ctx(c) {
    if (!ctx->profile) return;
    ProfRec r{prof_class(ctx, name), 0, -1, fl, by};
    cudaEventRecord(prof_event(ctx, &r.ev0), ctx->stream);
    ctx->prof_recs.push_back(r);
    rec = static_cast<int>(ctx->prof_recs.size()) - 1;
  }
  ~ProfScope() {
    if (rec < 0) return;
    int i1 = -1;
    cudaEventRecord(prof_event(ctx, &i1), ctx->stream);
    ctx->prof_recs[rec].ev1 = i1;
  }
};

// Fold completed profile records into the per-class statistics (call after
// the stream has drained).
void prof_resolve(qa_ctx* ctx) {
  for (const ProfRec& r : ctx->prof_recs) {
    if (r.ev1 < 0) continue;
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, ctx->prof_pool[r.ev0], ctx->prof_pool[r.ev1]) != cudaSuccess) continue;
    qa_kernel_stat& st = ctx->prof_stats[r.cls];
    st.launches += 1;
    st.total_ms += ms;
    st.flops += r.flops;
    st.bytes += r.bytes;
  }
  ctx->prof_recs.clear();
  ctx->prof_next = 0;
}

double gemm_flops(double M, double N, double K) { return 2.0 * M * N * K; }
double gemm_bytes(double M, double N, double K, double ob) { return (M * K + N * K) * 2.0 + M * N * ob; }

#define TRY(expr)            \
  do {                       \
    int r_ = (expr);         \
    if (r_) return r_;       \
  } while (0)

// Run f(i) for i in [0, n) on all host cores (weight conversion at load).
template <typename F>
void parallel_for(int64_t n, F f) {
  const int64_t nt = std::max<int64_t>(1, std::min<int64_t>(std::thread::hardware_concurrency(), n / 65536));
  if (nt <= 1) {
    for (int64_t i = 0; i < n; ++i) f(i);
    return;
  }
  std::vector<std::thread> th;
  for (int64_t t = 0; t < nt; ++t)
    th.emplace_back([=, &f] {
      const int64_t a = n * t / nt, b = n * (t + 1) / nt;
      for (int64_t i = a; i < b; ++i) f(i);
    });
  for (auto& x : th) x.join();
}

// ------------------------------------------------------------ 16-bit host conversions

uint16_t f32_to_f16(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  const uint32_t sign = (u >> 16) & 0x8000u;
  const uint32_t a = u & 0x7FFFFFFFu;
  if (a >= 0x7F800000u) return static_cast<uint16_t>(sign | (a == 0x7F800000u ? 0x7C00u : 0x7E00u));
  if (a >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);
  if (a < 0x38800000u) {
    if (a < 0x33000000u) return static_cast<uint16_t>(sign);
    const uint32_t e = a >> 23, m = (a & 0x7FFFFFu) | 0x800000u, sh = 126 - e;
    uint32_t r = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u), hf = 1u << (sh - 1);
    if (rem > hf || (rem == hf && (r & 1u))) ++r;
    return static_cast<uint16_t>(sign | r);
  }
  uint32_t r = (a >> 13) - ((127u - 15u) << 10);
  const uint32_t rem = a & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
  return static_cast<uint16_t>(sign | r);
}

float f16_to_f32(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu, u;
  if (e == 0) {
    if (m == 0) {
      u = sign;
    } else {
      int ee = -1;
      do {
        ++ee;
        m <<= 1;
      } while (!(m & 0x400u));
      u = sign | ((127u - 15u - ee) << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    u = sign | 0x7F800000u | (m << 13);
  } else {
    u = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

uint16_t f32_to_bf16(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
  return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

float bf16_to_f32(uint16_t h) {
  const uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

uint16_t to_half_bits(float x, bool bf16) { return bf16 ? f32_to_bf16(x) : f32_to_f16(x); }
float round_half(float x, bool bf16) {
  return bf16 ? bf16_to_f32(f32_to_bf16(x)) : f16_to_f32(f32_to_f16(x));
}

// ------------------------------------------------------------ workspace

int ensure(qa_ctx* ctx, DevBuf& b, size_t bytes) {
  if (bytes <= b.cap) return QA_OK;
  if (b.p) cudaFree(b.p);
  b.p = nullptr;
  b.cap = 0;
  const size_t want = std::max<size_t>(bytes + bytes / 8, 256);
  CK(cudaMalloc(&b.p, want));
  b.cap = want;
  return QA_OK;
}

// ensure() for a buffer whose bytes that kernels never write must read as zero
// (the pad channels of the conv activations): zeroed on the stream whenever it
// is (re)allocated.
int ensure_zeroed(qa_ctx* ctx, DevBuf& b, size_t bytes) {
  if (bytes <= b.cap) return QA_OK;
  TRY(ensure(ctx, b, bytes));
  CK(cudaMemsetAsync(b.p, 0, b.cap, ctx->stream));
  return QA_OK;
}

int ensure_pin(qa_ctx* ctx, PinBuf& b, size_t bytes) {
  if (bytes <= b.cap) return QA_OK;
  if (b.p) cudaFreeHost(b.p);
  b.p = nullptr;
  b.cap = 0;
  const size_t want = std::max<size_t>(bytes + bytes / 8, 4096);
  CK(cudaMallocHost(&b.p, want));
  b.cap = want;
  return QA_OK;
}

// ------------------------------------------------------------ weights

struct HostT {
  int dtype = 0;
  std::vector<int64_t> shape;
  const void* data = nullptr;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

// src/weights.rs:231-265
std::string remap(const std::string& n) {
  auto starts = [&](const char* p) { return n.rfind(p, 0) == 0; };
  if (starts("model.multi_modal_projector.linear_1"))
    return "thinker.audio_tower.proj1" + n.substr(std::strlen("model.multi_modal_projector.linear_1"));
  if (starts("model.multi_modal_projector.linear_2"))
    return "thinker.audio_tower.proj2" + n.substr(std::strlen("model.multi_modal_projector.linear_2"));
  if (starts("model.audio_tower.")) return "thinker.audio_tower." + n.substr(18);
  if (starts("model.language_model.")) return "thinker.model." + n.substr(21);
  if (starts("thinker.lm_head.")) return "score." + n.substr(16);
  return n;
}

struct Loader {
  qa_ctx* ctx;
  std::map<std::string, HostT> t;
  std::string missing;

  const HostT* get(const std::string& name, std::vector<int64_t> shape) {
    auto it = t.find(name);
    if (it == t.end()) {
      if (missing.empty()) missing = "weight not found: " + name;
      return nullptr;
    }
    if (!shape.empty() && it->second.shape != shape) {
      if (missing.empty()) {
        missing = "weight " + name + " has shape [";
        for (auto s : it->second.shape) missing += std::to_string(s) + ",";
        missing += "], expected [";
        for (auto s : shape) missing += std::to_string(s) + ",";
        missing += "]";
      }
      return nullptr;
    }
    return &it->second;
  }
  bool has(const std::string& name) const { return t.count(name) != 0; }
  static float elem(const HostT& v, int64_t i) {
    switch (v.dtype) {
      case QA_DTYPE_F32: return static_cast<const float*>(v.data)[i];
      case QA_DTYPE_F16: return f16_to_f32(static_cast<const uint16_t*>(v.data)[i]);
      default: return bf16_to_f32(static_cast<const uint16_t*>(v.data)[i]);
    }
  }
  std::vector<float> f32(const std::string& name, std::vector<int64_t> shape) {
    const HostT* v = get(name, shape);
    if (!v) return {};
    std::vector<float> o(v->numel());
    parallel_for(v->numel(), [&](int64_t i) { o[i] = elem(*v, i); });
    return o;
  }
  std::vector<float> f32_or_zero(const std::string& name, int64_t n) {
    if (!has(name)) return std::vector<float>(n, 0.0f);
    return f32(name, {n});
  }
};

template <typename T>
T* upload(qa_ctx* ctx, const void* host, size_t bytes, int* rc) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, std::max<size_t>(bytes, 16));
  if (e != cudaSuccess) {
    *rc = fail(ctx, QA_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    return nullptr;
  }
  ctx->allocations.push_back(p);
  e = cudaMemcpy(p, host, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    *rc = fail(ctx, QA_ERR_CUDA, "cudaMemcpy: %s", cudaGetErrorString(e));
    return nullptr;
  }
  return static_cast<T*>(p);
}

float* up_f32(qa_ctx* ctx, const std::vector<float>& v, int* rc) {
  return upload<float>(ctx, v.data(), v.size() * 4, rc);
}

void* up_h16(qa_ctx* ctx, const std::vector<float>& v, int* rc) {
  std::vector<uint16_t> b(v.size());
  const bool bf = ctx->bf16;
  parallel_for(static_cast<int64_t>(v.size()), [&](int64_t i) { b[i] = to_half_bits(v[i], bf); });
  return upload<void>(ctx, b.data(), b.size() * 2, rc);
}

std::vector<float> rounded(std::vector<float> v, bool bf16) {
  for (auto& x : v) x = round_half(x, bf16);
  return v;
}

// src/mel.rs:101-164 filterbank (f64 build, f32 weights) in compact form.
void mel_bank(std::vector<int>& start, std::vector<int>& len, std::vector<int>& woff,
              std::vector<float>& w) {
  const int num_mels = 128, n_fft = 400, n_freqs = 201;
  const double sr = 16000.0, f_sp = 200.0 / 3.0, min_log_hz = 1000.0;
  const double min_log_mel = min_log_hz / f_sp, logstep = std::log(6.4) / 27.0;
  auto hz_to_mel = [&](double f) {
    return f < min_log_hz ? f / f_sp : min_log_mel + std::log(f / min_log_hz) / logstep;
  };
  auto mel_to_hz = [&](double m) {
    return m < min_log_mel ? f_sp * m : min_log_hz * std::exp(logstep * (m - min_log_mel));
  };
  const double mmin = hz_to_mel(0.0), mmax = hz_to_mel(sr / 2.0);
  std::vector<double> ff(num_mels + 2), fd(num_mels + 1);
  for (int i = 0; i < num_mels + 2; ++i)
    ff[i] = mel_to_hz(mmin + (mmax - mmin) * i / static_cast<double>(num_mels + 1));
  for (int i = 0; i < num_mels + 1; ++i) fd[i] = ff[i + 1] - ff[i];
  start.assign(num_mels, 0);
  len.assign(num_mels, 0);
  woff.assign(num_mels, 0);
  w.clear();
  for (int i = 0; i < num_mels; ++i) {
    const double enorm = 2.0 / (ff[i + 2] - ff[i]);
    std::vector<float> row(n_freqs);
    for (int j = 0; j < n_freqs; ++j) {
      const double f = j * sr / n_fft;
      const double down = (f - ff[i]) / fd[i], up = (ff[i + 2] - f) / fd[i + 1];
      row[j] = static_cast<float>(std::max(std::min(down, up), 0.0));
      row[j] *= static_cast<float>(enorm);
    }
    int a = 0, b = n_freqs - 1;
    while (a < n_freqs && row[a] == 0.0f) ++a;
    while (b >= a && row[b] == 0.0f) --b;
    start[i] = a < n_freqs ? a : 0;
    len[i] = a < n_freqs ? b - a + 1 : 0;
    woff[i] = static_cast<int>(w.size());
    for (int j = a; j <= b && a < n_freqs; ++j) w.push_back(row[j]);
  }
}

int64_t feo(int64_t l) {
  auto f = [](int64_t x) { return (x - 1) / 2 + 1; };
  return f(f(f(l)));
}
int64_t conv3_length(int64_t len) {
  int64_t l = len;
  for (int i = 0; i < 3; ++i) l = l > 0 ? (l - 1) / 2 + 1 : 0;
  return l;
}
int64_t audio_token_count(int64_t valid, int64_t n_window) {
  return (valid / (2 * n_window)) * 13 + conv3_length(valid % (2 * n_window));
}

int load_weights(qa_ctx* ctx, const qa_tensor* tensors, int n, const qa_cfg& c) {
  Loader L{ctx, {}, {}};
  bool hf = false;
  for (int i = 0; i < n; ++i) {
    if (!tensors[i].name || !tensors[i].data || tensors[i].ndim < 1 || tensors[i].ndim > 4)
      return fail(ctx, QA_ERR_ARG, "tensor %d: null name/data or bad rank", i);
    std::string nm = tensors[i].name;
    if (nm.rfind("model.audio_tower.", 0) == 0 || nm.rfind("model.language_model.", 0) == 0 ||
        nm.rfind("thinker.lm_head.", 0) == 0)
      hf = true;
  }
  for (int i = 0; i < n; ++i) {
    HostT h;
    h.dtype = tensors[i].dtype;
    if (h.dtype < 0 || h.dtype > 2) return fail(ctx, QA_ERR_ARG, "tensor %s: bad dtype", tensors[i].name);
    h.data = tensors[i].data;
    for (int d = 0; d < tensors[i].ndim; ++d) h.shape.push_back(tensors[i].shape[d]);
    L.t[hf ? remap(tensors[i].name) : std::string(tensors[i].name)] = h;
  }
  const bool bf = ctx->bf16;
  int rc = QA_OK;
  Weights& W = ctx->w;
  const std::string A = "thinker.audio_tower.";
  const int dm = c.d_model, ds = c.downsample_hidden;
  int f3 = c.num_mel_bins;
  for (int i = 0; i < 3; ++i) f3 = (f3 - 1) / 2 + 1;
  ctx->f3 = f3;
  if (dm % 64 || dm != c.encoder_heads * 64 || ds % 8 || c.hidden_size != c.output_dim ||
      c.head_dim != 128 || c.num_heads != 2 * c.num_kv_heads || c.hidden_size % 512 ||
      c.hidden_size > 1024 ||
      c.intermediate_size % 128 || c.num_mel_bins != 128 || c.n_window <= 0)
    return fail(ctx, QA_ERR_SHAPE, "unsupported model geometry");
  {
    // the tower's attention windows: 1..128 tokens (104 for n_window_infer 800)
    const long long ws = feo(2LL * c.n_window) * (c.n_window_infer / (2LL * c.n_window));
    if (ws <= 0 || ws > 128)
      return fail(ctx, QA_ERR_SHAPE, "attention window of %lld tokens (1..128 supported)", ws);
  }

  // ---- mel constants (src/mel.rs:19-27, 101-164)
  {
    std::vector<float> win(400);
    for (int i = 0; i < 400; ++i) {
      const float x = 2.0f * static_cast<float>(M_PI) * static_cast<float>(i) / 400.0f;
      win[i] = 0.5f * (1.0f - std::cos(x));
    }
    std::vector<int> st, ln, wo;
    std::vector<float> fw;
    mel_bank(st, ln, wo, fw);
    std::vector<uint16_t> dft(static_cast<size_t>(kMelDftRows) * kMelDftK);
    mel_dft_hilo(win.data(), dft.data());
    W.mel_dft = upload<uint16_t>(ctx, dft.data(), dft.size() * 2, &rc);
    W.fb_start = upload<int>(ctx, st.data(), st.size() * 4, &rc);
    W.fb_len = upload<int>(ctx, ln.data(), ln.size() * 4, &rc);
    W.fb_woff = upload<int>(ctx, wo.data(), wo.size() * 4, &rc);
    W.fb_w = up_f32(ctx, fw, &rc);
    if (rc) return rc;
  }

  // ---- conv stem: weights in the run's format; conv2/conv3 permuted to
  // k = (kh*3 + kw)*c_in + ic; conv_out columns to f*c + ch (NHWC order)
  {
    auto w1 = L.f32(A + "conv2d1.weight", {ds, 1, 3, 3});
    auto w2 = L.f32(A + "conv2d2.weight", {ds, ds, 3, 3});
    auto w3 = L.f32(A + "conv2d3.weight", {ds, ds, 3, 3});
    auto co = L.f32(A + "conv_out.weight", {dm, (int64_t)ds * f3});
    auto b1 = L.f32(A + "conv2d1.bias", {ds});
    auto b2 = L.f32(A + "conv2d2.bias", {ds});
    auto b3 = L.f32(A + "conv2d3.bias", {ds});
    if (!L.missing.empty()) return fail(ctx, QA_ERR_WEIGHTS, "%s", L.missing.c_str());
    // conv2/conv3 weights as [oc][(kh*3 + kw)*cp + ic]: the activations carry
    // cp = ds rounded up to 64 channels per pixel (the pad channels are zero),
    // so a 64-channel k-block never straddles two taps
    const int cp = conv_channels_padded(ds);
    auto perm = [&](const std::vector<float>& w) {
      std::vector<float> o(static_cast<size_t>(ds) * 9 * cp, 0.0f);
      for (int oc = 0; oc < ds; ++oc)
        for (int ic = 0; ic < ds; ++ic)
          for (int k = 0; k < 9; ++k)
            o[(static_cast<size_t>(oc) * 9 + k) * cp + ic] = w[(static_cast<size_t>(oc) * ds + ic) * 9 + k];
      return o;
    };
    std::vector<float> cop(co.size());
    for (int o = 0; o < dm; ++o)
      for (int ch = 0; ch < ds; ++ch)
        for (int f = 0; f < f3; ++f)
          cop[static_cast<size_t>(o) * ds * f3 + f * ds + ch] = co[static_cast<size_t>(o) * ds * f3 + ch * f3 + f];
    W.c1_w = up_f32(ctx, rounded(w1, bf), &rc);
    W.c1_b = up_f32(ctx, b1, &rc);
    W.c2_w = up_h16(ctx, perm(w2), &rc);
    W.c2_b = up_f32(ctx, b2, &rc);
    W.c3_w = up_h16(ctx, perm(w3), &rc);
    W.c3_b = up_f32(ctx, b3, &rc);
    W.co_w = up_h16(ctx, cop, &rc);
    W.co_b = up_f32(ctx, L.f32_or_zero(A + "conv_out.bias", dm), &rc);
    // sinusoidal PE rows 0..12 (src/audio_encoder.rs:263-275)
    const int tpc = static_cast<int>(feo(2 * c.n_window));
    std::vector<float> pe(static_cast<size_t>(tpc) * dm);
    const int half = dm / 2;
    const double lt = std::log(10000.0) / (half - 1.0);
    for (int p = 0; p < tpc; ++p)
      for (int i = 0; i < half; ++i) {
        const double a = p * std::exp(-i * lt);
        pe[static_cast<size_t>(p) * dm + i] = static_cast<float>(std::sin(a));
        pe[static_cast<size_t>(p) * dm + half + i] = static_cast<float>(std::cos(a));
      }
    W.pe = up_f32(ctx, pe, &rc);
    if (rc) return rc;
  }
  // ---- encoder layers
  W.enc.clear();
  for (int l = 0; l < c.encoder_layers; ++l) {
    const std::string p = A + "layers." + std::to_string(l) + ".";
    EncLayerW e{};
    auto q = L.f32(p + "self_attn.q_proj.weight", {dm, dm});
    auto k = L.f32(p + "self_attn.k_proj.weight", {dm, dm});
    auto v = L.f32(p + "self_attn.v_proj.weight", {dm, dm});
    std::vector<float> qkv(q);
    qkv.insert(qkv.end(), k.begin(), k.end());
    qkv.insert(qkv.end(), v.begin(), v.end());
    auto qb = L.f32_or_zero(p + "self_attn.q_proj.bias", dm);
    auto kb = L.f32_or_zero(p + "self_attn.k_proj.bias", dm);
    auto vb = L.f32_or_zero(p + "self_attn.v_proj.bias", dm);
    std::vector<float> qkvb(qb);
    qkvb.insert(qkvb.end(), kb.begin(), kb.end());
    qkvb.insert(qkvb.end(), vb.begin(), vb.end());
    auto ow = L.f32(p + "self_attn.out_proj.weight", {dm, dm});
    auto f1 = L.f32(p + "fc1.weight", {c.encoder_ffn_dim, dm});
    auto f2 = L.f32(p + "fc2.weight", {dm, c.encoder_ffn_dim});
    auto g1 = L.f32(p + "self_attn_layer_norm.weight", {dm});
    auto be1 = L.f32(p + "self_attn_layer_norm.bias", {dm});
    auto g2 = L.f32(p + "final_layer_norm.weight", {dm});
    auto be2 = L.f32(p + "final_layer_norm.bias", {dm});
    if (!L.missing.empty()) return fail(ctx, QA_ERR_WEIGHTS, "%s", L.missing.c_str());
    e.qkv_w = up_h16(ctx, qkv, &rc);
    e.qkv_b = up_f32(ctx, qkvb, &rc);
    e.o_w = up_h16(ctx, ow, &rc);
    e.o_b = up_f32(ctx, L.f32_or_zero(p + "self_attn.out_proj.bias", dm), &rc);
    e.fc1_w = up_h16(ctx, f1, &rc);
    e.fc1_b = up_f32(ctx, L.f32_or_zero(p + "fc1.bias", c.encoder_ffn_dim), &rc);
    e.fc2_w = up_h16(ctx, f2, &rc);
    e.fc2_b = up_f32(ctx, L.f32_or_zero(p + "fc2.bias", dm), &rc);
    e.ln1_g = up_f32(ctx, g1, &rc);
    e.ln1_b = up_f32(ctx, be1, &rc);
    e.ln2_g = up_f32(ctx, g2, &rc);
    e.ln2_b = up_f32(ctx, be2, &rc);
    if (rc) return rc;
    W.enc.push_back(e);
  }
  {
    auto g = L.f32(A + "ln_post.weight", {dm});
    auto b = L.f32(A + "ln_post.bias", {dm});
    auto p1 = L.f32(A + "proj1.weight", {dm, dm});
    auto p2 = L.f32(A + "proj2.weight", {c.output_dim, dm});
    if (!L.missing.empty()) return fail(ctx, QA_ERR_WEIGHTS, "%s", L.missing.c_str());
    W.lnp_g = up_f32(ctx, g, &rc);
    W.lnp_b = up_f32(ctx, b, &rc);
    W.p1_w = up_h16(ctx, p1, &rc);
    W.p1_b = up_f32(ctx, L.f32_or_zero(A + "proj1.bias", dm), &rc);
    W.p2_w = up_h16(ctx, p2, &rc);
    W.p2_b = up_f32(ctx, L.f32_or_zero(A + "proj2.bias", c.output_dim), &rc);
    if (rc) return rc;
  }
  // ---- decoder
  const std::string T = "thinker.model.";
  const int H = c.hidden_size, hd = c.head_dim, nq = c.num_heads, nkv = c.num_kv_heads;
  const int I = c.intermediate_size;
  {
    const HostT* e = L.get(T + "embed_tokens.weight", {c.vocab_size, H});
    if (!e) return fail(ctx, QA_ERR_WEIGHTS, "%s", L.missing.c_str());
    std::vector<uint16_t> b(e->numel());
    parallel_for(e->numel(), [&](int64_t i) { b[i] = to_half_bits(Loader::elem(*e, i), bf); });
    W.embed = upload<void>(ctx, b.data(), b.size() * 2, &rc);
    if (rc) return rc;
  }
  W.dec.clear();
  for (int l = 0; l < c.num_layers; ++l) {
    const std::string p = T + "layers." + std::to_string(l) + ".";
    DecLayerW d{};
    auto q = L.f32(p + "self_attn.q_proj.weight", {(int64_t)nq * hd, H});
    auto k = L.f32(p + "self_attn.k_proj.weight", {(int64_t)nkv * hd, H});
    auto v = L.f32(p + "self_attn.v_proj.weight", {(int64_t)nkv * hd, H});
    auto o = L.f32(p + "self_attn.o_proj.weight", {H, (int64_t)nq * hd});
    auto gt = L.f32(p + "mlp.gate_proj.weight", {I, H});
    auto up = L.f32(p + "mlp.up_proj.weight", {I, H});
    auto dn = L.f32(p + "mlp.down_proj.weight", {H, I});
    auto iln = L.f32(p + "input_layernorm.weight", {H});
    auto pln = L.f32(p + "post_attention_layernorm.weight", {H});
    auto qn = L.f32(p + "self_attn.q_norm.weight", {hd});
    auto kn = L.f32(p + "self_attn.k_norm.weight", {hd});
    if (!L.missing.empty()) return fail(ctx, QA_ERR_WEIGHTS, "%s", L.missing.c_str());
    std::vector<float> qkv(q);
    qkv.insert(qkv.end(), k.begin(), k.end());
    qkv.insert(qkv.end(), v.begin(), v.end());
    // RMSNorm folded into the projections that follow it: column k of the
    // QKV (gate/up) weights carries input_layernorm (post_attention_layernorm)
    // gain k, rounded to the run's format as the reference rounds the gains;
    // the GEMM epilogue applies the row's 1 / rms.
    {
      const std::vector<float> gi = rounded(iln, bf), gp = rounded(pln, bf);
      for (size_t r = 0; r < qkv.size() / H; ++r)
        for (int j = 0; j < H; ++j) qkv[r * H + j] *= gi[j];
      for (size_t r = 0; r < gt.size() / H; ++r)
        for (int j = 0; j < H; ++j) {
          gt[r * H + j] *= gp[j];
          up[r * H + j] *= gp[j];
        }
    }
    // gate/up interleaved in blocks of 128 rows: a 256-wide GEMM tile holds
    // the gate and up rows of the same 128 outputs (SwiGLU epilogue).
    std::vector<float> gu(static_cast<size_t>(2) * I * H);
    for (int b = 0; b < I / 128; ++b)
      for (int r = 0; r < 128; ++r) {
        std::memcpy(&gu[(static_cast<size_t>(b) * 256 + r) * H], &gt[(static_cast<size_t>(b) * 128 + r) * H], H * 4);
        std::memcpy(&gu[(static_cast<size_t>(b) * 256 + 128 + r) * H], &up[(static_cast<size_t>(b) * 128 + r) * H], H * 4);
      }
    d.qkv_w = up_h16(ctx, qkv, &rc);
    d.o_w = up_h16(ctx, o, &rc);
    d.gu_w = up_h16(ctx, gu, &rc);
    d.down_w = up_h16(ctx, dn, &rc);
    d.iln = up_f32(ctx, rounded(iln, bf), &rc);
    d.pln = up_f32(ctx, rounded(pln, bf), &rc);
    d.qn = up_f32(ctx, rounded(qn, bf), &rc);
    d.kn = up_f32(ctx, rounded(kn, bf), &rc);
    if (rc) return rc;
    W.dec.push_back(d);
  }
  {
    auto fn = L.f32(T + "norm.weight", {H});
    auto sc = L.f32("score.weight", {c.num_labels, H});
    if (!L.missing.empty()) return fail(ctx, QA_ERR_WEIGHTS, "%s", L.missing.c_str());
    W.final_norm = up_f32(ctx, fn, &rc);
    // [score | score] in bf16: the head multiplies a hi/lo bf16 split of the
    // f32 normed rows by the checkpoint's exact bf16 weights.
    std::vector<uint16_t> w2(static_cast<size_t>(c.num_labels) * 2 * H);
    for (int r = 0; r < c.num_labels; ++r)
      for (int j = 0; j < H; ++j) {
        const uint16_t b = f32_to_bf16(sc[static_cast<size_t>(r) * H + j]);
        w2[static_cast<size_t>(r) * 2 * H + j] = b;
        w2[static_cast<size_t>(r) * 2 * H + H + j] = b;
      }
    W.head_w2 = upload<void>(ctx, w2.data(), w2.size() * 2, &rc);
    // RoPE (src/align_inference.rs:320-328, 371-373): theta 1e6, plain, f32
    // then rounded to the run's format; halves duplicate, keep one.
    const int half = hd / 2;
    std::vector<float> cs(static_cast<size_t>(c.max_seq) * half), sn(cs.size());
    for (int t = 0; t < c.max_seq; ++t)
      for (int j = 0; j < half; ++j) {
        const double inv = 1.0 / std::pow(1000000.0, 2.0 * j / hd);
        const double a = static_cast<double>(t) * inv;
        cs[static_cast<size_t>(t) * half + j] = round_half(static_cast<float>(std::cos(a)), bf);
        sn[static_cast<size_t>(t) * half + j] = round_half(static_cast<float>(std::sin(a)), bf);
      }
    W.rope_cos = up_h16(ctx, cs, &rc);  // exact: the values are already rounded to the format
    W.rope_sin = up_h16(ctx, sn, &rc);
    if (rc) return rc;
  }
  return QA_OK;
}

// ------------------------------------------------------------ batched-path plan

// Attention work items: 128 query positions of one clip (each K/V head of the
// item is one CTA-sized unit of the persistent tcgen05 attention kernel).
// Longest clips first for load balance; the blocks of one clip stay adjacent
// (last block first), so the CTAs running at the same time read the same K/V
// pages and most of those reads hit L2.
void plan_tiles(Plan& P) {
  P.tiles.clear();
  std::vector<int> order(P.n);
  for (int c = 0; c < P.n; ++c) order[c] = c;
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return P.seq[a] > P.seq[b]; });
  for (int c : order) {
    const int nb = (P.seq[c] + 127) / 128;
    for (int b = nb - 1; b >= 0; --b) P.tiles.push_back({c, b * 128, P.tok0[c], P.seq[c]});
  }
}

void plan_decoder(Plan& P) {
  P.clip_of.assign(P.T_d, 0);
  P.pos_of.assign(P.T_d, 0);
  P.max_pages = 0;
  P.total_pages = 0;
  for (int c = 0; c < P.n; ++c) {
    for (int p = 0; p < P.seq[c]; ++p) {
      P.clip_of[P.tok0[c] + p] = c;
      P.pos_of[P.tok0[c] + p] = p;
    }
    P.max_pages = std::max(P.max_pages, (P.seq[c] + 63) / 64);
  }
  P.block_tab.assign(static_cast<size_t>(P.n) * std::max(P.max_pages, 1), 0);
  for (int c = 0; c < P.n; ++c) {
    const int np = (P.seq[c] + 63) / 64;
    for (int j = 0; j < np; ++j) P.block_tab[static_cast<size_t>(c) * P.max_pages + j] = P.total_pages++;
  }
  plan_tiles(P);
}

template <typename T>
size_t pad16(size_t n) {
  return (n * sizeof(T) + 15) / 16 * 16;
}

int upload_plan(qa_ctx* ctx, const Plan& P, const std::vector<uint32_t>& ids, PlanDev& D,
                PinBuf& pin, DevBuf& dev, cudaStream_t st) {
  const size_t sz_mel = pad16<MelClip>(P.mel.size()), sz_cc = pad16<int>(P.chunk_clip.size()),
               sz_co = pad16<int>(P.co_map.size()), sz_w = pad16<int2>(P.windows.size()),
               sz_p2 = pad16<int>(P.p2_map.size()), sz_clip = pad16<int>(P.clip_of.size()),
               sz_pos = pad16<int>(P.pos_of.size()), sz_bt = pad16<int>(P.block_tab.size()),
               sz_t = pad16<AttnTile>(P.tiles.size()), sz_ts = pad16<int>(P.ts_rows.size()),
               sz_ids = pad16<uint32_t>(ids.size());
  const size_t total = sz_mel + sz_cc + sz_co + sz_w + sz_p2 + sz_clip + sz_pos + sz_bt + sz_t +
                       sz_ts + sz_ids;
  TRY(ensure(ctx, dev, total));
  TRY(ensure_pin(ctx, pin, total));
  uint8_t* h = static_cast<uint8_t*>(pin.p);
  uint8_t* d = dev.as<uint8_t>();
  size_t off = 0;
  auto put = [&](const void* src, size_t bytes, size_t padded) {
    if (bytes) std::memcpy(h + off, src, bytes);
    void* dp = d + off;
    off += padded;
    return dp;
  };
  D.mel = static_cast<MelClip*>(put(P.mel.data(), P.mel.size() * sizeof(MelClip), sz_mel));
  D.chunk_clip = static_cast<int*>(put(P.chunk_clip.data(), P.chunk_clip.size() * 4, sz_cc));
  D.co_map = static_cast<int*>(put(P.co_map.data(), P.co_map.size() * 4, sz_co));
  D.windows = static_cast<int2*>(put(P.windows.data(), P.windows.size() * sizeof(int2), sz_w));
  D.p2_map = static_cast<int*>(put(P.p2_map.data(), P.p2_map.size() * 4, sz_p2));
  D.clip_of = static_cast<int*>(put(P.clip_of.data(), P.clip_of.size() * 4, sz_clip));
  D.pos_of = static_cast<int*>(put(P.pos_of.data(), P.pos_of.size() * 4, sz_pos));
  D.block_tab = static_cast<int*>(put(P.block_tab.data(), P.block_tab.size() * 4, sz_bt));
  D.tiles = static_cast<AttnTile*>(put(P.tiles.data(), P.tiles.size() * sizeof(AttnTile), sz_t));
  D.ts_rows = static_cast<int*>(put(P.ts_rows.data(), P.ts_rows.size() * 4, sz_ts));
  D.ids = static_cast<uint32_t*>(put(ids.data(), ids.size() * 4, sz_ids));
  CK(cudaMemcpyAsync(d, h, total, cudaMemcpyHostToDevice, st));
  return QA_OK;
}

// Audio-tower bookkeeping for a set of clips whose mel is already chunked:
// conv_out row map, packed audio offsets and attention windows.
void plan_audio(Plan& P, const qa_cfg& c, const std::vector<int>& frames) {
  const int cs = 2 * c.n_window;
  const int tpc = static_cast<int>(feo(cs));
  const int ws = tpc * (c.n_window_infer / cs);
  P.atok0.assign(P.n, 0);
  P.n_audio.assign(P.n, 0);
  P.T_a = 0;
  P.co_map.assign(static_cast<size_t>(P.total_chunks) * tpc, -1);
  P.windows.clear();
  P.max_window = 0;
  for (int ci = 0; ci < P.n; ++ci) {
    const int nfull = frames[ci] / cs, tail = frames[ci] % cs;
    const int nch = nfull + (tail > 0);
    const int na = static_cast<int>(audio_token_count(frames[ci], c.n_window));
    P.atok0[ci] = P.T_a;
    P.n_audio[ci] = na;
    for (int i = 0; i < nch; ++i) {
      const int valid = i < nfull ? tpc : static_cast<int>(feo(tail));
      const int ch = P.mel[ci].chunk_off + i;
      for (int t = 0; t < valid; ++t) P.co_map[static_cast<size_t>(ch) * tpc + t] = P.T_a + i * tpc + t;
    }
    const int window = (ws > 0 && ws < na) ? ws : na;
    for (int st = 0; st < na; st += window) {
      P.windows.push_back(make_int2(P.T_a + st, std::min(window, na - st)));
      P.max_window = std::max(P.max_window, std::min(window, na - st));
    }
    P.T_a += na;
  }
}

// ------------------------------------------------------------ stages on device buffers

// Conv stem + transformer + projector over `chunks` mel chunks (already in
// ctx->mel_chunked).  Writes the projected audio rows through `p2_map`
// (row i -> out row map[i]; identity when null) into `out16` [.., out_dim].
int run_encoder(qa_ctx* ctx, const Plan& P, const PlanDev& D, void* out16, const int* p2_map) {
  const qa_cfg& c = ctx->cfg;
  const bool bf = ctx->bf16;
  cudaStream_t s = ctx->stream;
  const Weights& W = ctx->w;
  const int ds = c.downsample_hidden, dm = c.d_model, cs = 2 * c.n_window;
  const int h1 = (c.num_mel_bins - 1) / 2 + 1, w1 = (cs - 1) / 2 + 1;
  const int h2 = (h1 - 1) / 2 + 1, w2 = (w1 - 1) / 2 + 1;
  const int h3 = (h2 - 1) / 2 + 1, w3 = (w2 - 1) / 2 + 1;
  const int tpc = w3;
  const int G = std::max(1, std::min(P.total_chunks, 256));  // chunks per conv group
  const int cp = conv_channels_padded(ds);  // channels per pixel of act1 / act2 (pads zero)
  TRY(ensure_zeroed(ctx, ctx->act1, static_cast<size_t>(G) * h1 * w1 * cp * 2));
  TRY(ensure_zeroed(ctx, ctx->act2, static_cast<size_t>(G) * h2 * w2 * cp * 2));
  // conv3's output is kept for every chunk of the pass (≈ 200 KB a chunk), so
  // that conv_out runs as one GEMM over all of them instead of one per group
  TRY(ensure(ctx, ctx->act3, static_cast<size_t>(P.total_chunks) * h3 * w3 * ds * 2));
  TRY(ensure(ctx, ctx->xenc, static_cast<size_t>(std::max(P.T_a, 1)) * dm * 4));
  EpiParams ep;
  ep.status = ctx->status.as<unsigned>();
  for (int g0 = 0; g0 < P.total_chunks; g0 += G) {
    const int g = std::min(G, P.total_chunks - g0);
    const float* mel = ctx->mel_chunked.as<float>() + static_cast<size_t>(g0) * c.num_mel_bins * cs;
    KL("conv1", 18.0 * g * h1 * w1 * ds, 4.0 * g * c.num_mel_bins * cs + 2.0 * g * h1 * w1 * ds,
       conv1_direct(mel, g, c.num_mel_bins, cs, W.c1_w, W.c1_b, ds, cp, ctx->act1.p, bf,
                    ctx->status.as<unsigned>(), s));
    // conv2 / conv3: implicit GEMM on the tensor cores, A gathered from NHWC
    ep.mode = EPI_STORE16;
    ep.act = ACT_GELU;
    ep.bias = W.c2_b;
    ep.out = ctx->act2.p;
    ep.ldo = cp;
    ep.row_map = nullptr;
    KL("conv_gemm", gemm_flops(g * h2 * w2, ds, 9 * ds),
       2.0 * g * (h1 * w1 * ds + h2 * w2 * ds) + 2.0 * ds * 9 * ds,
       conv3x3s2_tc(ctx->act1.p, g, h1, w1, cp, W.c2_w, ds, false, bf, ep, s));
    ep.bias = W.c3_b;
    ep.out = static_cast<uint8_t*>(ctx->act3.p) + static_cast<size_t>(g0) * h3 * w3 * ds * 2;
    ep.ldo = ds;
    KL("conv_gemm", gemm_flops(g * h3 * w3, ds, 9 * ds),
       2.0 * g * (h2 * w2 * ds + h3 * w3 * ds) + 2.0 * ds * 9 * ds,
       conv3x3s2_tc(ctx->act2.p, g, h2, w2, cp, W.c3_w, ds, true, bf, ep, s));
  }
  {  // conv_out + bias + PE[t] over every chunk, scattered into the packed token rows
    EpiParams eo;
    eo.status = ep.status;
    eo.mode = EPI_STORE32;
    eo.bias = W.co_b;
    eo.pe = W.pe;
    eo.pe_period = tpc;
    eo.out = ctx->xenc.p;
    eo.ldo = dm;
    eo.row_map = D.co_map;
    const int rows = P.total_chunks * tpc;
    KL("gemm:conv_out", gemm_flops(rows, dm, h3 * ds), gemm_bytes(rows, dm, h3 * ds, 4),
       gemm_tc(ctx->act3.p, (long long)h3 * ds, W.co_w, (long long)h3 * ds, rows, dm, h3 * ds,
               bf, eo, s));
  }
  const int Ta = P.T_a;
  double win_flops = 0;  // 4 * len^2 * dm per window (QKᵀ and PV)
  for (const int2& wv : P.windows) win_flops += 4.0 * wv.y * wv.y * dm;
  TRY(ensure(ctx, ctx->h16a, static_cast<size_t>(Ta) * dm * 2));
  TRY(ensure(ctx, ctx->qkv_enc, static_cast<size_t>(Ta) * 3 * dm * 2));
  TRY(ensure(ctx, ctx->attn_enc, static_cast<size_t>(Ta) * dm * 2));
  TRY(ensure(ctx, ctx->ffn_enc, static_cast<size_t>(Ta) * c.encoder_ffn_dim * 2));
  for (const EncLayerW& L : W.enc) {
    KL("layernorm", 0, 6.0 * Ta * dm, layernorm_rows(ctx->xenc.as<float>(), Ta, dm, L.ln1_g, L.ln1_b, 1e-5f, ctx->h16a.p, bf, s));
    ep.mode = EPI_STORE16;
    ep.act = ACT_NONE;
    ep.bias = L.qkv_b;
    ep.out = ctx->qkv_enc.p;
    ep.ldo = 3 * dm;
    KL("gemm:enc_qkv", gemm_flops(Ta, 3 * dm, dm), gemm_bytes(Ta, 3 * dm, dm, 2),
       gemm_tc(ctx->h16a.p, dm, L.qkv_w, dm, Ta, 3 * dm, dm, bf, ep, s));
    KL("window_attn", win_flops, 2.0 * Ta * 4 * dm,
       window_attention(ctx->qkv_enc.p, Ta, dm, c.encoder_heads, 64, D.windows,
                        static_cast<int>(P.windows.size()), P.max_window, ctx->attn_enc.p, bf,
                        ctx->status.as<unsigned>(), s));
    ep.mode = EPI_RESID32;
    ep.bias = L.o_b;
    ep.out = ctx->xenc.p;
    ep.ldo = dm;
    KL("gemm:enc_out", gemm_flops(Ta, dm, dm), gemm_bytes(Ta, dm, dm, 8),
       gemm_tc(ctx->attn_enc.p, dm, L.o_w, dm, Ta, dm, dm, bf, ep, s));
    KL("layernorm", 0, 6.0 * Ta * dm, layernorm_rows(ctx->xenc.as<float>(), Ta, dm, L.ln2_g, L.ln2_b, 1e-5f, ctx->h16a.p, bf, s));
    ep.mode = EPI_STORE16;
    ep.act = ACT_GELU;
    ep.bias = L.fc1_b;
    ep.out = ctx->ffn_enc.p;
    ep.ldo = c.encoder_ffn_dim;
    KL("gemm:enc_fc1", gemm_flops(Ta, c.encoder_ffn_dim, dm), gemm_bytes(Ta, c.encoder_ffn_dim, dm, 2),
       gemm_tc(ctx->h16a.p, dm, L.fc1_w, dm, Ta, c.encoder_ffn_dim, dm, bf, ep, s));
    ep.mode = EPI_RESID32;
    ep.act = ACT_NONE;
    ep.bias = L.fc2_b;
    ep.out = ctx->xenc.p;
    ep.ldo = dm;
    KL("gemm:enc_fc2", gemm_flops(Ta, dm, c.encoder_ffn_dim), gemm_bytes(Ta, dm, c.encoder_ffn_dim, 8),
       gemm_tc(ctx->ffn_enc.p, c.encoder_ffn_dim, L.fc2_w, c.encoder_ffn_dim, Ta, dm,
               c.encoder_ffn_dim, bf, ep, s));
  }
  // ln_post -> proj1 + GELU -> proj2 (src/audio_encoder.rs:816-821)
  TRY(ensure(ctx, ctx->proj1, static_cast<size_t>(Ta) * dm * 2));
  KL("layernorm", 0, 6.0 * Ta * dm, layernorm_rows(ctx->xenc.as<float>(), Ta, dm, W.lnp_g, W.lnp_b, 1e-5f, ctx->h16a.p, bf, s));
  ep.mode = EPI_STORE16;
  ep.act = ACT_GELU;
  ep.bias = W.p1_b;
  ep.out = ctx->proj1.p;
  ep.ldo = dm;
  KL("gemm:proj1", gemm_flops(Ta, dm, dm), gemm_bytes(Ta, dm, dm, 2),
     gemm_tc(ctx->h16a.p, dm, W.p1_w, dm, Ta, dm, dm, bf, ep, s));
  ep.act = ACT_NONE;
  ep.bias = W.p2_b;
  ep.out = out16;
  ep.ldo = c.output_dim;
  ep.row_map = p2_map;
  KL("gemm:proj2", gemm_flops(Ta, c.output_dim, dm), gemm_bytes(Ta, c.output_dim, dm, 2),
     gemm_tc(ctx->proj1.p, dm, W.p2_w, dm, Ta, c.output_dim, dm, bf, ep, s));
  return QA_OK;
}

int ensure_kv(qa_ctx* ctx, int pages) {
  const qa_cfg& c = ctx->cfg;
  if (pages <= ctx->kv_pages) return QA_OK;
  const size_t bytes = static_cast<size_t>(c.num_layers) * pages * c.num_kv_heads * 64 * c.head_dim * 2;
  TRY(ensure(ctx, ctx->kcache, bytes));
  TRY(ensure(ctx, ctx->vcache, bytes));
  // Page rows past a clip's end are read by the attention tiles and masked;
  // start them at zero so that 0 * (stale value) is always 0.  The clear is
  // ordered on the context's stream: the stream is non-blocking, so a memset
  // on the legacy default stream could run after the QKV epilogues of the
  // same pass had appended K/V and wipe them.
  CK(cudaMemsetAsync(ctx->kcache.p, 0, ctx->kcache.cap, ctx->stream));
  CK(cudaMemsetAsync(ctx->vcache.p, 0, ctx->vcache.cap, ctx->stream));
  ctx->kv_pages = pages;
  ctx->kv_cap_tokens = std::min(pages * 64, c.max_seq);
  return QA_OK;
}

// 28 decoder layers over ctx->hid [T_d][H] (16-bit), in place.
int run_decoder(qa_ctx* ctx, const Plan& P, const PlanDev& D) {
  const qa_cfg& c = ctx->cfg;
  const bool bf = ctx->bf16;
  cudaStream_t s = ctx->stream;
  const int T = P.T_d, H = c.hidden_size, hd = c.head_dim, nq = c.num_heads, nkv = c.num_kv_heads;
  const int I = c.intermediate_size, qd = nq * hd, ldq = (nq + 2 * nkv) * hd;
  const int nch = H / 128;  // 128-column blocks per row (folded RMSNorm statistics)
  TRY(ensure(ctx, ctx->ssq_attn, static_cast<size_t>(T) * nch * 4));
  TRY(ensure(ctx, ctx->ssq_mlp, static_cast<size_t>(T) * nch * 4));
  TRY(ensure(ctx, ctx->qkv, static_cast<size_t>(T) * ldq * 2));
  TRY(ensure(ctx, ctx->attn, static_cast<size_t>(T) * qd * 2));
  TRY(ensure(ctx, ctx->mlp, static_cast<size_t>(T) * I * 2));
  TRY(ensure_kv(ctx, P.total_pages));
  const size_t layer_kv = static_cast<size_t>(ctx->kv_pages) * nkv * 64 * hd;  // elements
  double attn_flops = 0;  // exact causal: 4 * hd * nq per (query, key <= query) pair
  for (int cl = 0; cl < P.n; ++cl) attn_flops += 4.0 * hd * nq * 0.5 * P.seq[cl] * (P.seq[cl] + 1.0);
  const float eps = static_cast<float>(c.rms_norm_eps);
  EpiParams ep;
  ep.status = ctx->status.as<unsigned>();
  ep.ssq_n = nch;
  ep.rms_d = static_cast<float>(H);
  ep.rms_eps = eps;
  // Each RMSNorm (rms_norm_row, src/cpu_decoder.rs:289-300) is folded into
  // the projection after it: its gain sits in the weights' columns, and the
  // GEMM epilogue scales row r by 1 / rms(r), computed from the block sums of
  // squares that the residual epilogue before it wrote (the first layer's
  // from row_ssq over the embedded input).
  KL("row_ssq", 0, 2.0 * T * H + 4.0 * T * nch,
     row_ssq(ctx->hid.p, T, H, ctx->ssq_mlp.as<float>(), bf, s));
  for (int l = 0; l < c.num_layers; ++l) {
    const DecLayerW& L = ctx->w.dec[l];
    PagedKV kv{ctx->kcache.as<uint16_t>() + l * layer_kv, ctx->vcache.as<uint16_t>() + l * layer_kv, 64};
    // QKV projection of the normed rows with (d) fused into its epilogue: Q
    // (normed + roped) lands in the q columns of ctx->qkv, K and V in this
    // layer's pages.
    ep.mode = EPI_QKV_ROPE;
    ep.ssq_in = ctx->ssq_mlp.as<float>();
    ep.ssq_out = nullptr;
    ep.act = ACT_NONE;
    ep.bias = nullptr;
    ep.out = ctx->qkv.p;
    ep.ldo = ldq;
    ep.rk.pos_of = D.pos_of;
    ep.rk.clip_of = D.clip_of;
    ep.rk.block_tab = D.block_tab;
    ep.rk.max_pages = P.max_pages;
    ep.rk.page_size = 64;
    ep.rk.kc = kv.k;
    ep.rk.vc = kv.v;
    ep.rk.cos_t = ctx->w.rope_cos;
    ep.rk.sin_t = ctx->w.rope_sin;
    ep.rk.qn = L.qn;
    ep.rk.kn = L.kn;
    ep.rk.eps = eps;
    ep.rk.nq = nq;
    ep.rk.nkv = nkv;
    KL("gemm:dec_qkv", gemm_flops(T, ldq, H), gemm_bytes(T, ldq, H, 2),
       gemm_tc(ctx->hid.p, H, L.qkv_w, H, T, ldq, H, bf, ep, s, 0));
    KL("causal_attn", attn_flops, T * (2.0 * qd * 2 + 2.0 * nkv * hd * 2),
       causal_attention_tc(ctx->qkv.p, ldq, T, nq, nkv, hd, D.tiles,
                           static_cast<int>(P.tiles.size()), D.block_tab, P.max_pages, kv,
                           ctx->kv_pages, ctx->attn.p, bf, ctx->status.as<unsigned>(), s));
    ep.mode = EPI_RESID16;
    ep.out = ctx->hid.p;
    ep.ldo = H;
    ep.ssq_in = nullptr;
    ep.ssq_out = ctx->ssq_attn.as<float>();  // statistics of the post-attention norm
    KL("gemm:dec_o", gemm_flops(T, H, qd), gemm_bytes(T, H, qd, 4) + 4.0 * T * nch,
       gemm_tc(ctx->attn.p, qd, L.o_w, qd, T, H, qd, bf, ep, s));
    ep.mode = EPI_SWIGLU16;
    ep.out = ctx->mlp.p;
    ep.ldo = I;
    ep.ssq_in = ctx->ssq_attn.as<float>();
    ep.ssq_out = nullptr;
    KL("gemm:dec_gate_up", gemm_flops(T, 2 * I, H), gemm_bytes(T, I, H, 2) + 2.0 * I * H,
       gemm_tc(ctx->hid.p, H, L.gu_w, H, T, 2 * I, H, bf, ep, s, 0));
    ep.mode = EPI_RESID16;
    ep.out = ctx->hid.p;
    ep.ldo = H;
    ep.ssq_in = nullptr;
    ep.ssq_out = ctx->ssq_mlp.as<float>();  // statistics of the next layer's input norm
    KL("gemm:dec_down", gemm_flops(T, H, I), gemm_bytes(T, H, I, 4) + 4.0 * T * nch,
       gemm_tc(ctx->mlp.p, I, L.down_w, I, T, H, I, bf, ep, s));
  }
  return QA_OK;
}

// Timestamp head over `rows` of a hidden buffer (kind 0 f16, 1 bf16, 2 f32).
int run_head(qa_ctx* ctx, const void* hidden, int kind, int n_hidden, const int* rows_dev, int R,
             bool want_logits, bool want_normed) {
  const qa_cfg& c = ctx->cfg;
  cudaStream_t s = ctx->stream;
  const int H = c.hidden_size;
  TRY(ensure(ctx, ctx->head_a, static_cast<size_t>(R) * 2 * H * 2));
  TRY(ensure(ctx, ctx->head_keys, static_cast<size_t>(R) * 8));
  TRY(ensure(ctx, ctx->head_raw, static_cast<size_t>(R) * 8));
  if (want_logits) TRY(ensure(ctx, ctx->head_logits, static_cast<size_t>(R) * c.num_labels * 4));
  if (want_normed) TRY(ensure(ctx, ctx->head_normed, static_cast<size_t>(R) * H * 4));
  KL("head_norm", 0, R * (H * (kind == 2 ? 4.0 : 2.0) + 4.0 * H),
     head_gather_norm(hidden, kind, n_hidden, rows_dev, R, H, ctx->w.final_norm,
                      static_cast<float>(c.rms_norm_eps), ctx->head_a.p,
                      want_normed ? ctx->head_normed.as<float>() : nullptr,
                      ctx->badflag.as<int>(), s));
  CK(cudaMemsetAsync(ctx->head_keys.p, 0, static_cast<size_t>(R) * 8, s));
  EpiParams ep;
  ep.status = ctx->status.as<unsigned>();
  ep.mode = EPI_ARGMAX;
  ep.out = want_logits ? ctx->head_logits.p : nullptr;
  ep.ldo = c.num_labels;
  ep.keys = ctx->head_keys.as<unsigned long long>();
  KL("gemm:head", gemm_flops(R, c.num_labels, 2 * H), gemm_bytes(R, c.num_labels, 2 * H, want_logits ? 4 : 0),
     gemm_tc(ctx->head_a.p, 2 * H, ctx->w.head_w2, 2 * H, R, c.num_labels, 2 * H, true, ep, s));
  KL("argmax", 0, 16.0 * R, argmax_finalize(ctx->head_keys.as<unsigned long long>(), R, c.timestamp_segment_time_ms,
                     ctx->head_raw.as<long long>(), s));
  return QA_OK;
}

int reset_flags(qa_ctx* ctx) {
  CK(cudaMemsetAsync(ctx->status.p, 0, 4, ctx->stream));
  CK(cudaMemsetAsync(ctx->badflag.p, 0, 4, ctx->stream));
  return QA_OK;
}

int need_loaded(qa_ctx* ctx) {
  if (!ctx) return QA_ERR_ARG;
  if (!ctx->loaded) return fail(ctx, QA_ERR_STATE, "qa_load has not succeeded on this context");
  CK(cudaSetDevice(ctx->device));
  ctx->err.clear();
  ctx->launches = 0;
  return QA_OK;
}

float elapsed(qa_ctx* ctx, int a, int b) {
  float ms = 0.f;
  cudaEventElapsedTime(&ms, ctx->ev[a], ctx->ev[b]);
  return ms;
}

float elapsed(const Staged& S, int a, int b) {
  float ms = 0.f;
  cudaEventElapsedTime(&ms, S.ev[a], S.ev[b]);
  return ms;
}

// The oldest batch in `state`, or nullptr.
Staged* oldest(qa_ctx* ctx, int state) {
  Staged* best = nullptr;
  for (auto& sl : ctx->slots)
    if (sl && sl->state == state && (!best || sl->seq < best->seq)) best = sl.get();
  return best;
}

// Bounded wait for one event.
int wait_event(qa_ctx* ctx, cudaEvent_t e) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaEventQuery(e);
    if (q == cudaSuccess) return QA_OK;
    if (q != cudaErrorNotReady)
      return fail(ctx, QA_ERR_CUDA, "device error: %s", cudaGetErrorString(q));
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0)
                        .count();
    if (ms > ctx->timeout_ms)
      return fail(ctx, QA_ERR_TIMEOUT, "device did not finish within %d ms", ctx->timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// ------------------------------------------------------------ Local Head

constexpr int kLhDim = 128, kLhQwen = 1024, kLhTaps = 5;

// `_mel_filterbank` of the Local Head (src/local_head.rs:927-973): HTK mel
// points over 0..8 kHz, floored bin edges of a 512-point FFT, triangles, each
// row normalised to unit sum; [80][257].
std::vector<float> lh_mel_bank() {
  auto hz_to_mel = [](double hz) { return 2595.0 * std::log10(1.0 + hz / 700.0); };
  auto mel_to_hz = [](double m) { return 700.0 * (std::pow(10.0, m / 2595.0) - 1.0); };
  const double lo = hz_to_mel(0.0), hi = hz_to_mel(8000.0);
  std::vector<int> edge(kLhMels + 2);
  for (int i = 0; i < kLhMels + 2; ++i) {
    const double p = mel_to_hz(lo + (hi - lo) * i / (kLhMels + 1));
    edge[i] = static_cast<int>(std::max<long long>(static_cast<long long>(std::floor(513.0 * p / 16000.0)), 0));
  }
  std::vector<float> bank(static_cast<size_t>(kLhMels) * kLhBins, 0.f);
  for (int m = 0; m < kLhMels; ++m) {
    const int l = edge[m], c = std::max(edge[m + 1], l + 1);
    const int r = std::min(std::max(edge[m + 2], c + 1), kLhBins - 1);
    if (c >= kLhBins) continue;
    float* row = &bank[static_cast<size_t>(m) * kLhBins];
    for (int i = 0; i < c - l; ++i) row[l + i] = static_cast<float>(i) / (c - l);
    for (int i = 0; i < r - c; ++i) row[c + i] = 1.0f - static_cast<float>(i) / (r - c);
    float tot = 0.f;
    for (int b = 0; b < kLhBins; ++b) tot += row[b];
    if (tot > 0.f)
      for (int b = 0; b < kLhBins; ++b) row[b] /= tot;
  }
  return bank;
}

// The bf16 pair of an f32: hi = bf16(v), lo = bf16(v - hi).
void split_bf16(float v, uint16_t* hi, uint16_t* lo) {
  *hi = f32_to_bf16(v);
  *lo = f32_to_bf16(v - bf16_to_f32(*hi));
}

// B operand rows of a three-term product: for output row d, the K-blocks of
// `width` inputs each hold [w_hi | w_hi | w_lo] (zero past `n_in`).
void put_b3(std::vector<uint16_t>& dst, size_t row_off, int width, int n_in,
            const std::function<float(int)>& w) {
  for (int i = 0; i < width; ++i) {
    uint16_t h = 0, l = 0;
    if (i < n_in) split_bf16(w(i), &h, &l);
    dst[row_off + i] = h;
    dst[row_off + width + i] = h;
    dst[row_off + 2 * width + i] = l;
  }
}

int lh_load(qa_ctx* ctx, const qa_tensor* t, int n, const float* mean, const float* stdv) {
  std::map<std::string, const qa_tensor*> by;
  for (int i = 0; i < n; ++i)
    if (t[i].name) by[t[i].name] = &t[i];
  std::map<std::string, std::vector<float>> w;
  auto get = [&](const char* name, std::vector<int64_t> shape) -> int {
    auto it = by.find(name);
    if (it == by.end()) return fail(ctx, QA_ERR_WEIGHTS, "local head tensor %s is missing", name);
    const qa_tensor& x = *it->second;
    bool ok = x.dtype == QA_DTYPE_F32 && x.ndim == static_cast<int>(shape.size()) && x.data;
    size_t count = 1;
    for (int d = 0; ok && d < x.ndim; ++d) {
      ok = x.shape[d] == shape[d];
      count *= static_cast<size_t>(shape[d]);
    }
    if (!ok) return fail(ctx, QA_ERR_WEIGHTS, "local head tensor %s is not F32 of the expected shape", name);
    const float* p = static_cast<const float*>(x.data);
    w[name].assign(p, p + count);
    return QA_OK;
  };
  const int D = kLhDim;
  TRY(get("audio.0.weight", {D, kLhFeat, kLhTaps}));
  TRY(get("audio.0.bias", {D}));
  TRY(get("audio.2.weight", {D, D, kLhTaps}));
  TRY(get("audio.2.bias", {D}));
  TRY(get("context_projection.weight", {D, kLhQwen}));
  TRY(get("context_projection.bias", {D}));
  TRY(get("role_embedding.weight", {4, D}));
  TRY(get("endpoint_embedding.weight", {2, D}));
  for (const char* a : {"context_attention", "audio_attention"}) {
    const std::string p(a);
    TRY(get((p + ".in_proj_weight").c_str(), {3 * D, D}));
    TRY(get((p + ".in_proj_bias").c_str(), {3 * D}));
    TRY(get((p + ".out_proj.weight").c_str(), {D, D}));
    TRY(get((p + ".out_proj.bias").c_str(), {D}));
  }
  for (const char* nm : {"query_norm", "audio_norm"}) {
    TRY(get((std::string(nm) + ".weight").c_str(), {D}));
    TRY(get((std::string(nm) + ".bias").c_str(), {D}));
  }
  TRY(get("activity_bias.weight", {1, D}));
  TRY(get("activity_bias.bias", {1}));
  TRY(get("boundary_bias.weight", {1, D}));
  TRY(get("boundary_bias.bias", {1}));
  TRY(get("qwen_prior", {13}));
  {  // a scalar: one F32 element of any rank (src/local_head.rs:834-846)
    auto it = by.find("derivative_scale");
    long long cnt = 1;
    if (it != by.end())
      for (int d = 0; d < it->second->ndim; ++d) cnt *= it->second->shape[d];
    if (it == by.end() || it->second->dtype != QA_DTYPE_F32 || cnt != 1 || !it->second->data)
      return fail(ctx, QA_ERR_WEIGHTS, "local head tensor derivative_scale must be one F32 value");
    w["derivative_scale"] = {*static_cast<const float*>(it->second->data)};
  }
  for (int c = 0; c < kLhFeat; ++c)
    if (!std::isfinite(mean[c]) || !std::isfinite(stdv[c]) || !(stdv[c] > 0.f))
      return fail(ctx, QA_ERR_WEIGHTS, "normalizer must be finite with positive std");

  auto L = std::make_unique<LocalHeadDev>();
  int rc = QA_OK;
  // the two convs: B row c, tap k = [w_hi | w_hi | w_lo] over the 128 input channels
  for (int layer = 0; layer < 2; ++layer) {
    const std::vector<float>& cw = w[layer == 0 ? "audio.0.weight" : "audio.2.weight"];
    const int cin = layer == 0 ? kLhFeat : D;
    std::vector<uint16_t> b(static_cast<size_t>(D) * kLhTaps * kLhXw);
    for (int c = 0; c < D; ++c)
      for (int k = 0; k < kLhTaps; ++k)
        put_b3(b, (static_cast<size_t>(c) * kLhTaps + k) * kLhXw, kLhCh, cin,
               [&](int ic) { return cw[(static_cast<size_t>(c) * cin + ic) * kLhTaps + k]; });
    void* dev = upload<void>(ctx, b.data(), b.size() * 2, &rc);
    if (rc) return rc;
    (layer == 0 ? L->conv1_w : L->conv2_w) = dev;
  }
  L->conv1_b = up_f32(ctx, w["audio.0.bias"], &rc);
  L->conv2_b = up_f32(ctx, w["audio.2.bias"], &rc);
  // audio attention k / v projections: rows 0..127 k, 128..255 v
  {
    const std::vector<float>& ip = w["audio_attention.in_proj_weight"];
    const std::vector<float>& ib = w["audio_attention.in_proj_bias"];
    std::vector<uint16_t> b(static_cast<size_t>(2 * D) * kLhXw);
    for (int r = 0; r < 2 * D; ++r)
      put_b3(b, static_cast<size_t>(r) * kLhXw, kLhCh, D,
             [&](int j) { return ip[static_cast<size_t>(D + r) * D + j]; });
    L->kv_w = upload<void>(ctx, b.data(), b.size() * 2, &rc);
    L->kv_b = up_f32(ctx, std::vector<float>(ib.begin() + D, ib.end()), &rc);
  }
  // context projection over [hi | lo | hi] rows of the 1024-wide context
  {
    const std::vector<float>& cw = w["context_projection.weight"];
    std::vector<uint16_t> b(static_cast<size_t>(D) * 3 * kLhQwen);
    for (int d = 0; d < D; ++d)
      put_b3(b, static_cast<size_t>(d) * 3 * kLhQwen, kLhQwen, kLhQwen,
             [&](int j) { return cw[static_cast<size_t>(d) * kLhQwen + j]; });
    L->ctx_w = upload<void>(ctx, b.data(), b.size() * 2, &rc);
    L->ctx_b = up_f32(ctx, w["context_projection.bias"], &rc);
  }
  if (rc) return rc;
  // the tail's 128 x 128 matrices, transposed to [in][out]
  auto up_t = [&](const std::vector<float>& m, size_t off) {
    std::vector<float> tr(static_cast<size_t>(D) * D);
    for (int o = 0; o < D; ++o)
      for (int i = 0; i < D; ++i) tr[static_cast<size_t>(i) * D + o] = m[off + static_cast<size_t>(o) * D + i];
    return up_f32(ctx, tr, &rc);
  };
  auto slice = [&](const std::vector<float>& v, size_t a, size_t b2) {
    return up_f32(ctx, std::vector<float>(v.begin() + a, v.begin() + b2), &rc);
  };
  LhTailW& T = L->tail;
  const std::vector<float>& cip = w["context_attention.in_proj_weight"];
  const std::vector<float>& cib = w["context_attention.in_proj_bias"];
  const std::vector<float>& aip = w["audio_attention.in_proj_weight"];
  const std::vector<float>& aib = w["audio_attention.in_proj_bias"];
  const size_t blk = static_cast<size_t>(D) * D;
  T.cq = up_t(cip, 0);
  T.ck = up_t(cip, blk);
  T.cv = up_t(cip, 2 * blk);
  T.co = up_t(w["context_attention.out_proj.weight"], 0);
  T.aq = up_t(aip, 0);
  T.ao = up_t(w["audio_attention.out_proj.weight"], 0);
  T.cbq = slice(cib, 0, D);
  T.cbk = slice(cib, D, 2 * D);
  T.cbv = slice(cib, 2 * D, 3 * D);
  T.co_b = up_f32(ctx, w["context_attention.out_proj.bias"], &rc);
  T.abq = slice(aib, 0, D);
  T.ao_b = up_f32(ctx, w["audio_attention.out_proj.bias"], &rc);
  T.ctx_b = L->ctx_b;
  T.role = up_f32(ctx, w["role_embedding.weight"], &rc);
  T.endpoint = up_f32(ctx, w["endpoint_embedding.weight"], &rc);
  T.qn_w = up_f32(ctx, w["query_norm.weight"], &rc);
  T.qn_b = up_f32(ctx, w["query_norm.bias"], &rc);
  T.an_w = up_f32(ctx, w["audio_norm.weight"], &rc);
  T.an_b = up_f32(ctx, w["audio_norm.bias"], &rc);
  T.act_w = up_f32(ctx, w["activity_bias.weight"], &rc);
  T.bnd_w = up_f32(ctx, w["boundary_bias.weight"], &rc);
  T.prior = up_f32(ctx, w["qwen_prior"], &rc);
  T.act_b = w["activity_bias.bias"][0];
  T.bnd_b = w["boundary_bias.bias"][0];
  T.derivative_scale = w["derivative_scale"][0];
  // feature constants: symmetric Hann (src/local_head.rs:917-925), the mel
  // bank and its nonzero ranges, the normalizer, the FFT twiddles
  LhFeatConst& F = L->feat;
  {
    std::vector<float> hann(kLhFrameLen);
    for (int i = 0; i < kLhFrameLen; ++i)
      hann[i] = static_cast<float>(0.5 - 0.5 * std::cos(2.0 * M_PI * i / (kLhFrameLen - 1)));
    F.hann = up_f32(ctx, hann, &rc);
    const std::vector<float> bank = lh_mel_bank();
    F.bank = up_f32(ctx, bank, &rc);
    std::vector<int2> range(kLhMels, make_int2(0, 0));
    for (int m = 0; m < kLhMels; ++m) {
      int a = -1, z = -1;
      for (int b = 0; b < kLhBins; ++b)
        if (bank[static_cast<size_t>(m) * kLhBins + b] != 0.f) {
          if (a < 0) a = b;
          z = b + 1;
        }
      if (a >= 0) range[m] = make_int2(a, z);
    }
    F.bank_range = upload<int2>(ctx, range.data(), range.size() * sizeof(int2), &rc);
    F.mean = up_f32(ctx, std::vector<float>(mean, mean + kLhFeat), &rc);
    F.stdv = up_f32(ctx, std::vector<float>(stdv, stdv + kLhFeat), &rc);
    std::vector<double2> tw(kLhNfft / 2);
    for (int k = 0; k < kLhNfft / 2; ++k) {
      const double a = 2.0 * M_PI * k / kLhNfft;
      tw[k] = make_double2(std::cos(a), -std::sin(a));
    }
    F.twiddle = upload<double2>(ctx, tw.data(), tw.size() * sizeof(double2), &rc);
  }
  if (rc) return rc;
  ctx->lh = std::move(L);
  ctx->lh_on = true;
  return QA_OK;
}

// One Local Head pass over E endpoints of n_clips clips, all inputs on the
// device: samples (clip ranges in `clips`), the head's logits [E][n_labels]
// and unfolded norm rows [E][1024]; intervals [E/2][2] seconds out.
int run_local_head(qa_ctx* ctx, int E, int n_clips, const LhClip* clips, const int* ep_clip,
                   int max_slots, const float* samples, const float* logits, int n_labels,
                   const float* normed, double* intervals, float* feat_out) {
  LocalHeadDev& L = *ctx->lh;
  cudaStream_t s = ctx->stream;
  const int Wt = E / 2, ctx_rows = E + Wt;
  const size_t conv_rows = static_cast<size_t>(E) * kLhRows;
  const size_t frame_rows = static_cast<size_t>(E) * kLhFrames;
  TRY(ensure(ctx, L.raw, static_cast<size_t>(E) * 8));
  TRY(ensure(ctx, L.fixed, static_cast<size_t>(E) * 8));
  TRY(ensure(ctx, L.x1, conv_rows * kLhXw * 2));
  TRY(ensure(ctx, L.x2, conv_rows * kLhXw * 2));
  TRY(ensure(ctx, L.audio, frame_rows * kLhDim * 4));
  TRY(ensure(ctx, L.asplit, frame_rows * kLhXw * 2));
  TRY(ensure(ctx, L.kv, frame_rows * 2 * kLhDim * 4));
  TRY(ensure(ctx, L.ctxa, static_cast<size_t>(ctx_rows) * 3 * kLhQwen * 2));
  TRY(ensure(ctx, L.proj, static_cast<size_t>(ctx_rows) * kLhDim * 4));
  TRY(ensure(ctx, L.off, static_cast<size_t>(E) * 4));
  unsigned* status = ctx->status.as<unsigned>();
  KL("lh_argmax", 0, 4.0 * E * n_labels,
     lh_masked_argmax(logits, E, n_labels, clips, ep_clip, L.raw.as<long long>(), s));
  KL("lh_fix", 0, 16.0 * E,
     lh_fix(L.raw.as<long long>(), clips, n_clips, max_slots, L.fixed.as<long long>(), s));
  // 41 FFTs of 512 points per endpoint (5 N log2 N flops each, f64)
  KL("lh_features", 41.0 * 5 * 512 * 9 * E, 41.0 * 400 * 4 * E + 2.0 * conv_rows * kLhXw * 2,
     lh_features(samples, clips, ep_clip, L.fixed.as<long long>(), E, L.feat, L.x1.as<uint16_t>(),
                 L.x2.as<uint16_t>(), feat_out, s));
  EpiParams ep;
  ep.status = status;
  ep.mode = EPI_SPLIT3;
  ep.act = ACT_GELU;
  ep.conv_kb = kLhXw / 64;
  ep.row_period = kLhRows;
  ep.row_valid = kLhFrames;
  ep.bias = L.conv1_b;
  ep.out = L.x2.p;
  ep.ldo = kLhXw;
  ep.row_out_period = kLhRows;
  ep.row_out_off = 2;
  const int Kc = kLhTaps * kLhXw;
  KL("gemm:lh_conv1", 2.0 * conv_rows * kLhDim * Kc, conv_rows * kLhXw * 4.0,
     gemm_tc(L.x1.p, kLhXw, L.conv1_w, Kc, static_cast<int>(conv_rows), kLhDim, Kc, true, ep, s, kLhDim));
  ep.bias = L.conv2_b;
  ep.out = L.asplit.p;
  ep.out2 = L.audio.as<float>();
  ep.ldo2 = kLhDim;
  ep.row_out_period = kLhFrames;
  ep.row_out_off = 0;
  KL("gemm:lh_conv2", 2.0 * conv_rows * kLhDim * Kc, conv_rows * kLhXw * 2.0 + frame_rows * (kLhXw * 2.0 + kLhDim * 4.0),
     gemm_tc(L.x2.p, kLhXw, L.conv2_w, Kc, static_cast<int>(conv_rows), kLhDim, Kc, true, ep, s, kLhDim));
  EpiParams e2;
  e2.status = status;
  e2.mode = EPI_STORE32;
  e2.bias = L.kv_b;
  e2.out = L.kv.p;
  e2.ldo = 2 * kLhDim;
  KL("gemm:lh_kv", 2.0 * frame_rows * 2 * kLhDim * kLhXw, frame_rows * (kLhXw * 2.0 + 2 * kLhDim * 4.0),
     gemm_tc(L.asplit.p, kLhXw, L.kv_w, kLhXw, static_cast<int>(frame_rows), 2 * kLhDim, kLhXw, true, e2, s));
  KL("lh_ctx_pack", 0, E * kLhQwen * 4.0 + ctx_rows * 3.0 * kLhQwen * 2,
     lh_ctx_pack(normed, E, kLhQwen, L.ctxa.as<uint16_t>(), s));
  e2.bias = L.ctx_b;
  e2.out = L.proj.p;
  e2.ldo = kLhDim;
  KL("gemm:lh_ctx", 2.0 * ctx_rows * kLhDim * 3 * kLhQwen, ctx_rows * (3.0 * kLhQwen * 2 + kLhDim * 4.0),
     gemm_tc(L.ctxa.p, 3 * kLhQwen, L.ctx_w, 3 * kLhQwen, ctx_rows, kLhDim, 3 * kLhQwen, true, e2, s));
  KL("lh_tail", 2.0 * E * (12.0 * kLhDim * kLhDim + 2.0 * kLhFrames * kLhDim), E * (kLhFrames * 2.0 * kLhDim * 4 + 14.0 * kLhDim * 4),
     lh_tail(L.proj.as<float>(), L.kv.as<float>(), L.audio.as<float>(), clips, ep_clip, E, L.tail,
             L.off.as<float>(), s));
  KL("lh_repair", 0, 12.0 * E,
     lh_repair(L.fixed.as<long long>(), L.off.as<float>(), clips, n_clips, intervals, s));
  return QA_OK;
}

int lh_valid_classes(long long n_samples, int n_labels) {
  const double ms = static_cast<double>(n_samples) * 1000.0 / 16000.0;
  const long long by_audio = static_cast<long long>(std::floor(ms / 80.0)) + 1;
  return static_cast<int>(std::min<long long>(std::max<long long>(by_audio, 1), n_labels));
}

}  // namespace

// Bounded wait for everything queued on the context's stream.
int qa::wait_stream(qa_ctx* ctx) {
  cudaEvent_t e = ctx->ev[11];
  CK(cudaEventRecord(e, ctx->stream));
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaEventQuery(e);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady)
      return fail(ctx, QA_ERR_CUDA, "device error: %s", cudaGetErrorString(q));
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0)
                        .count();
    if (ms > ctx->timeout_ms)
      return fail(ctx, QA_ERR_TIMEOUT, "device did not finish within %d ms", ctx->timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  if (!ctx->prof_recs.empty()) prof_resolve(ctx);
  return QA_OK;
}

int qa::check_status(qa_ctx* ctx) {
  unsigned st = 0;
  int bad = 0;
  CK(cudaMemcpy(&st, ctx->status.p, sizeof st, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(&bad, ctx->badflag.p, sizeof bad, cudaMemcpyDeviceToHost));
  if (st & kStatusTimeout)
    return fail(ctx, QA_ERR_TIMEOUT, "a tensor-core pipeline wait ran out (status %u)", st);
  if (bad) return flag_error(ctx, bad);
  return QA_OK;
}


// ====================================================================== C ABI

extern "C" {

int qa_open(int device, int half, qa_ctx** out) {
  if (!out) return QA_ERR_ARG;
  *out = nullptr;
  if (half != QA_HALF_F16 && half != QA_HALF_BF16) return QA_ERR_ARG;
  auto* ctx = new qa_ctx();
  ctx->device = device;
  ctx->half = half;
  ctx->bf16 = half == QA_HALF_BF16;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    delete ctx;
    return QA_ERR_CUDA;
  }
  if (cudaSetDevice(device) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete ctx;
    return QA_ERR_CUDA;
  }
  ctx->stream = ctx->own_stream;
  for (auto& e : ctx->ev) cudaEventCreate(&e);
  if (ensure(ctx, ctx->status, 16) || ensure(ctx, ctx->badflag, 16)) {
    qa_close(ctx);
    return QA_ERR_OOM;
  }
  cudaMemset(ctx->status.p, 0, 16);
  cudaMemset(ctx->badflag.p, 0, 16);
  *out = ctx;
  return QA_OK;
}

int qa_load(qa_ctx* ctx, const qa_tensor* tensors, int n, const qa_cfg* cfg) {
  if (!ctx || !tensors || !cfg || n <= 0) return QA_ERR_ARG;
  if (ctx->loaded) return fail(ctx, QA_ERR_STATE, "weights are already loaded on this context");
  CK(cudaSetDevice(ctx->device));
  ctx->cfg = *cfg;
  if (ctx->cfg.max_seq <= 0) ctx->cfg.max_seq = 8192;
  const int rc = load_weights(ctx, tensors, n, ctx->cfg);
  if (rc) {
    for (void* p : ctx->allocations) cudaFree(p);
    ctx->allocations.clear();
    return rc;
  }
  ctx->loaded = true;
  return QA_OK;
}

int qa_close(qa_ctx* ctx) {
  if (!ctx) return QA_ERR_ARG;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  for (void* p : ctx->allocations) cudaFree(p);
  DevBuf* bufs[] = {&ctx->samples, &ctx->mel_scratch, &ctx->mel_chunked, &ctx->maxkey,
                    &ctx->mel_frames, &ctx->mel_spec,
                    &ctx->clips_dev, &ctx->idx_dev, &ctx->act1, &ctx->cols, &ctx->act2,
                    &ctx->act3, &ctx->xenc, &ctx->h16a, &ctx->qkv_enc, &ctx->attn_enc,
                    &ctx->ffn_enc, &ctx->proj1, &ctx->emb_out, &ctx->hid, &ctx->ssq_attn,
                    &ctx->ssq_mlp, &ctx->qkv,
                    &ctx->attn, &ctx->mlp, &ctx->kcache, &ctx->vcache, &ctx->head_a,
                    &ctx->head_keys, &ctx->head_raw, &ctx->head_logits, &ctx->head_normed,
                    &ctx->hidden_f32, &ctx->status, &ctx->badflag};
  for (DevBuf* b : bufs)
    if (b->p) cudaFree(b->p);
  if (ctx->lh) {
    LocalHeadDev& L = *ctx->lh;
    for (DevBuf* b : {&L.raw, &L.fixed, &L.x1, &L.x2, &L.audio, &L.asplit, &L.kv, &L.ctxa, &L.proj,
                      &L.off, &L.iv, &L.samples, &L.logits, &L.normed, &L.plan, &L.feat_out})
      if (b->p) cudaFree(b->p);
  }
  if (ctx->pin_in.p) cudaFreeHost(ctx->pin_in.p);
  if (ctx->pin_out.p) cudaFreeHost(ctx->pin_out.p);
  if (ctx->pin_res.p) cudaFreeHost(ctx->pin_res.p);
  for (auto& sl : ctx->slots) {
    if (!sl) continue;
    for (PinBuf* b : {&sl->pin_samples, &sl->pin_plan, &sl->pin_res, &sl->pin_lh})
      if (b->p) cudaFreeHost(b->p);
    for (DevBuf* b : {&sl->samples, &sl->plan, &sl->lh_plan})
      if (b->p) cudaFree(b->p);
    for (auto& e : sl->ev)
      if (e) cudaEventDestroy(e);
  }
  for (auto& e : ctx->ev)
    if (e) cudaEventDestroy(e);
  for (auto& e : ctx->prof_pool)
    if (e) cudaEventDestroy(e);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  if (ctx->copy_stream) cudaStreamDestroy(ctx->copy_stream);
  delete ctx;
  return QA_OK;
}

const char* qa_last_error(const qa_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

int qa_set_timeout_ms(qa_ctx* ctx, int ms) {
  if (!ctx || ms <= 0) return QA_ERR_ARG;
  ctx->timeout_ms = ms;
  return QA_OK;
}

int qa_half(const qa_ctx* ctx) { return ctx ? ctx->half : -1; }

int qa_get_timings(const qa_ctx* ctx, qa_timings* out) {
  if (!ctx || !out) return QA_ERR_ARG;
  *out = ctx->timings;
  return QA_OK;
}

int qa_mel(qa_ctx* ctx, const float* samples, int64_t n, float* out, int64_t out_len,
           int* n_frames) {
  TRY(need_loaded(ctx));
  if (!samples || !out) return fail(ctx, QA_ERR_ARG, "null buffer");
  if (n <= 0) return fail(ctx, QA_ERR_SHAPE, "empty audio");
  const int frames = static_cast<int>(n / 160);
  if (out_len < static_cast<int64_t>(frames) * 128)
    return fail(ctx, QA_ERR_SHAPE, "out holds %lld floats, needs %d", (long long)out_len, frames * 128);
  if (n_frames) *n_frames = frames;
  if (frames == 0) return QA_OK;
  cudaStream_t s = ctx->stream;
  TRY(ensure(ctx, ctx->samples, n * 4));
  TRY(ensure(ctx, ctx->mel_scratch, static_cast<size_t>(frames) * 128 * 4));
  TRY(ensure(ctx, ctx->mel_chunked, static_cast<size_t>(frames) * 128 * 4));
  TRY(ensure(ctx, ctx->mel_frames, static_cast<size_t>(frames) * kMelDftK * 2));
  TRY(ensure(ctx, ctx->mel_spec, static_cast<size_t>(frames) * kMelDftRows * 4));
  TRY(ensure(ctx, ctx->maxkey, 16));
  TRY(ensure(ctx, ctx->clips_dev, sizeof(MelClip)));
  MelClip mc{0, static_cast<int>(n), 0, frames, 0};
  CK(cudaMemcpyAsync(ctx->clips_dev.p, &mc, sizeof mc, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(ctx->samples.p, samples, n * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemsetAsync(ctx->maxkey.p, 0, 4, s));
  const Weights& W = ctx->w;
  MelBank bank{W.fb_start, W.fb_len, W.fb_woff, W.fb_w};
  KL("mel", 2.0 * frames * kMelDftRows * kMelDftK, 4.0 * n + 512.0 * frames,
     mel_logpower_tc(ctx->samples.as<float>(), ctx->clips_dev.as<MelClip>(), 1, frames, frames,
                     W.mel_dft, bank, 1.0f / std::log(10.0f), ctx->mel_frames.p,
                     ctx->mel_spec.as<float>(), ctx->mel_scratch.as<float>(),
                     ctx->maxkey.as<unsigned>(), ctx->status.as<unsigned>(), s));
  ctx->launches += 2;  // mel_logpower_tc is three launches (rows, GEMM, power)
  KL("mel_finalize", 0, 1024.0 * frames, mel_finalize_rows(ctx->mel_scratch.as<float>(), frames, ctx->maxkey.as<unsigned>(),
                       ctx->mel_chunked.as<float>(), s));
  CK(cudaMemcpyAsync(out, ctx->mel_chunked.p, static_cast<size_t>(frames) * 128 * 4,
                     cudaMemcpyDeviceToHost, s));
  return wait_stream(ctx);
}

int qa_audio_embeds(qa_ctx* ctx, const float* mel, int n_mels, int valid_frames, uint16_t* out,
                    int64_t out_len) {
  TRY(need_loaded(ctx));
  const qa_cfg& c = ctx->cfg;
  if (!mel || !out) return fail(ctx, QA_ERR_ARG, "null buffer");
  if (n_mels != c.num_mel_bins) return fail(ctx, QA_ERR_SHAPE, "mel has %d bins, expected %d", n_mels, c.num_mel_bins);
  const int cs = 2 * c.n_window;
  const int na = static_cast<int>(audio_token_count(valid_frames, c.n_window));
  if (valid_frames <= 0 || na <= 0) return fail(ctx, QA_ERR_SHAPE, "audio produced 0 tokens (%d mel frames)", valid_frames);
  if (na > 16384) return fail(ctx, QA_ERR_CAP, "%d audio tokens exceed the tower's 16384", na);
  if (out_len < static_cast<int64_t>(na) * c.output_dim)
    return fail(ctx, QA_ERR_SHAPE, "audio tower returns %d x %d values, out holds %lld", na, c.output_dim, (long long)out_len);
  TRY(reset_flags(ctx));
  Plan P;
  P.n = 1;
  const int nch = (valid_frames + cs - 1) / cs;
  P.mel.push_back({0, 0, 0, valid_frames, 0});
  P.total_chunks = nch;
  P.chunk_clip.assign(nch, 0);
  plan_audio(P, c, {valid_frames});
  // chunk the mel on the host (src/audio_encoder.rs:763-790), zero padded
  const size_t chunk_elems = static_cast<size_t>(nch) * n_mels * cs;
  TRY(ensure_pin(ctx, ctx->pin_out, chunk_elems * 4));
  float* ch = static_cast<float*>(ctx->pin_out.p);
  std::memset(ch, 0, chunk_elems * 4);
  for (int i = 0; i < nch; ++i) {
    const int len = std::min(cs, valid_frames - i * cs);
    for (int m = 0; m < n_mels; ++m)
      std::memcpy(ch + (static_cast<size_t>(i) * n_mels + m) * cs,
                  mel + static_cast<size_t>(m) * valid_frames + static_cast<size_t>(i) * cs, len * 4);
  }
  TRY(ensure(ctx, ctx->mel_chunked, chunk_elems * 4));
  CK(cudaMemcpyAsync(ctx->mel_chunked.p, ch, chunk_elems * 4, cudaMemcpyHostToDevice, ctx->stream));
  PlanDev D{};
  TRY(upload_plan(ctx, P, {}, D, ctx->pin_in, ctx->idx_dev, ctx->stream));
  TRY(ensure(ctx, ctx->emb_out, static_cast<size_t>(na) * c.output_dim * 2));
  TRY(run_encoder(ctx, P, D, ctx->emb_out.p, nullptr));
  CK(cudaMemcpyAsync(out, ctx->emb_out.p, static_cast<size_t>(na) * c.output_dim * 2,
                     cudaMemcpyDeviceToHost, ctx->stream));
  TRY(wait_stream(ctx));
  return check_status(ctx);
}

int qa_ensure_capacity(qa_ctx* ctx, int need, int* cap) {
  TRY(need_loaded(ctx));
  const int target = std::min(((std::max(need, 1) + 255) / 256) * 256, ctx->cfg.max_seq);
  TRY(ensure_kv(ctx, (target + 63) / 64));
  if (cap) *cap = ctx->kv_cap_tokens;
  return QA_OK;
}

int qa_text_hidden(qa_ctx* ctx, const uint16_t* emb, int seq, float* out) {
  TRY(need_loaded(ctx));
  const qa_cfg& c = ctx->cfg;
  if (!emb || !out) return fail(ctx, QA_ERR_ARG, "null buffer");
  if (seq <= 0) return fail(ctx, QA_ERR_SHAPE, "empty sequence");
  if (seq > c.max_seq) return fail(ctx, QA_ERR_CAP, "prefill needs %d positions, max_seq is %d", seq, c.max_seq);
  TRY(qa_ensure_capacity(ctx, seq, nullptr));
  TRY(reset_flags(ctx));
  Plan P;
  P.n = 1;
  P.tok0 = {0};
  P.seq = {seq};
  P.T_d = seq;
  plan_decoder(P);
  PlanDev D{};
  TRY(upload_plan(ctx, P, {}, D, ctx->pin_in, ctx->idx_dev, ctx->stream));
  const int H = c.hidden_size;
  TRY(ensure(ctx, ctx->hid, static_cast<size_t>(seq) * H * 2));
  TRY(ensure(ctx, ctx->hidden_f32, static_cast<size_t>(seq) * H * 4));
  CK(cudaMemcpyAsync(ctx->hid.p, emb, static_cast<size_t>(seq) * H * 2, cudaMemcpyHostToDevice, ctx->stream));
  TRY(run_decoder(ctx, P, D));
  KL("widen", 0, 6.0 * seq * H, widen16(ctx->hid.p, static_cast<long long>(seq) * H, ctx->hidden_f32.as<float>(), ctx->bf16, ctx->stream));
  CK(cudaMemcpyAsync(out, ctx->hidden_f32.p, static_cast<size_t>(seq) * H * 4, cudaMemcpyDeviceToHost, ctx->stream));
  TRY(wait_stream(ctx));
  return check_status(ctx);
}

int qa_head(qa_ctx* ctx, const float* hidden, int seq, const int* rows, int n_rows,
            int64_t* raw_ms, float* logits, float* normed) {
  TRY(need_loaded(ctx));
  const qa_cfg& c = ctx->cfg;
  if (!hidden || !rows || !raw_ms) return fail(ctx, QA_ERR_ARG, "null buffer");
  if (n_rows <= 0) return QA_OK;
  for (int i = 0; i < n_rows; ++i)
    if (rows[i] < 0 || rows[i] >= seq) return fail(ctx, QA_ERR_SHAPE, "row %d out of range", rows[i]);
  TRY(reset_flags(ctx));
  const int H = c.hidden_size;
  TRY(ensure(ctx, ctx->hidden_f32, static_cast<size_t>(seq) * H * 4));
  TRY(ensure(ctx, ctx->idx_dev, static_cast<size_t>(n_rows) * 4));
  CK(cudaMemcpyAsync(ctx->hidden_f32.p, hidden, static_cast<size_t>(seq) * H * 4, cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemcpyAsync(ctx->idx_dev.p, rows, static_cast<size_t>(n_rows) * 4, cudaMemcpyHostToDevice, ctx->stream));
  TRY(run_head(ctx, ctx->hidden_f32.p, 2, seq, ctx->idx_dev.as<int>(), n_rows, logits != nullptr,
               normed != nullptr));
  CK(cudaMemcpyAsync(raw_ms, ctx->head_raw.p, static_cast<size_t>(n_rows) * 8, cudaMemcpyDeviceToHost, ctx->stream));
  if (logits)
    CK(cudaMemcpyAsync(logits, ctx->head_logits.p, static_cast<size_t>(n_rows) * c.num_labels * 4, cudaMemcpyDeviceToHost, ctx->stream));
  if (normed)
    CK(cudaMemcpyAsync(normed, ctx->head_normed.p, static_cast<size_t>(n_rows) * H * 4, cudaMemcpyDeviceToHost, ctx->stream));
  TRY(wait_stream(ctx));
  return check_status(ctx);
}

int qa_local_head_load(qa_ctx* ctx, const qa_tensor* tensors, int n, const float* mean,
                       const float* std_) {
  if (!ctx || !tensors || n <= 0 || !mean || !std_) return QA_ERR_ARG;
  if (ctx->lh) return fail(ctx, QA_ERR_STATE, "a Local Head is already loaded on this context");
  CK(cudaSetDevice(ctx->device));
  const size_t before = ctx->allocations.size();
  const int rc = lh_load(ctx, tensors, n, mean, std_);
  if (rc) {
    for (size_t i = before; i < ctx->allocations.size(); ++i) cudaFree(ctx->allocations[i]);
    ctx->allocations.resize(before);
  }
  return rc;
}

int qa_set_local_head_enabled(qa_ctx* ctx, int enabled) {
  if (!ctx) return QA_ERR_ARG;
  if (enabled && !ctx->lh) return fail(ctx, QA_ERR_STATE, "this checkpoint has no local_head/ package");
  ctx->lh_on = enabled != 0;
  return QA_OK;
}

int qa_local_head_enabled(const qa_ctx* ctx) { return ctx && ctx->lh && ctx->lh_on ? 1 : 0; }

int qa_local_head_refine(qa_ctx* ctx, const float* samples, int64_t n, int n_words,
                         const float* logits, int n_labels, const float* hidden, int hidden_size,
                         double* intervals, int64_t* fixed_ms, float* offsets_ms,
                         float* features) {
  if (!ctx) return QA_ERR_ARG;
  if (!ctx->lh) return fail(ctx, QA_ERR_STATE, "no Local Head is loaded on this context");
  CK(cudaSetDevice(ctx->device));
  ctx->err.clear();
  ctx->launches = 0;
  if (hidden_size != kLhQwen)
    return fail(ctx, QA_ERR_SHAPE, "hidden size %d != local head context input %d", hidden_size, kLhQwen);
  if (n <= 0 || !samples) return fail(ctx, QA_ERR_SHAPE, "local head needs non-empty audio");
  if (n > 0x7FFFFFFF) return fail(ctx, QA_ERR_CAP, "%lld samples exceed the local head's range", (long long)n);
  if (n_labels <= 0) return fail(ctx, QA_ERR_SHAPE, "timestamp head has no classes");
  if (n_words < 0) return fail(ctx, QA_ERR_ARG, "negative word count");
  if (n_words == 0) return QA_OK;
  if (!logits || !hidden || !intervals) return fail(ctx, QA_ERR_ARG, "null buffer");
  const int E = 2 * n_words;
  if (static_cast<size_t>(E) * 20 > 200 * 1024)
    return fail(ctx, QA_ERR_CAP, "%d words exceed the per-clip repair capacity", n_words);
  LocalHeadDev& L = *ctx->lh;
  cudaStream_t s = ctx->stream;
  TRY(reset_flags(ctx));
  LhClip cl{0, static_cast<int>(n), 0, n_words, lh_valid_classes(n, n_labels)};
  std::vector<uint8_t> plan(pad16<LhClip>(1) + static_cast<size_t>(E) * 4, 0);
  std::memcpy(plan.data(), &cl, sizeof cl);
  TRY(ensure(ctx, L.samples, static_cast<size_t>(n) * 4));
  TRY(ensure(ctx, L.logits, static_cast<size_t>(E) * n_labels * 4));
  TRY(ensure(ctx, L.normed, static_cast<size_t>(E) * kLhQwen * 4));
  TRY(ensure(ctx, L.plan, plan.size()));
  TRY(ensure(ctx, L.iv, static_cast<size_t>(E) * 8));
  if (features) TRY(ensure(ctx, L.feat_out, static_cast<size_t>(E) * kLhFrames * kLhFeat * 4));
  CK(cudaMemcpyAsync(L.samples.p, samples, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(L.logits.p, logits, static_cast<size_t>(E) * n_labels * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(L.normed.p, hidden, static_cast<size_t>(E) * kLhQwen * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(L.plan.p, plan.data(), plan.size(), cudaMemcpyHostToDevice, s));
  const LhClip* clips_d = L.plan.as<LhClip>();
  const int* ep_clip_d = reinterpret_cast<const int*>(L.plan.as<uint8_t>() + pad16<LhClip>(1));
  CK(cudaEventRecord(ctx->ev[0], s));
  TRY(run_local_head(ctx, E, 1, clips_d, ep_clip_d, E, L.samples.as<float>(), L.logits.as<float>(),
                     n_labels, L.normed.as<float>(), L.iv.as<double>(),
                     features ? L.feat_out.as<float>() : nullptr));
  CK(cudaEventRecord(ctx->ev[1], s));
  CK(cudaMemcpyAsync(intervals, L.iv.p, static_cast<size_t>(E) * 8, cudaMemcpyDeviceToHost, s));
  if (fixed_ms) CK(cudaMemcpyAsync(fixed_ms, L.fixed.p, static_cast<size_t>(E) * 8, cudaMemcpyDeviceToHost, s));
  if (offsets_ms) CK(cudaMemcpyAsync(offsets_ms, L.off.p, static_cast<size_t>(E) * 4, cudaMemcpyDeviceToHost, s));
  if (features)
    CK(cudaMemcpyAsync(features, L.feat_out.p, static_cast<size_t>(E) * kLhFrames * kLhFeat * 4,
                       cudaMemcpyDeviceToHost, s));
  TRY(wait_stream(ctx));
  ctx->timings.local_ms = elapsed(ctx, 0, 1);
  ctx->timings.gpu_launches = ctx->launches;
  return check_status(ctx);
}

int qa_batch_stage(qa_ctx* ctx, const qa_clip* clips, int n, const qa_result* results) {
  TRY(need_loaded(ctx));
  const qa_cfg& c = ctx->cfg;
  if (!clips || !results || n <= 0) return fail(ctx, QA_ERR_ARG, "empty batch");
  Staged* slot = nullptr;
  for (auto& sl : ctx->slots) {
    if (!sl) {
      sl.reset(new Staged());
      for (auto& e : sl->ev) CK(cudaEventCreate(&e));
    }
    if (sl->state == Staged::kFree) {
      slot = sl.get();
      break;
    }
  }
  if (!slot)
    return fail(ctx, QA_ERR_STATE, "two batches are already staged or running; fetch one first");
  Staged& S = *slot;
  const int cs = 2 * c.n_window;
  Plan& P = S.P;
  P = Plan();
  P.n = n;
  std::vector<int> frames(n);
  std::vector<uint32_t> ids;
  long long total_samples = 0;
  S.want_logits = S.want_normed = S.want_intervals = false;
  S.n_ts.assign(n, 0);
  // ---- validate and plan (host)
  for (int i = 0; i < n; ++i) {
    const qa_clip& cl = clips[i];
    if (!cl.samples || !cl.input_ids || cl.n_samples <= 0 || cl.seq_len <= 0)
      return fail(ctx, QA_ERR_ARG, "clip %d: empty audio or input", i);
    if (cl.seq_len > c.max_seq)
      return fail(ctx, QA_ERR_CAP, "clip %d: prefill needs %d positions, max_seq is %d", i, cl.seq_len, c.max_seq);
    frames[i] = static_cast<int>(cl.n_samples / 160);
    const int na = static_cast<int>(audio_token_count(frames[i], c.n_window));
    if (na <= 0) return fail(ctx, QA_ERR_SHAPE, "clip %d: audio produced 0 tokens (%d mel frames)", i, frames[i]);
    if (na > 16384) return fail(ctx, QA_ERR_CAP, "clip %d: %d audio tokens exceed 16384", i, na);
    int pads = 0, ts = 0;
    for (int p = 0; p < cl.seq_len; ++p) {
      pads += static_cast<int>(cl.input_ids[p]) == c.audio_token_id;
      ts += static_cast<int>(cl.input_ids[p]) == c.timestamp_token_id;
    }
    if (pads != na)
      return fail(ctx, QA_ERR_SHAPE, "clip %d: %d audio tokens in the input, the audio gives %d", i, pads, na);
    if (ts != results[i].n_ts)
      return fail(ctx, QA_ERR_SHAPE, "clip %d: %d timestamp tokens, result holds %d", i, ts, results[i].n_ts);
    S.n_ts[i] = ts;
    S.want_logits |= results[i].logits != nullptr;
    S.want_normed |= results[i].normed != nullptr;
    if (results[i].intervals) {
      if (!ctx->lh || !ctx->lh_on)
        return fail(ctx, QA_ERR_STATE, "clip %d asks for Local Head intervals, but it is %s", i,
                    ctx->lh ? "disabled" : "not loaded");
      if (ts % 2) return fail(ctx, QA_ERR_SHAPE, "clip %d: %d timestamp tokens do not pair into words", i, ts);
      if (c.hidden_size != kLhQwen)
        return fail(ctx, QA_ERR_SHAPE, "hidden size %d != local head context input %d", c.hidden_size, kLhQwen);
      if (static_cast<size_t>(ts) * 20 > 200 * 1024)
        return fail(ctx, QA_ERR_CAP, "clip %d: %d timestamp slots exceed the repair capacity", i, ts);
      S.want_intervals = true;
    }
    P.mel.push_back({total_samples, static_cast<int>(cl.n_samples), P.total_frames, frames[i], P.total_chunks});
    const int nch = (frames[i] + cs - 1) / cs;
    for (int k = 0; k < nch; ++k) P.chunk_clip.push_back(i);
    P.total_frames += frames[i];
    P.total_chunks += nch;
    P.max_frames = std::max(P.max_frames, frames[i]);
    total_samples += cl.n_samples;
    P.tok0.push_back(P.T_d);
    P.seq.push_back(cl.seq_len);
    P.T_d += cl.seq_len;
  }
  plan_audio(P, c, frames);
  P.p2_map.assign(P.T_a, 0);
  P.ts_off.assign(n + 1, 0);
  ids.reserve(P.T_d);
  for (int i = 0; i < n; ++i) {
    int k = 0;
    for (int p = 0; p < clips[i].seq_len; ++p) {
      const uint32_t id = clips[i].input_ids[p];
      ids.push_back(id);
      if (static_cast<int>(id) == c.audio_token_id) P.p2_map[P.atok0[i] + k++] = P.tok0[i] + p;
      if (static_cast<int>(id) == c.timestamp_token_id) P.ts_rows.push_back(P.tok0[i] + p);
    }
    P.ts_off[i + 1] = static_cast<int>(P.ts_rows.size());
  }
  plan_decoder(P);
  S.R = static_cast<int>(P.ts_rows.size());
  S.lh_clips.clear();
  S.lh_ep_clip.clear();
  S.lh_max_slots = 0;
  if (S.want_intervals) {
    for (int i = 0; i < n; ++i) {
      // the Local Head runs over the whole batch: every clip's slots pair into words
      if (S.n_ts[i] % 2)
        return fail(ctx, QA_ERR_SHAPE, "clip %d: %d timestamp tokens do not pair into words", i, S.n_ts[i]);
      S.lh_clips.push_back({P.mel[i].sample_off, P.mel[i].n_samples, P.ts_off[i], S.n_ts[i] / 2,
                            lh_valid_classes(P.mel[i].n_samples, c.num_labels)});
      S.lh_ep_clip.insert(S.lh_ep_clip.end(), S.n_ts[i], i);
      S.lh_max_slots = std::max(S.lh_max_slots, S.n_ts[i]);
    }
  }
  // ---- inputs to the device (sample staging is pinned; one copy each)
  // The other slot's batch may still be running: this batch's pinned and
  // device input buffers are its own (their previous batch has been fetched),
  // and the uploads go on the copy stream, overlapping that batch's kernels.
  TRY(ensure(ctx, S.samples, total_samples * 4));
  TRY(ensure_pin(ctx, S.pin_samples, total_samples * 4));
  float* st = static_cast<float*>(S.pin_samples.p);
  // clips spread over the host cores: one pass, pageable -> pinned
  {
    std::atomic<int> next{0};
    auto worker = [&] {
      for (int i = next++; i < n; i = next++)
        std::memcpy(st + P.mel[i].sample_off, clips[i].samples, clips[i].n_samples * 4);
    };
    const int nt = std::max(1, std::min<int>(n, std::min<int>(8, std::thread::hardware_concurrency())));
    std::vector<std::thread> th;
    for (int k = 1; k < nt; ++k) th.emplace_back(worker);
    worker();
    for (auto& x : th) x.join();
  }
  cudaStream_t cp = ctx->copy_stream;
  CK(cudaEventRecord(S.ev[0], cp));
  CK(cudaMemcpyAsync(S.samples.p, st, total_samples * 4, cudaMemcpyHostToDevice, cp));
  TRY(upload_plan(ctx, P, ids, S.D, S.pin_plan, S.plan, cp));
  size_t lh_bytes = 0;
  if (S.want_intervals) {  // the Local Head's clip table and endpoint -> clip map
    const size_t a = pad16<LhClip>(S.lh_clips.size());
    lh_bytes = a + S.lh_ep_clip.size() * 4;
    TRY(ensure_pin(ctx, S.pin_lh, lh_bytes));
    TRY(ensure(ctx, S.lh_plan, lh_bytes));
    uint8_t* pl = static_cast<uint8_t*>(S.pin_lh.p);
    std::memcpy(pl, S.lh_clips.data(), S.lh_clips.size() * sizeof(LhClip));
    std::memcpy(pl + a, S.lh_ep_clip.data(), S.lh_ep_clip.size() * 4);
    CK(cudaMemcpyAsync(S.lh_plan.p, pl, lh_bytes, cudaMemcpyHostToDevice, cp));
  }
  CK(cudaEventRecord(S.ev[1], cp));
  S.h2d_bytes = total_samples * 4 + static_cast<long long>(ids.size()) * 4 +
                 static_cast<long long>(P.mel.size() * sizeof(MelClip) + P.chunk_clip.size() * 4 +
                                        P.co_map.size() * 4 + P.windows.size() * 8 +
                                        P.p2_map.size() * 4 + P.clip_of.size() * 8 +
                                        P.block_tab.size() * 4 + P.tiles.size() * sizeof(AttnTile) +
                                        P.ts_rows.size() * 4) +
                 static_cast<long long>(lh_bytes);
  // workspaces sized here so that qa_batch_run allocates nothing
  const int H = c.hidden_size;
  TRY(ensure(ctx, ctx->mel_scratch, static_cast<size_t>(P.total_frames) * 128 * 4));
  TRY(ensure(ctx, ctx->mel_chunked, static_cast<size_t>(P.total_chunks) * 128 * cs * 4));
  TRY(ensure(ctx, ctx->mel_frames, static_cast<size_t>(P.total_frames) * kMelDftK * 2));
  TRY(ensure(ctx, ctx->mel_spec, static_cast<size_t>(P.total_frames) * kMelDftRows * 4));
  TRY(ensure(ctx, ctx->maxkey, static_cast<size_t>(n) * 4));
  TRY(ensure(ctx, ctx->hid, static_cast<size_t>(P.T_d) * H * 2));
  {  // conv3's output for every chunk of the pass (the tower's conv_out input)
    const int ds = c.downsample_hidden;
    const int h3 = ((c.num_mel_bins - 1) / 2 / 2) / 2 + 1, w3 = ((cs - 1) / 2 / 2) / 2 + 1;
    TRY(ensure(ctx, ctx->act3, static_cast<size_t>(P.total_chunks) * h3 * w3 * ds * 2));
  }
  S.seq = ++ctx->batch_seq;
  S.state = Staged::kStaged;
  return QA_OK;
}

int qa_batch_run(qa_ctx* ctx) {
  if (!ctx) return QA_ERR_ARG;
  // the oldest batch not yet run, else the most recently run one again
  Staged* slot = ctx->loaded ? oldest(ctx, Staged::kStaged) : nullptr;
  if (!slot && ctx->loaded)
    for (auto& sl : ctx->slots)
      if (sl && sl->state == Staged::kRunning && (!slot || sl->seq > slot->seq)) slot = sl.get();
  if (!slot) return fail(ctx, QA_ERR_STATE, "qa_batch_run needs a staged batch (qa_batch_stage)");
  CK(cudaSetDevice(ctx->device));
  ctx->launches = 0;
  Staged& S = *slot;
  const Plan& P = S.P;
  const PlanDev& D = S.D;
  const qa_cfg& c = ctx->cfg;
  cudaStream_t s = ctx->stream;
  const int cs = 2 * c.n_window, n = P.n, H = c.hidden_size;
  CK(cudaStreamWaitEvent(s, S.ev[1], 0));  // this batch's uploads
  CK(cudaEventRecord(S.ev[2], s));
  TRY(reset_flags(ctx));
  // (a) mel
  CK(cudaMemsetAsync(ctx->maxkey.p, 0, static_cast<size_t>(n) * 4, s));
  const Weights& W = ctx->w;
  MelBank bank{W.fb_start, W.fb_len, W.fb_woff, W.fb_w};
  KL("mel", 2.0 * P.total_frames * kMelDftRows * kMelDftK,
     4.0 * P.mel.back().sample_off + 4.0 * P.mel.back().n_samples + 512.0 * P.total_frames,
     mel_logpower_tc(S.samples.as<float>(), D.mel, n, P.max_frames, P.total_frames, W.mel_dft,
                     bank, 1.0f / std::log(10.0f), ctx->mel_frames.p, ctx->mel_spec.as<float>(),
                     ctx->mel_scratch.as<float>(), ctx->maxkey.as<unsigned>(),
                     ctx->status.as<unsigned>(), s));
  ctx->launches += 2;  // mel_logpower_tc is three launches (rows, GEMM, power)
  KL("mel_finalize", 0, 512.0 * P.total_frames + 512.0 * P.total_chunks * cs,
     mel_finalize_chunked(ctx->mel_scratch.as<float>(), D.mel, D.chunk_clip, P.total_chunks, cs,
                          ctx->maxkey.as<unsigned>(), ctx->mel_chunked.as<float>(), s));
  CK(cudaEventRecord(S.ev[3], s));
  // (b) audio tower, projected rows scattered straight into the decoder input
  TRY(run_encoder(ctx, P, D, ctx->hid.p, D.p2_map));
  CK(cudaEventRecord(S.ev[4], s));
  // embedding gather for the text rows
  KL("embed", 0, 4.0 * (P.T_d - P.T_a) * H,
     embed_gather(D.ids, P.T_d, W.embed, c.vocab_size, H, c.audio_token_id, ctx->hid.p,
                  ctx->badflag.as<int>(), s));
  CK(cudaEventRecord(S.ev[5], s));
  // (c)(d)(e) decoder prefill
  TRY(run_decoder(ctx, P, D));
  CK(cudaEventRecord(S.ev[6], s));
  // (f) head
  TRY(run_head(ctx, ctx->hid.p, ctx->bf16 ? 1 : 0, P.T_d, D.ts_rows, S.R,
               S.want_logits || S.want_intervals, S.want_normed || S.want_intervals));
  CK(cudaEventRecord(S.ev[7], s));
  // the Local Head over every word of the batch (logits and unfolded rows
  // stay on the device)
  const size_t iv_bytes = S.want_intervals ? static_cast<size_t>(S.R) * 8 : 0;
  if (S.want_intervals && S.R > 0) {
    LocalHeadDev& L = *ctx->lh;
    TRY(ensure(ctx, L.iv, iv_bytes));
    const LhClip* clips_d = S.lh_plan.as<LhClip>();
    const int* ep_clip_d = reinterpret_cast<const int*>(
        S.lh_plan.as<uint8_t>() + pad16<LhClip>(S.lh_clips.size()));
    TRY(run_local_head(ctx, S.R, n, clips_d, ep_clip_d, S.lh_max_slots, S.samples.as<float>(),
                       ctx->head_logits.as<float>(), c.num_labels, ctx->head_normed.as<float>(),
                       L.iv.as<double>(), nullptr));
  }
  CK(cudaEventRecord(S.ev[10], s));
  // results and the two status words to this batch's pinned buffer, queued
  // before any later batch can overwrite them
  const size_t raw_bytes = static_cast<size_t>(S.R) * 8;
  const size_t lg_bytes = S.want_logits ? static_cast<size_t>(S.R) * c.num_labels * 4 : 0;
  const size_t nm_bytes = S.want_normed ? static_cast<size_t>(S.R) * H * 4 : 0;
  TRY(ensure_pin(ctx, S.pin_res, 16 + raw_bytes + lg_bytes + nm_bytes + iv_bytes));
  uint8_t* pr = static_cast<uint8_t*>(S.pin_res.p);
  CK(cudaEventRecord(S.ev[8], s));
  CK(cudaMemcpyAsync(pr, ctx->status.p, 4, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(pr + 4, ctx->badflag.p, 4, cudaMemcpyDeviceToHost, s));
  if (raw_bytes) CK(cudaMemcpyAsync(pr + 16, ctx->head_raw.p, raw_bytes, cudaMemcpyDeviceToHost, s));
  if (lg_bytes)
    CK(cudaMemcpyAsync(pr + 16 + raw_bytes, ctx->head_logits.p, lg_bytes, cudaMemcpyDeviceToHost, s));
  if (nm_bytes)
    CK(cudaMemcpyAsync(pr + 16 + raw_bytes + lg_bytes, ctx->head_normed.p, nm_bytes,
                       cudaMemcpyDeviceToHost, s));
  if (iv_bytes && S.R > 0)
    CK(cudaMemcpyAsync(pr + 16 + raw_bytes + lg_bytes + nm_bytes, ctx->lh->iv.p, iv_bytes,
                       cudaMemcpyDeviceToHost, s));
  CK(cudaEventRecord(S.ev[9], s));
  S.launches = ctx->launches;
  S.state = Staged::kRunning;
  ctx->timings.gpu_launches = ctx->launches;
  return QA_OK;
}

int qa_batch_fetch(qa_ctx* ctx, qa_result* results) {
  if (!ctx || !results) return QA_ERR_ARG;
  Staged* slot = oldest(ctx, Staged::kRunning);
  if (!slot) {
    if (oldest(ctx, Staged::kStaged)) return fail(ctx, QA_ERR_STATE, "the staged batch has not been run");
    return fail(ctx, QA_ERR_STATE, "no staged batch");
  }
  CK(cudaSetDevice(ctx->device));
  Staged& S = *slot;
  const Plan& P = S.P;
  const qa_cfg& c = ctx->cfg;
  const int H = c.hidden_size;
  for (int i = 0; i < P.n; ++i)
    if (results[i].n_ts != S.n_ts[i] || (S.n_ts[i] > 0 && !results[i].raw_ms))
      return fail(ctx, QA_ERR_SHAPE, "clip %d: result holds %d timestamps, the batch has %d", i,
                  results[i].n_ts, S.n_ts[i]);
  // the batch is consumed by this call whatever happens next
  S.state = Staged::kFree;
  TRY(wait_event(ctx, S.ev[9]));
  if (!ctx->prof_recs.empty() && !oldest(ctx, Staged::kRunning)) prof_resolve(ctx);
  const uint8_t* pr = static_cast<const uint8_t*>(S.pin_res.p);
  unsigned st = 0;
  int bad = 0;
  std::memcpy(&st, pr, 4);
  std::memcpy(&bad, pr + 4, 4);
  if (st & kStatusTimeout)
    return fail(ctx, QA_ERR_TIMEOUT, "a tensor-core pipeline wait ran out (status %u)", st);
  if (bad) return flag_error(ctx, bad);
  const size_t raw_bytes = static_cast<size_t>(S.R) * 8;
  const size_t lg_bytes = S.want_logits ? static_cast<size_t>(S.R) * c.num_labels * 4 : 0;
  const size_t nm_bytes = S.want_normed ? static_cast<size_t>(S.R) * H * 4 : 0;
  const size_t iv_bytes = S.want_intervals ? static_cast<size_t>(S.R) * 8 : 0;
  const int64_t* raw = reinterpret_cast<const int64_t*>(pr + 16);
  const float* lg = reinterpret_cast<const float*>(pr + 16 + raw_bytes);
  const float* nm = reinterpret_cast<const float*>(pr + 16 + raw_bytes + lg_bytes);
  const double* iv = reinterpret_cast<const double*>(pr + 16 + raw_bytes + lg_bytes + nm_bytes);
  for (int i = 0; i < P.n; ++i) {
    const int o = P.ts_off[i], k = P.ts_off[i + 1] - o;
    if (k) std::memcpy(results[i].raw_ms, raw + o, static_cast<size_t>(k) * 8);
    if (results[i].intervals && iv_bytes && k)
      std::memcpy(results[i].intervals, iv + o, static_cast<size_t>(k) * 8);
    if (results[i].logits && lg_bytes)
      std::memcpy(results[i].logits, lg + static_cast<size_t>(o) * c.num_labels, static_cast<size_t>(k) * c.num_labels * 4);
    if (results[i].normed && nm_bytes)
      std::memcpy(results[i].normed, nm + static_cast<size_t>(o) * H, static_cast<size_t>(k) * H * 4);
  }
  qa_timings& t = ctx->timings;
  t.h2d_ms = elapsed(S, 0, 1);
  t.mel_ms = elapsed(S, 2, 3);
  t.enc_ms = elapsed(S, 3, 4);
  t.gather_ms = elapsed(S, 4, 5);
  t.prefill_ms = elapsed(S, 5, 6);
  t.head_ms = elapsed(S, 6, 7);
  t.local_ms = S.want_intervals ? elapsed(S, 7, 10) : 0.0;
  t.d2h_ms = elapsed(S, 8, 9);
  t.total_ms = t.h2d_ms + elapsed(S, 2, 10) + t.d2h_ms;
  t.h2d_bytes = S.h2d_bytes;
  t.d2h_bytes = static_cast<long long>(8 + raw_bytes + lg_bytes + nm_bytes + iv_bytes);
  t.gpu_launches = S.launches;
  return QA_OK;
}

int qa_align_batch(qa_ctx* ctx, const qa_clip* clips, int n, qa_result* results) {
  TRY(qa_batch_stage(ctx, clips, n, results));
  TRY(qa_batch_run(ctx));
  return qa_batch_fetch(ctx, results);
}

int qa_set_stream(qa_ctx* ctx, void* stream) {
  if (!ctx) return QA_ERR_ARG;
  ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
  return QA_OK;
}

int qa_set_profile(qa_ctx* ctx, int on) {
  if (!ctx) return QA_ERR_ARG;
  ctx->profile = on != 0;
  ctx->prof_recs.clear();
  ctx->prof_next = 0;
  ctx->prof_names.clear();
  ctx->prof_stats.clear();
  return QA_OK;
}

int qa_get_profile(qa_ctx* ctx, qa_kernel_stat* stats, int max, int* n) {
  if (!ctx || !n) return QA_ERR_ARG;
  CK(cudaSetDevice(ctx->device));
  TRY(wait_stream(ctx));  // resolves pending records
  const int k = static_cast<int>(ctx->prof_stats.size());
  *n = k;
  for (int i = 0; i < k && i < max && stats; ++i) stats[i] = ctx->prof_stats[i];
  return QA_OK;
}

}  // extern "C"
