// TEST INFRASTRUCTURE (parity oracle) — weight loading for the CPU restatement.
#include "model.h"

#include <cstdio>
#include <stdexcept>

namespace {

struct View {
  int dtype;
  std::vector<int64_t> shape;
  const void* data;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

// src/weights.rs:231-265: `-hf` names to the reference's internal names.
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

float elem_f32(const View& v, int64_t i) {
  switch (v.dtype) {
    case QA_DTYPE_F32: return static_cast<const float*>(v.data)[i];
    case QA_DTYPE_F16: return orc::f16_to_f32(static_cast<const uint16_t*>(v.data)[i]);
    case QA_DTYPE_BF16: return orc::bf16_to_f32(static_cast<const uint16_t*>(v.data)[i]);
  }
  return 0.0f;
}

struct Loader {
  std::map<std::string, View> t;
  const View& get(const std::string& name) const {
    auto it = t.find(name);
    if (it == t.end()) throw std::runtime_error("weight not found: " + name);
    return it->second;
  }
  bool has(const std::string& name) const { return t.count(name) != 0; }
  // RawTensor::to_f32_vec (src/weights.rs:129-151): exact widening.
  std::vector<float> f32(const std::string& name) const {
    const View& v = get(name);
    std::vector<float> o(v.numel());
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < v.numel(); ++i) o[i] = elem_f32(v, i);
    return o;
  }
  // RawTensor::to_f16_vec then widen (src/weights.rs:100-127): the CPU
  // path's f16 weights, held as f32.
  std::vector<float> f16w(const std::string& name) const {
    const View& v = get(name);
    std::vector<float> o(v.numel());
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < v.numel(); ++i) o[i] = orc::r16(elem_f32(v, i));
    return o;
  }
  int64_t dim(const std::string& name, int d) const { return get(name).shape.at(d); }
};

}  // namespace

extern "C" or_model* or_load(const qa_tensor* tensors, int n, const qa_cfg* cfg, char* err,
                             int err_len) {
  try {
    Loader L;
    bool hf = false;
    for (int i = 0; i < n; ++i) {
      std::string nm = tensors[i].name;
      if (nm.rfind("model.audio_tower.", 0) == 0 || nm.rfind("model.language_model.", 0) == 0 ||
          nm.rfind("thinker.lm_head.", 0) == 0)
        hf = true;
    }
    for (int i = 0; i < n; ++i) {
      View v{tensors[i].dtype, {}, tensors[i].data};
      for (int d = 0; d < tensors[i].ndim; ++d) v.shape.push_back(tensors[i].shape[d]);
      std::string nm = tensors[i].name;
      L.t[hf ? remap(nm) : nm] = v;
    }
    auto* m = new or_model();
    m->cfg = *cfg;
    const qa_cfg& c = *cfg;
    const std::string A = "thinker.audio_tower.";
    // conv stem (src/audio_encoder.rs:249-277)
    m->c1w = L.f16w(A + "conv2d1.weight");
    m->c1b = L.f32(A + "conv2d1.bias");
    m->c2w = L.f16w(A + "conv2d2.weight");
    m->c2b = L.f32(A + "conv2d2.bias");
    m->c3w = L.f16w(A + "conv2d3.weight");
    m->c3b = L.f32(A + "conv2d3.bias");
    m->c1_out = static_cast<int>(L.dim(A + "conv2d1.weight", 0));
    m->c2_out = static_cast<int>(L.dim(A + "conv2d2.weight", 0));
    m->c3_out = static_cast<int>(L.dim(A + "conv2d3.weight", 0));
    m->co_w = L.f16w(A + "conv_out.weight");
    m->co_in = static_cast<int>(L.dim(A + "conv_out.weight", 1));
    if (L.has(A + "conv_out.bias")) m->co_b = L.f32(A + "conv_out.bias");
    // sinusoidal PE (src/audio_encoder.rs:263-275)
    {
      const int dm = c.d_model, maxp = c.max_source_positions, half = dm / 2;
      const double lt = std::log(10000.0) / (half - 1.0);
      m->pe.assign(static_cast<size_t>(maxp) * dm, 0.0f);
      for (int p = 0; p < maxp; ++p)
        for (int i = 0; i < half; ++i) {
          const double a = p * std::exp(-i * lt);
          m->pe[static_cast<size_t>(p) * dm + i] = static_cast<float>(std::sin(a));
          m->pe[static_cast<size_t>(p) * dm + half + i] = static_cast<float>(std::cos(a));
        }
    }
    auto bias_or_zero = [&](const std::string& nm, int64_t len) {
      return L.has(nm) ? L.f32(nm) : std::vector<float>(len, 0.0f);
    };
    for (int l = 0; l < c.encoder_layers; ++l) {
      const std::string p = A + "layers." + std::to_string(l) + ".";
      EncLayer e;
      e.ln1_w = L.f32(p + "self_attn_layer_norm.weight");
      e.ln1_b = L.f32(p + "self_attn_layer_norm.bias");
      e.ln2_w = L.f32(p + "final_layer_norm.weight");
      e.ln2_b = L.f32(p + "final_layer_norm.bias");
      e.q_w = L.f16w(p + "self_attn.q_proj.weight");
      e.k_w = L.f16w(p + "self_attn.k_proj.weight");
      e.v_w = L.f16w(p + "self_attn.v_proj.weight");
      e.o_w = L.f16w(p + "self_attn.out_proj.weight");
      e.q_b = bias_or_zero(p + "self_attn.q_proj.bias", c.d_model);
      e.k_b = bias_or_zero(p + "self_attn.k_proj.bias", c.d_model);
      e.v_b = bias_or_zero(p + "self_attn.v_proj.bias", c.d_model);
      e.o_b = bias_or_zero(p + "self_attn.out_proj.bias", c.d_model);
      e.fc1_w = L.f16w(p + "fc1.weight");
      e.fc1_b = bias_or_zero(p + "fc1.bias", c.encoder_ffn_dim);
      e.fc2_w = L.f16w(p + "fc2.weight");
      e.fc2_b = bias_or_zero(p + "fc2.bias", c.d_model);
      m->enc.push_back(std::move(e));
    }
    m->lnp_w = L.f32(A + "ln_post.weight");
    m->lnp_b = L.f32(A + "ln_post.bias");
    m->p1_w = L.f16w(A + "proj1.weight");
    m->p1_b = bias_or_zero(A + "proj1.bias", c.d_model);
    m->p2_w = L.f16w(A + "proj2.weight");
    m->p2_b = bias_or_zero(A + "proj2.bias", c.output_dim);

    // text decoder (src/cpu_decoder.rs:163-187): norms through f16, matrices f16
    const std::string T = "thinker.model.";
    for (int l = 0; l < c.num_layers; ++l) {
      const std::string p = T + "layers." + std::to_string(l) + ".";
      DecLayer d;
      d.iln = L.f16w(p + "input_layernorm.weight");
      d.pln = L.f16w(p + "post_attention_layernorm.weight");
      d.qn = L.f16w(p + "self_attn.q_norm.weight");
      d.kn = L.f16w(p + "self_attn.k_norm.weight");
      d.q = L.f16w(p + "self_attn.q_proj.weight");
      d.k = L.f16w(p + "self_attn.k_proj.weight");
      d.v = L.f16w(p + "self_attn.v_proj.weight");
      d.o = L.f16w(p + "self_attn.o_proj.weight");
      d.gate = L.f16w(p + "mlp.gate_proj.weight");
      d.up = L.f16w(p + "mlp.up_proj.weight");
      d.down = L.f16w(p + "mlp.down_proj.weight");
      m->dec.push_back(std::move(d));
    }
    {
      const View& e = L.get(T + "embed_tokens.weight");
      m->embed.resize(e.numel());
#pragma omp parallel for schedule(static)
      for (int64_t i = 0; i < e.numel(); ++i) m->embed[i] = orc::f32_to_f16(elem_f32(e, i));
    }
    m->final_norm = L.f32(T + "norm.weight");
    m->score = L.f32("score.weight");
    // RoPE tables (src/align_inference.rs:320-328 + 394-396): f64 -> f32 -> f16
    {
      const int hd = c.head_dim;
      m->cos.resize(static_cast<size_t>(c.max_seq) * hd);
      m->sin.resize(static_cast<size_t>(c.max_seq) * hd);
      or_rope_tables(c.max_seq, hd, 1000000.0, m->cos.data(), m->sin.data());
      for (auto& v : m->cos) v = orc::r16(v);
      for (auto& v : m->sin) v = orc::r16(v);
    }
    return m;
  } catch (const std::exception& e) {
    if (err && err_len > 0) std::snprintf(err, err_len, "%s", e.what());
    return nullptr;
  }
}

extern "C" void or_free(or_model* m) { delete m; }

// src/mrope.rs:55-89 with section [head_dim/2, 0, 0], blocked: every
// frequency reads the position axis, i.e. plain RoPE; halves duplicate.
extern "C" void or_rope_tables(int positions, int head_dim, double theta, float* cos_out,
                               float* sin_out) {
  const int half = head_dim / 2;
  std::vector<double> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = 1.0 / std::pow(theta, 2.0 * i / head_dim);
  for (int t = 0; t < positions; ++t)
    for (int j = 0; j < half; ++j) {
      const double a = static_cast<double>(t) * inv[j];
      const float cv = static_cast<float>(std::cos(a)), sv = static_cast<float>(std::sin(a));
      cos_out[static_cast<size_t>(t) * head_dim + j] = cv;
      sin_out[static_cast<size_t>(t) * head_dim + j] = sv;
      cos_out[static_cast<size_t>(t) * head_dim + j + half] = cv;
      sin_out[static_cast<size_t>(t) * head_dim + j + half] = sv;
    }
}
