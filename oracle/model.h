// TEST INFRASTRUCTURE (parity oracle) — the CPU model, restating the weight
// handling of src/cpu_decoder.rs:34-51,163-187 (f16 matrices widened to f32),
// src/audio_encoder.rs:104-192,249-277,454-464 (f16 matrices, f32 biases and
// LayerNorm parameters) and src/align_inference.rs:405-428 (embed table in the
// CPU path's f16, score and final norm widened to f32 exactly).
#pragma once

#include <map>
#include <string>
#include <vector>

#include "common.h"

struct EncLayer {
  std::vector<float> ln1_w, ln1_b, ln2_w, ln2_b;
  std::vector<float> q_w, q_b, k_w, k_b, v_w, v_b, o_w, o_b;  // [dm, dm], bias [dm]
  std::vector<float> fc1_w, fc1_b, fc2_w, fc2_b;
};

struct DecLayer {
  std::vector<float> iln, pln, qn, kn;
  std::vector<float> q, k, v, o, gate, up, down;
};

struct or_model {
  qa_cfg cfg;
  // audio tower
  int c1_out = 0, c2_out = 0, c3_out = 0;
  std::vector<float> c1w, c1b, c2w, c2b, c3w, c3b;  // [c_out, c_in*9]
  std::vector<float> co_w, co_b;                    // conv_out [dm, c*f]
  int co_in = 0;
  std::vector<float> pe;  // [max_pos, dm]
  std::vector<EncLayer> enc;
  std::vector<float> lnp_w, lnp_b, p1_w, p1_b, p2_w, p2_b;
  // text decoder
  std::vector<DecLayer> dec;
  std::vector<uint16_t> embed;  // [vocab, hidden] f16
  std::vector<float> final_norm, score;
  std::vector<float> cos, sin;  // [max_seq, head_dim], f16-rounded
};
