"""An independent float64 forward (PyTorch on the CPU) against the oracle's
model: it catches restatement mistakes in oracle/encoder.cpp, decoder.cpp and
head.cpp that the known-answer tests cannot see.  The forward here is written
from the reference's CPU path directly:

* audio tower (src/audio_encoder.rs:102-832): 100-frame chunks (the tail
  zero-padded, feo(tail) tokens kept), three conv2d(3x3, stride 2, pad 1) +
  bias + erf-GELU, [b, c, f, t] -> [b, t, c*f], conv_out, sinusoidal PE (sin
  in the first half, log step ln(1e4)/(d/2 - 1)), pre-LN layers (eps 1e-5)
  with attention inside windows of 104 tokens, ln_post, proj1, GELU, proj2;
* decoder (src/cpu_decoder.rs:283-512): RMSNorm (eps 1e-6), q/k/v, per-head
  RMSNorm with the q_norm / k_norm gains, rotate-half RoPE (theta 1e6) at the
  token's position, causal GQA attention, o_proj + residual, SwiGLU MLP;
* head (src/align_inference.rs:766-783): the folded final norm and the
  score projection.

No f16 rounding here, so the oracle's decoder (which rounds where the
reference does) is compared within the 2e-2 max-abs relative bound; the f32
tower and head are compared within 1e-4."""
import math
import os
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT, pkg

D = torch.float64


def _w(weights, name):
    v = weights[name]
    if isinstance(v, tuple):
        return torch.tensor(np.asarray(v[1], np.float64), dtype=D)
    bits = np.asarray(v, np.uint16).astype(np.uint32) << 16
    return torch.tensor(bits.view(np.float32).astype(np.float64), dtype=D)


def _gelu(x):
    return 0.5 * x * (1.0 + torch.erf(x / math.sqrt(2.0)))


def _feo(n):
    for _ in range(3):
        n = (n - 1) // 2 + 1
    return n


def tower_f64(W, cfg, mel):
    A = "model.audio_tower."
    n_mels, frames = mel.shape
    cs = 2 * cfg.n_window
    n_chunks = -(-frames // cs)
    x = torch.zeros(n_chunks, 1, n_mels, cs, dtype=D)
    tokens = []
    for c in range(n_chunks):
        seg = mel[:, c * cs:(c + 1) * cs]
        x[c, 0, :, :seg.shape[1]] = torch.tensor(seg, dtype=D)
        tokens.append(_feo(seg.shape[1]))
    for k in (1, 2, 3):
        x = _gelu(torch.nn.functional.conv2d(x, _w(W, f"{A}conv2d{k}.weight"),
                                             _w(W, f"{A}conv2d{k}.bias"), stride=2, padding=1))
    b, c, f, t = x.shape
    x = x.permute(0, 3, 1, 2).reshape(b, t, c * f) @ _w(W, f"{A}conv_out.weight").T
    dm = cfg.d_model
    half = dm // 2
    lt = math.log(10000.0) / (half - 1)
    pos = torch.arange(t, dtype=D)[:, None] * torch.exp(-lt * torch.arange(half, dtype=D))[None]
    x = x + torch.cat([torch.sin(pos), torch.cos(pos)], dim=1)[None]
    h = torch.cat([x[i, :tokens[i]] for i in range(b)], dim=0)
    ws = _feo(cs) * (cfg.n_window_infer // cs)
    nh, hd = cfg.encoder_heads, dm // cfg.encoder_heads

    def ln(v, name):
        return torch.nn.functional.layer_norm(v, (dm,), _w(W, name + ".weight"), _w(W, name + ".bias"),
                                              eps=1e-5)

    def lin(v, name, bias=True):
        y = v @ _w(W, name + ".weight").T
        return y + _w(W, name + ".bias") if bias and (name + ".bias") in W else y

    for li in range(cfg.encoder_layers):
        P = f"{A}layers.{li}."
        r = h
        y = ln(h, P + "self_attn_layer_norm")
        q, k, v = (lin(y, P + f"self_attn.{n}_proj") for n in "qkv")
        out = torch.zeros_like(q)
        for st in range(0, len(h), ws):
            e = min(len(h), st + ws)
            qh = q[st:e].reshape(e - st, nh, hd).transpose(0, 1)
            kh = k[st:e].reshape(e - st, nh, hd).transpose(0, 1)
            vh = v[st:e].reshape(e - st, nh, hd).transpose(0, 1)
            p = torch.softmax(qh @ kh.transpose(1, 2) / math.sqrt(hd), dim=-1)
            out[st:e] = (p @ vh).transpose(0, 1).reshape(e - st, dm)
        h = r + lin(out, P + "self_attn.out_proj")
        r = h
        y = _gelu(lin(ln(h, P + "final_layer_norm"), P + "fc1"))
        h = r + lin(y, P + "fc2")
    h = ln(h, A + "ln_post")
    h = _gelu(lin(h, "model.multi_modal_projector.linear_1"))
    return lin(h, "model.multi_modal_projector.linear_2")


def decoder_f64(W, cfg, emb):
    T = "model.language_model."
    L, H = emb.shape
    nq, nkv, hd, eps = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.rms_norm_eps
    half = hd // 2
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(half, dtype=D) * 2.0 / hd))
    ang = torch.arange(L, dtype=D)[:, None] * inv[None]
    cos, sin = torch.cos(ang).repeat(1, 2), torch.sin(ang).repeat(1, 2)

    def rms(v, w):
        return v / torch.sqrt((v * v).mean(-1, keepdim=True) + eps) * w

    def rope(v):  # [heads, L, hd]
        rot = torch.cat([-v[..., half:], v[..., :half]], dim=-1)
        return v * cos[None] + rot * sin[None]

    x = emb.clone()
    mask = torch.ones(L, L, dtype=torch.bool).tril()
    for li in range(cfg.num_layers):
        P = f"{T}layers.{li}."
        y = rms(x, _w(W, P + "input_layernorm.weight"))
        q = (y @ _w(W, P + "self_attn.q_proj.weight").T).reshape(L, nq, hd).transpose(0, 1)
        k = (y @ _w(W, P + "self_attn.k_proj.weight").T).reshape(L, nkv, hd).transpose(0, 1)
        v = (y @ _w(W, P + "self_attn.v_proj.weight").T).reshape(L, nkv, hd).transpose(0, 1)
        q = rope(rms(q, _w(W, P + "self_attn.q_norm.weight")))
        k = rope(rms(k, _w(W, P + "self_attn.k_norm.weight")))
        rep = nq // nkv
        k, v = k.repeat_interleave(rep, 0), v.repeat_interleave(rep, 0)
        s = (q @ k.transpose(1, 2)) / math.sqrt(hd)
        s = s.masked_fill(~mask[None], float("-inf"))
        a = (torch.softmax(s, -1) @ v).transpose(0, 1).reshape(L, nq * hd)
        x = x + a @ _w(W, P + "self_attn.o_proj.weight").T
        y = rms(x, _w(W, P + "post_attention_layernorm.weight"))
        g = y @ _w(W, P + "mlp.gate_proj.weight").T
        u = y @ _w(W, P + "mlp.up_proj.weight").T
        x = x + (g * torch.sigmoid(g) * u) @ _w(W, P + "mlp.down_proj.weight").T
    return x


def head_f64(W, cfg, hidden, rows):
    h = hidden[rows] * _w(W, "model.language_model.norm.weight")
    h = h / torch.sqrt((h * h).mean(-1, keepdim=True) + cfg.rms_norm_eps)
    return h @ _w(W, "score.weight").T


@pytest.fixture(scope="module")
def case():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    qa = pkg()
    orc.build()
    cfg = qa.synth.ModelConfig(encoder_layers=2, num_layers=2)
    W = qa.synth.random_weights(cfg, 3)
    om = orc.Model(W, cfg)
    samples = qa.synth.synth_audio(9.37, 41)  # 9 full chunks + a 37-frame tail: 2 windows
    rng = np.random.default_rng(41)
    b = qa.synth.InputBuilder(None, n_window=cfg.n_window)
    inp = b.build(qa.synth.split_words(" ".join(qa.synth.english_words(6, rng)), "English"),
                  qa.synth.valid_mel_frames(len(samples)))
    return orc, qa, cfg, W, om, samples, inp


def _rel(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def test_tower_matches_float64(case):
    orc, qa, cfg, W, om, samples, inp = case
    mel = orc.mel(samples)
    got = om.audio_embeds(mel)
    ref = tower_f64(W, cfg, mel).numpy()
    assert got.shape == ref.shape == (inp.n_audio_tokens, cfg.output_dim)
    assert _rel(got, ref) <= 1e-4


def test_decoder_and_head_match_float64(case):
    orc, qa, cfg, W, om, samples, inp = case
    audio16 = orc.f32_to_f16_array(om.audio_embeds(orc.mel(samples)))
    emb = om.gather(inp.input_ids, audio16)
    got = orc.f16_bits_to_f32(om.text_hidden(emb))
    emb64 = torch.tensor(orc.f16_bits_to_f32(emb), dtype=D)
    ref = decoder_f64(W, cfg, emb64)
    assert _rel(got, ref.numpy()) <= 2e-2
    rows = list(inp.timestamp_positions)
    _, logits, _, _ = om.head(got, rows)
    ref_logits = head_f64(W, cfg, torch.tensor(got, dtype=D), rows).numpy()
    assert _rel(logits, ref_logits) <= 1e-4
