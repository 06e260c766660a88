"""Seeded synthetic assets for the aligner: a random-init checkpoint in the
reference's `-hf` safetensors layout, a tokenizer with the reference's marker
ids, and synthetic audio + transcripts for each benchmark configuration.

No checkpoint, tokenizer or audio fixture of the reference exists in this
environment, so every parity test and benchmark runs on these stand-ins:

* weights: N(0, 0.02) for every matrix, embedding and bias, RMSNorm and
  LayerNorm gains 1, LayerNorm biases 0, stored bf16 (the checkpoint's dtype);
  each tensor has its own generator seeded from (seed, name) so a model with
  fewer layers shares its tensors with the full one;
* audio: 16 kHz Gaussian noise, low-passed (4th-order Butterworth at 3.4 kHz,
  zero phase), shaped by Hann bursts of 150-400 ms separated by 40-200 ms gaps,
  scaled to RMS 0.1;
* transcripts: English pseudo-words of 3-8 lowercase letters, Chinese words of
  one CJK ideograph in U+4E00..U+62FF;
* tokenizer: the markers of src/align_input.rs:33-44 are atomic tokens with
  the checkpoint's ids (151669, 151670, 151676, 151705); a CJK character is one
  token; a Latin word is split into 3-letter pieces, each one token.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from dataclasses import dataclass, field, asdict

import numpy as np

AUDIO_START_ID = 151669
AUDIO_END_ID = 151670
AUDIO_PAD_ID = 151676
TIMESTAMP_ID = 151705
AUDIO_START = "<|audio_start|>"
AUDIO_END = "<|audio_end|>"
AUDIO_PAD = "<|audio_pad|>"
TIMESTAMP = "<timestamp>"
SAMPLE_RATE = 16000
HOP = 160


@dataclass
class ModelConfig:
    """Geometry of the Qwen3-ForcedAligner-0.6B checkpoint (src/config.rs:81-137)."""
    # audio tower
    d_model: int = 896
    encoder_layers: int = 18
    encoder_heads: int = 14
    encoder_ffn_dim: int = 3584
    num_mel_bins: int = 128
    downsample_hidden: int = 480
    max_source_positions: int = 1500
    n_window: int = 50
    n_window_infer: int = 800
    output_dim: int = 1024
    # text decoder
    vocab_size: int = 151936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_layers: int = 28
    num_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    # head
    num_labels: int = 5000
    timestamp_token_id: int = TIMESTAMP_ID
    audio_token_id: int = AUDIO_PAD_ID
    timestamp_segment_time_ms: float = 80.0
    max_seq: int = 8192

    def config_json(self) -> dict:
        """config.json in the `-hf` layout the reference parses (src/config.rs:153-236)."""
        return {
            "audio_config": {
                "d_model": self.d_model, "encoder_layers": self.encoder_layers,
                "encoder_attention_heads": self.encoder_heads,
                "encoder_ffn_dim": self.encoder_ffn_dim, "num_mel_bins": self.num_mel_bins,
                "downsample_hidden_size": self.downsample_hidden,
                "max_source_positions": self.max_source_positions, "n_window": self.n_window,
                "n_window_infer": self.n_window_infer, "output_dim": self.output_dim,
            },
            "text_config": {
                "vocab_size": self.vocab_size, "hidden_size": self.hidden_size,
                "intermediate_size": self.intermediate_size,
                "num_hidden_layers": self.num_layers, "num_attention_heads": self.num_heads,
                "num_key_value_heads": self.num_kv_heads, "head_dim": self.head_dim,
                "rms_norm_eps": self.rms_norm_eps, "rope_theta": self.rope_theta,
            },
            "audio_token_id": self.audio_token_id,
            "audio_start_token_id": AUDIO_START_ID,
            "audio_end_token_id": AUDIO_END_ID,
            "timestamp_token_id": self.timestamp_token_id,
            "timestamp_segment_time": self.timestamp_segment_time_ms,
            "id2label": {str(i): f"LABEL_{i}" for i in range(self.num_labels)},
        }

    @staticmethod
    def from_config_json(d: dict) -> "ModelConfig":
        a = d.get("audio_config") or d["thinker_config"]["audio_config"]
        t = d.get("text_config") or d["thinker_config"]["text_config"]
        c = ModelConfig()
        c.d_model = a.get("d_model", c.d_model)
        c.encoder_layers = a.get("encoder_layers", c.encoder_layers)
        c.encoder_heads = a.get("encoder_attention_heads", c.encoder_heads)
        c.encoder_ffn_dim = a.get("encoder_ffn_dim", c.encoder_ffn_dim)
        c.num_mel_bins = a.get("num_mel_bins", c.num_mel_bins)
        c.downsample_hidden = a.get("downsample_hidden_size", c.downsample_hidden)
        c.max_source_positions = a.get("max_source_positions", c.max_source_positions)
        c.n_window = a.get("n_window", c.n_window)
        c.n_window_infer = a.get("n_window_infer", c.n_window_infer)
        c.output_dim = a.get("output_dim", c.output_dim)
        c.vocab_size = t.get("vocab_size", c.vocab_size)
        c.hidden_size = t.get("hidden_size", c.hidden_size)
        c.intermediate_size = t.get("intermediate_size", c.intermediate_size)
        c.num_layers = t.get("num_hidden_layers", c.num_layers)
        c.num_heads = t.get("num_attention_heads", c.num_heads)
        c.num_kv_heads = t.get("num_key_value_heads", c.num_kv_heads)
        c.head_dim = t.get("head_dim", c.head_dim)
        c.rms_norm_eps = t.get("rms_norm_eps", c.rms_norm_eps)
        rp = t.get("rope_parameters") or {}
        c.rope_theta = rp.get("rope_theta", t.get("rope_theta", c.rope_theta))
        c.audio_token_id = d.get("audio_token_id", c.audio_token_id)
        c.timestamp_token_id = d.get("timestamp_token_id", c.timestamp_token_id)
        c.timestamp_segment_time_ms = d.get("timestamp_segment_time", 80.0)
        c.num_labels = len(d.get("id2label") or {}) or c.num_labels
        return c


# ---------------------------------------------------------------- weights

def _bf16_bits(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bits, round to nearest even (src/shaders.rs:74-80)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _rng(seed: int, name: str) -> np.random.Generator:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return np.random.default_rng(int.from_bytes(h[:8], "little"))


def weight_specs(cfg: ModelConfig) -> list:
    """(name, shape, kind) of every checkpoint tensor, `-hf` names
    (src/weights.rs:231-249).  kind: 'normal' | 'ones' | 'zeros'."""
    s = []
    A = "model.audio_tower."
    ds, dm = cfg.downsample_hidden, cfg.d_model
    f3 = cfg.num_mel_bins
    for _ in range(3):
        f3 = (f3 - 1) // 2 + 1
    s += [(A + "conv2d1.weight", (ds, 1, 3, 3), "normal"), (A + "conv2d1.bias", (ds,), "normal"),
          (A + "conv2d2.weight", (ds, ds, 3, 3), "normal"), (A + "conv2d2.bias", (ds,), "normal"),
          (A + "conv2d3.weight", (ds, ds, 3, 3), "normal"), (A + "conv2d3.bias", (ds,), "normal"),
          (A + "conv_out.weight", (dm, ds * f3), "normal")]
    for i in range(cfg.encoder_layers):
        p = f"{A}layers.{i}."
        for ln in ("self_attn_layer_norm", "final_layer_norm"):
            s += [(p + ln + ".weight", (dm,), "ones"), (p + ln + ".bias", (dm,), "zeros")]
        for pr in ("q_proj", "k_proj", "v_proj", "out_proj"):
            s += [(p + f"self_attn.{pr}.weight", (dm, dm), "normal")]
            if pr != "k_proj":
                s += [(p + f"self_attn.{pr}.bias", (dm,), "normal")]
        s += [(p + "fc1.weight", (cfg.encoder_ffn_dim, dm), "normal"),
              (p + "fc1.bias", (cfg.encoder_ffn_dim,), "normal"),
              (p + "fc2.weight", (dm, cfg.encoder_ffn_dim), "normal"),
              (p + "fc2.bias", (dm,), "normal")]
    s += [(A + "ln_post.weight", (dm,), "ones"), (A + "ln_post.bias", (dm,), "zeros"),
          ("model.multi_modal_projector.linear_1.weight", (dm, dm), "normal"),
          ("model.multi_modal_projector.linear_1.bias", (dm,), "normal"),
          ("model.multi_modal_projector.linear_2.weight", (cfg.output_dim, dm), "normal"),
          ("model.multi_modal_projector.linear_2.bias", (cfg.output_dim,), "normal")]
    T = "model.language_model."
    H, hd = cfg.hidden_size, cfg.head_dim
    s += [(T + "embed_tokens.weight", (cfg.vocab_size, H), "normal")]
    for i in range(cfg.num_layers):
        p = f"{T}layers.{i}."
        s += [(p + "input_layernorm.weight", (H,), "ones"),
              (p + "post_attention_layernorm.weight", (H,), "ones"),
              (p + "self_attn.q_norm.weight", (hd,), "ones"),
              (p + "self_attn.k_norm.weight", (hd,), "ones"),
              (p + "self_attn.q_proj.weight", (cfg.num_heads * hd, H), "normal"),
              (p + "self_attn.k_proj.weight", (cfg.num_kv_heads * hd, H), "normal"),
              (p + "self_attn.v_proj.weight", (cfg.num_kv_heads * hd, H), "normal"),
              (p + "self_attn.o_proj.weight", (H, cfg.num_heads * hd), "normal"),
              (p + "mlp.gate_proj.weight", (cfg.intermediate_size, H), "normal"),
              (p + "mlp.up_proj.weight", (cfg.intermediate_size, H), "normal"),
              (p + "mlp.down_proj.weight", (H, cfg.intermediate_size), "normal")]
    s += [(T + "norm.weight", (H,), "ones"), ("score.weight", (cfg.num_labels, H), "normal")]
    return s


def random_weights(cfg: ModelConfig, seed: int = 0, std: float = 0.02) -> dict:
    """name -> bf16 bits (np.uint16) in the tensor's shape."""
    out = {}
    for name, shape, kind in weight_specs(cfg):
        n = int(np.prod(shape))
        if kind == "ones":
            v = np.ones(n, np.float32)
        elif kind == "zeros":
            v = np.zeros(n, np.float32)
        else:
            v = _rng(seed, name).standard_normal(n, dtype=np.float32) * np.float32(std)
        out[name] = _bf16_bits(v).reshape(shape)
    return out


def save_safetensors(path: str, tensors: dict) -> None:
    """Write a safetensors file: values are bf16 bits (np.uint16) or
    (dtype str, array) pairs with dtype "BF16" | "F16" | "F32"."""
    np_t = {"BF16": np.uint16, "F16": np.float16, "F32": np.float32}
    items = []
    for name, v in tensors.items():
        dt, arr = v if isinstance(v, tuple) else ("BF16", v)
        # np.asarray keeps a rank-0 tensor rank 0 (ascontiguousarray would not)
        items.append((name, dt, np.asarray(arr, dtype=np_t[dt], order="C")))
    header, off = {}, 0
    for name, dt, arr in items:
        nb = arr.nbytes
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + nb]}
        off += nb
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for _, _, arr in items:
            f.write(arr.tobytes())


def load_safetensors(path: str) -> dict:
    """mmap a safetensors file: name -> (dtype str, np array view)."""
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    hl = int(np.frombuffer(mm[:8].tobytes(), "<u8")[0])
    header = json.loads(bytes(mm[8:8 + hl]).decode())
    base = 8 + hl
    out = {}
    np_t = {"BF16": np.uint16, "F16": np.float16, "F32": np.float32}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        a, b = meta["data_offsets"]
        arr = mm[base + a:base + b].view(np_t[meta["dtype"]]).reshape(meta["shape"])
        out[name] = (meta["dtype"], arr)
    return out


def write_model_dir(path: str, cfg: ModelConfig, seed: int = 0) -> None:
    """A complete `-hf` model directory: config.json, model.safetensors and the
    tokenizer files (a real tokenizer.json for the `tokenizers` binding that
    encodes as SyntheticTokenizer does, and tokenizer_config.json)."""
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg.config_json(), f)
    save_safetensors(os.path.join(path, "model.safetensors"), random_weights(cfg, seed))
    write_tokenizer_dir(path)


# ---------------------------------------------------------------- Local Head package

LOCAL_HEAD_OFFSETS_MS = [float(o) for o in range(-60, 61, 10)]
LOCAL_HEAD_FEATURES = 91


def local_head_prior() -> np.ndarray:
    """The canonical inference prior, -0.5 (o / 35)^2 x 2 (src/local_head.rs:709-714)."""
    return np.array([-0.5 * (o / 35.0) ** 2 * 2.0 for o in LOCAL_HEAD_OFFSETS_MS], np.float32)


def local_head_specs() -> list:
    """(name, shape, kind, fan_in) of every Local Head tensor (src/local_head.rs:876-912).
    kind: 'normal' (std 1/sqrt(fan_in)) | 'ones' | 'zeros' | 'prior' | 'scale'."""
    d, q, f = 128, 1024, LOCAL_HEAD_FEATURES
    s = [("audio.0.weight", (d, f, 5), "normal", f * 5), ("audio.0.bias", (d,), "normal", f * 5),
         ("audio.2.weight", (d, d, 5), "normal", d * 5), ("audio.2.bias", (d,), "normal", d * 5),
         ("context_projection.weight", (d, q), "normal", q),
         ("context_projection.bias", (d,), "normal", q),
         ("role_embedding.weight", (4, d), "normal", 1),
         ("endpoint_embedding.weight", (2, d), "normal", 1)]
    for att in ("context_attention", "audio_attention"):
        s += [(att + ".in_proj_weight", (3 * d, d), "normal", d),
              (att + ".in_proj_bias", (3 * d,), "zeros", d),
              (att + ".out_proj.weight", (d, d), "normal", d),
              (att + ".out_proj.bias", (d,), "zeros", d)]
    for nm in ("query_norm", "audio_norm"):
        s += [(nm + ".weight", (d,), "ones", 1), (nm + ".bias", (d,), "zeros", 1)]
    s += [("activity_bias.weight", (1, d), "normal", d), ("activity_bias.bias", (1,), "normal", d),
          ("boundary_bias.weight", (1, d), "normal", d), ("boundary_bias.bias", (1,), "normal", d),
          ("derivative_scale", (), "scale", 1), ("qwen_prior", (13,), "prior", 1)]
    return s


def random_local_head(seed: int = 0):
    """(tensors name -> ("F32", array), mean [91], std [91]) of a seeded random
    Local Head with the canonical prior and a positive normalizer."""
    out = {}
    for name, shape, kind, fan_in in local_head_specs():
        n = int(np.prod(shape)) if shape else 1
        if kind == "ones":
            v = np.ones(n, np.float32)
        elif kind == "zeros":
            v = np.zeros(n, np.float32)
        elif kind == "prior":
            v = local_head_prior()
        elif kind == "scale":
            v = np.array([0.5], np.float32)
        else:
            v = _rng(seed, "local_head:" + name).standard_normal(n, dtype=np.float32)
            v *= np.float32(1.0 / np.sqrt(fan_in))
        out[name] = ("F32", v.reshape(shape))
    r = _rng(seed, "local_head:normalizer")
    mean = np.concatenate([r.uniform(-9.0, -4.0, 80), r.uniform(-5.0, -3.0, 1),
                           r.uniform(-0.1, 0.1, 1), r.uniform(0.2, 0.6, 1),
                           r.uniform(0.3, 1.2, 8)]).astype(np.float32)
    std = np.concatenate([r.uniform(1.5, 3.5, 80), r.uniform(1.0, 2.0, 1),
                          r.uniform(0.2, 0.6, 1), r.uniform(0.2, 0.8, 1),
                          r.uniform(0.2, 0.8, 8)]).astype(np.float32)
    return out, mean, std


def local_head_config_json() -> dict:
    """config.json of a Local Head package, the contract of src/local_head.rs:617-700."""
    return {
        "schema": "qwen-fa-ultra.local-head.v1",
        "architecture": "IdentityConditionedBoundaryHead",
        "offsets_ms": LOCAL_HEAD_OFFSETS_MS,
        "decoder_temperature": 1.5,
        "decoder_amplitude": 1.0,
        "inference_prior_scale": 2.0,
        "context_roles": ["timestamp slot", "current avg", "prev avg", "next avg"],
        "feature_contract": {"center_source": "fixed", "context_ms": 200, "feature_dim": 91,
                             "frame_count": 41, "frame_ms": 25, "hop_ms": 10, "n_fft": 512,
                             "n_mels": 80, "sample_rate": 16000, "spectral_distance_bands": 4},
        "model_config": {"acoustic_dim": 91, "activity_weight": 0.25, "heads": 4,
                         "model_dim": 128, "prior_sigma_ms": 35.0, "qwen_dim": 1024},
    }


def write_local_head_dir(model_dir: str, seed: int = 0) -> str:
    """<model_dir>/local_head/ with config.json, normalizer.json and the F32
    model.safetensors; returns the package directory."""
    d = os.path.join(model_dir, "local_head")
    os.makedirs(d, exist_ok=True)
    tensors, mean, std = random_local_head(seed)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(local_head_config_json(), f)
    with open(os.path.join(d, "normalizer.json"), "w") as f:
        json.dump({"mean": mean.tolist(), "std": std.tolist()}, f)
    save_safetensors(os.path.join(d, "model.safetensors"), tensors)
    return d


# ---------------------------------------------------------------- tokenizer

class SyntheticTokenizer:
    """Deterministic stand-in for the checkpoint's BPE (`tokenizers` 0.22.2).

    Contract kept from the reference's use of it (src/align_input.rs:183-262):
    the four markers are atomic with the checkpoint ids; encoding adds no
    special tokens; every other character sequence maps to ordinary ids below
    151643.  A CJK ideograph is one token; Latin letters are grouped in 3s."""

    MARKERS = {AUDIO_START: AUDIO_START_ID, AUDIO_END: AUDIO_END_ID, AUDIO_PAD: AUDIO_PAD_ID,
               TIMESTAMP: TIMESTAMP_ID}
    ORDINARY = 151643

    def token_to_id(self, s: str):
        return self.MARKERS.get(s)

    _IDS: dict = {}  # piece -> id (the mapping is a pure function of the piece)

    def _piece_id(self, piece: str) -> int:
        i = self._IDS.get(piece)
        if i is None:
            h = hashlib.blake2b(piece.encode(), digest_size=8).digest()
            i = self._IDS[piece] = int.from_bytes(h, "little") % self.ORDINARY
        return i

    _SPLIT = None

    def encode(self, text: str) -> list:
        import re
        if SyntheticTokenizer._SPLIT is None:
            SyntheticTokenizer._SPLIT = re.compile(
                "(" + "|".join(re.escape(k) for k in self.MARKERS) + ")")
        ids = []
        for part in self._SPLIT.split(text):
            if not part:
                continue
            m = self.MARKERS.get(part)
            if m is not None:
                ids.append(m)
                continue
            if part.isascii():  # no CJK: one run, cut in threes
                pid = self._piece_id
                ids += [pid(part[j:j + 3]) for j in range(0, len(part), 3)]
                continue
            buf = ""
            for ch in part:
                if 0x3400 <= ord(ch) <= 0x9FFF or 0xF900 <= ord(ch) <= 0xFAFF:
                    if buf:
                        ids += self._word(buf)
                        buf = ""
                    ids.append(self._piece_id(ch))
                else:
                    buf += ch
            if buf:
                ids += self._word(buf)
        return ids

    def _word(self, w: str) -> list:
        return [self._piece_id(w[j:j + 3]) for j in range(0, len(w), 3)]

    def encode_batch(self, texts: list) -> list:
        return [self.encode(t) for t in texts]


class HFTokenizer:
    """A `tokenizers.Tokenizer` (the Python binding of the `tokenizers` crate
    0.22.2 the reference links, Cargo.lock) behind the interface InputBuilder
    uses: `token_to_id`, `encode(text) -> ids` with no special tokens added
    (src/align_input.rs:180-186), and `encode_batch(texts)`, which the binding
    spreads over the host cores."""

    def __init__(self, tok):
        self.tok = tok

    @classmethod
    def from_file(cls, path: str) -> "HFTokenizer":
        import tokenizers
        return cls(tokenizers.Tokenizer.from_file(str(path)))

    def token_to_id(self, s: str):
        return self.tok.token_to_id(s)

    def encode(self, text: str) -> list:
        return self.tok.encode(text, add_special_tokens=False).ids

    def encode_batch(self, texts: list) -> list:
        # encode_batch_fast computes no character offsets (ids are all the
        # input builder needs); the same ids as encode_batch
        f = getattr(self.tok, "encode_batch_fast", None) or self.tok.encode_batch
        return [e.ids for e in f(list(texts), add_special_tokens=False)]


def as_tokenizer(tok):
    """SyntheticTokenizer / HFTokenizer as they are; a bare `tokenizers.Tokenizer`
    wrapped; None -> SyntheticTokenizer."""
    if tok is None:
        return SyntheticTokenizer()
    if hasattr(tok, "encode_batch") and hasattr(tok, "get_vocab_size"):
        return HFTokenizer(tok)
    return tok


# Ordinary-token alphabet of the synthetic tokenizer.json: every 1-3 letter
# lowercase piece and every CJK ideograph the workloads draw (U+4E00..U+62FF).
_SYN_CJK = (0x4E00, 0x62FF)
_SYN_CJK_CLASS = r"\x{3400}-\x{9FFF}\x{F900}-\x{FAFF}"  # Oniguruma syntax


def synthetic_tokenizer_json() -> dict:
    """A tokenizer.json (`tokenizers` 0.22.2 format) that encodes exactly as
    SyntheticTokenizer does over the workloads' alphabet: the four markers
    are added tokens with the checkpoint's ids; a Split pre-tokenizer cuts
    every run of non-CJK characters into 3-character pieces and isolates each
    CJK character; a WordLevel model maps each piece to SyntheticTokenizer's
    id for it.  Pieces outside the alphabet map to <unk>."""
    import itertools
    import string
    st = SyntheticTokenizer()
    vocab = {}
    for n in (1, 2, 3):
        for p in itertools.product(string.ascii_lowercase, repeat=n):
            piece = "".join(p)
            vocab[piece] = st._piece_id(piece)
    for c in range(_SYN_CJK[0], _SYN_CJK[1] + 1):
        vocab[chr(c)] = st._piece_id(chr(c))
    vocab["<unk>"] = SyntheticTokenizer.ORDINARY - 1
    markers = [(AUDIO_START, AUDIO_START_ID), (AUDIO_END, AUDIO_END_ID),
               (AUDIO_PAD, AUDIO_PAD_ID), (TIMESTAMP, TIMESTAMP_ID)]
    for m, i in markers:
        vocab[m] = i
    cjk = _SYN_CJK_CLASS
    return {
        "version": "1.0", "truncation": None, "padding": None,
        "added_tokens": [{"id": i, "content": m, "single_word": False, "lstrip": False,
                          "rstrip": False, "normalized": False, "special": True}
                         for m, i in markers],
        "normalizer": None,
        "pre_tokenizer": {"type": "Split", "pattern": {"Regex": f"[^{cjk}]{{1,3}}|[{cjk}]"},
                          "behavior": "Isolated", "invert": False},
        "post_processor": None, "decoder": None,
        "model": {"type": "WordLevel", "vocab": vocab, "unk_token": "<unk>"},
    }


def write_tokenizer_dir(path: str) -> None:
    """tokenizer.json + tokenizer_config.json (with the marker keys the
    reference reads, src/align_input.rs:138-151) into a model directory."""
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "tokenizer.json"), "w") as f:
        json.dump(synthetic_tokenizer_json(), f)
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        json.dump({"audio_token": AUDIO_PAD, "audio_bos_token": AUDIO_START,
                   "audio_eos_token": AUDIO_END}, f)


# ---------------------------------------------------------------- words / inputs

def is_cjk_char(c: str) -> bool:
    """src/words.rs:30-40."""
    k = ord(c)
    return (0x4E00 <= k <= 0x9FFF or 0x3400 <= k <= 0x4DBF or 0x20000 <= k <= 0x2A6DF
            or 0x2A700 <= k <= 0x2B73F or 0x2B740 <= k <= 0x2B81F or 0x2B820 <= k <= 0x2CEAF
            or 0xF900 <= k <= 0xFAFF or 0x2F800 <= k <= 0x2FA1F)


def is_hangul_char(c: str) -> bool:
    """src/words.rs:44-51."""
    k = ord(c)
    return (0x1100 <= k <= 0x11FF or 0x3130 <= k <= 0x318F or 0xA960 <= k <= 0xA97F
            or 0xAC00 <= k <= 0xD7A3 or 0xD7B0 <= k <= 0xD7FF)


def is_kept_char(c: str) -> bool:
    """src/words.rs:59-74: apostrophe, or general category L* / N*, or CJK."""
    import unicodedata
    return c == "'" or unicodedata.category(c)[0] in "LN" or is_cjk_char(c)


# Rust's char::is_whitespace: the Unicode White_Space property.
_WHITE_SPACE = "\t\n\x0b\x0c\r \x85\xa0\u1680\u2000-\u200a\u2028\u2029\u202f\u205f\u3000"
# is_cjk_char's ranges (src/words.rs:30-40).
_CJK_RANGES = ("\u4e00-\u9fff\u3400-\u4dbf\U00020000-\U0002a6df\U0002a700-\U0002b73f"
               "\U0002b740-\U0002b81f\U0002b820-\U0002ceaf\uf900-\ufaff\U0002f800-\U0002fa1f")
# is_hangul_char's ranges (src/words.rs:44-51).
_HANGUL_RANGES = "\u1100-\u11ff\u3130-\u318f\ua960-\ua97f\uac00-\ud7a3\ud7b0-\ud7ff"
_SPLIT_RE = None


def _split_res():
    global _SPLIT_RE
    if _SPLIT_RE is None:
        import re
        import regex  # Unicode general categories (\p{L}, \p{N})
        _SPLIT_RE = (
            # neither kept (apostrophe, L*, N*, CJK) nor whitespace: dropped
            regex.compile(f"[^\\p{{L}}\\p{{N}}'{_WHITE_SPACE}{_CJK_RANGES}]+"),
            # a CJK character alone, or a run of kept non-CJK characters
            # (explicit ranges only: the standard engine is faster here)
            re.compile(f"[{_CJK_RANGES}]|[^{_WHITE_SPACE}{_CJK_RANGES}]+"),
            re.compile(f"[{_HANGUL_RANGES}]"),
        )
    return _SPLIT_RE


def split_words(text: str, language=None) -> list:
    """src/words.rs:107-118 + split_default (:190-232) for every language but
    Japanese (which needs the reference's nagisa tagger and is out of scope).

    split_default walks the characters: a CJK character is a word of its own;
    whitespace (Unicode White_Space) ends a word; apostrophes, letters (L*)
    and numbers (N*) are kept; anything else is dropped without ending the
    word ("50-minute" is one word); a change between Hangul and non-Hangul
    letters inside a run ends the word, numbers and apostrophes attaching to
    the current run.  Here the dropped characters are removed first (that
    cannot end a word), the words are then the CJK characters and the runs
    between whitespace and CJK characters, and only runs holding Hangul are
    walked character by character for the script change."""
    drop, word, hangul = _split_res()
    lang = (language or "").lower()
    if lang in ("japanese", "ja"):
        raise ValueError("Japanese word splitting requires the nagisa tagger (not available)")
    tokens = word.findall(drop.sub("", text))
    if not hangul.search(text):
        return tokens
    out = []
    for t in tokens:
        if hangul.search(t):
            _split_script(t, out)
        else:
            out.append(t)
    return out


def _split_script(run: str, tokens: list) -> None:
    """A run of kept non-CJK characters cut where the letters change between
    Hangul and other scripts (src/words.rs:205-224)."""
    import unicodedata
    buf, buf_hangul = "", None
    for c in run:
        if c != "'" and unicodedata.category(c)[0] == "L":  # a script letter, not a number
            h = is_hangul_char(c)
            if buf_hangul is not None and buf_hangul != h:
                tokens.append(buf)
                buf = ""
            buf_hangul = h
        buf += c
    if buf:
        tokens.append(buf)


def conv3_length(n: int) -> int:
    """src/align_input.rs:49-57."""
    for _ in range(3):
        n = (n - 1) // 2 + 1 if n > 0 else 0
    return n


def audio_token_count(valid_mel_frames: int, n_window: int = 50) -> int:
    """src/align_input.rs:63-67."""
    cl = n_window * 2
    return (valid_mel_frames // cl) * 13 + conv3_length(valid_mel_frames % cl)


def padded_mel_frames(valid: int, n_window: int = 50) -> int:
    """src/align_input.rs:71-79."""
    m = n_window * 2
    r = valid % m
    return valid if r == 0 else valid + (m - r)


def valid_mel_frames(n_samples: int) -> int:
    """src/align_input.rs:85-87."""
    return n_samples // HOP


@dataclass
class AlignerInput:
    """src/align_input.rs:91-111 (input_ids / timestamp_positions: int
    sequences, lists or numpy arrays)."""
    input_ids: list
    words: list
    n_audio_tokens: int
    valid_mel_frames: int
    padded_mel_frames: int
    timestamp_positions: list = field(default_factory=list)

    def seq_len(self) -> int:
        return len(self.input_ids)


class InputBuilder:
    """InputBuilder (src/align_input.rs:119-262): the checkpoint's tokenizer
    and the marker ids, with the reference's structural checks."""

    def __init__(self, tokenizer=None, n_window: int = 50, timestamp_token_id: int = TIMESTAMP_ID,
                 markers: dict = None):
        self.tok = as_tokenizer(tokenizer)
        self.n_window = n_window
        m = {"audio_token": AUDIO_PAD, "audio_bos_token": AUDIO_START,
             "audio_eos_token": AUDIO_END, **(markers or {})}

        def id_of(text):
            i = self.tok.token_to_id(text)
            if i is None:
                raise ValueError(f"tokenizer has no {text!r}")
            return int(i)
        self.audio_start_token_id = id_of(m["audio_bos_token"])
        self.audio_end_token_id = id_of(m["audio_eos_token"])
        self.audio_token_id = id_of(m["audio_token"])
        self.timestamp_token_id = int(timestamp_token_id)

    @classmethod
    def load(cls, model_dir: str, timestamp_token_id: int = TIMESTAMP_ID, n_window: int = 50):
        """InputBuilder::load (src/align_input.rs:131-171): tokenizer.json via
        the `tokenizers` binding, the marker strings from
        tokenizer_config.json (defaults when a key is absent)."""
        tok = HFTokenizer.from_file(os.path.join(model_dir, "tokenizer.json"))
        with open(os.path.join(model_dir, "tokenizer_config.json")) as f:
            cfg = json.load(f)
        markers = {k: cfg[k] for k in ("audio_token", "audio_bos_token", "audio_eos_token")
                   if isinstance(cfg.get(k), str)}
        return cls(tok, n_window=n_window, timestamp_token_id=timestamp_token_id,
                   markers=markers)

    @staticmethod
    def _words_text(words: list) -> str:
        # w0 <ts><ts> w1 <ts><ts> ... wn <ts><ts> (src/align_input.rs:202-210)
        return (TIMESTAMP + TIMESTAMP).join(words) + TIMESTAMP + TIMESTAMP

    def build(self, words: list, valid_mel: int) -> AlignerInput:
        return self.build_batch([words], [valid_mel], as_arrays=False)[0]

    def build_batch(self, word_lists: list, valid_mels: list, as_arrays: bool = True) -> list:
        """One AlignerInput per clip, the words of all clips tokenised in one
        encode_batch call (spread over the host cores by the `tokenizers`
        binding).  input_ids / timestamp_positions are uint32 / int64 numpy
        arrays (lists with as_arrays=False)."""
        n_audio = [audio_token_count(v, self.n_window) for v in valid_mels]
        for na, v in zip(n_audio, valid_mels):
            if na <= 0:
                raise ValueError(f"audio produced 0 tokens ({v} mel frames)")
        texts = [self._words_text(w) for w in word_lists]
        tok = self.tok
        encs = tok.encode_batch(texts) if hasattr(tok, "encode_batch") else [tok.encode(t) for t in texts]
        out = []
        for words, v, na, enc in zip(word_lists, valid_mels, n_audio, encs):
            # The reference tokenises "<|audio_start|>" + pads + "<|audio_end|>" +
            # words as one string; the markers are atomic tokens (no merge
            # crosses them), so the marker run is emitted directly and only the
            # words go through the tokenizer: the same ids without scanning N pads.
            e = np.asarray(enc, dtype=np.uint32)
            ids = np.empty(na + 2 + len(e), np.uint32)
            ids[0] = self.audio_start_token_id
            ids[1:na + 1] = self.audio_token_id
            ids[na + 1] = self.audio_end_token_id
            ids[na + 2:] = e
            if int(np.count_nonzero(e == self.audio_token_id)) != 0:
                raise ValueError(f"expected {na} audio tokens, the words hold more")
            ts = np.flatnonzero(e == self.timestamp_token_id).astype(np.int64) + (na + 2)
            if len(ts) != 2 * len(words):
                raise ValueError(f"expected {2 * len(words)} timestamp tokens for {len(words)} "
                                 f"words, got {len(ts)}")
            if as_arrays:
                inp = AlignerInput(ids, list(words), na, v, padded_mel_frames(v, self.n_window), ts)
            else:
                inp = AlignerInput(ids.tolist(), list(words), na, v,
                                   padded_mel_frames(v, self.n_window), ts.tolist())
            out.append(inp)
        return out


# ---------------------------------------------------------------- audio / text

def synth_audio(seconds: float, seed: int, rate: int = SAMPLE_RATE) -> np.ndarray:
    """Syllable-like bursts of low-passed noise at RMS 0.1, f32 at `rate` Hz
    (16 kHz by default, the model's rate; other rates stand in for files that
    must be resampled)."""
    from scipy.signal import butter, sosfiltfilt
    rng = np.random.default_rng(seed)
    n = int(round(seconds * rate))
    noise = rng.standard_normal(n)
    sos = butter(4, 3400, btype="low", fs=rate, output="sos")
    x = sosfiltfilt(sos, noise)
    env = np.zeros(n)
    t = int(rng.uniform(0.04, 0.2) * rate)
    while t < n:
        d = int(rng.uniform(0.15, 0.40) * rate)
        e = min(n, t + d)
        env[t:e] = np.hanning(d)[: e - t]
        t = e + int(rng.uniform(0.04, 0.2) * rate)
    y = x * env
    rms = np.sqrt(np.mean(y * y)) if n else 1.0
    y = y * (0.1 / max(rms, 1e-12))
    return y.astype(np.float32)


def english_words(count: int, rng: np.random.Generator) -> list:
    letters = np.array(list("abcdefghijklmnopqrstuvwxyz"))
    return ["".join(rng.choice(letters, size=int(rng.integers(3, 9)))) for _ in range(count)]


def chinese_words(count: int, rng: np.random.Generator) -> list:
    return [chr(int(rng.integers(0x4E00, 0x62FF + 1))) for _ in range(count)]


@dataclass
class Clip:
    samples: np.ndarray
    text: str
    language: str
    seconds: float


def _clip_text(config: int, i: int, n_words: int, mix_cjk: bool, seed_base=None):
    seed = 1000 * config + i if seed_base is None else seed_base + i
    rng = np.random.default_rng(seed + 7)
    if mix_cjk:
        words, left, en = [], n_words, True
        while left > 0:
            run = min(left, int(rng.integers(2, 7)))
            words += english_words(run, rng) if en else chinese_words(run, rng)
            left -= run
            en = not en
        text, lang = "".join(w if is_cjk_char(w[0]) else f" {w} " for w in words), "Chinese"
    else:
        words = english_words(n_words, rng)
        text, lang = " ".join(words), "English"
    return " ".join(text.split()), lang, seed


def _spec(config: int, n: int) -> list:
    """(seconds, n_words, mix_cjk) of clips 0 .. n-1 of configuration 2 or 4."""
    if config == 2:
        rng = np.random.default_rng(2000)
        spec = [(float(rng.uniform(5, 30)), float(rng.uniform(2.5, 3.5))) for _ in range(n)]
        return [(sec, max(1, int(round(sec * rate))), True) for sec, rate in spec]
    if config == 4:
        rng = np.random.default_rng(4000)
        spec = [float(rng.uniform(5, 60)) for _ in range(n)]
        return [(sec, max(1, int(round(sec * 3.0))), False) for sec in spec]
    raise ValueError(config)


def workload_texts(config: int, n_clips: int) -> list:
    """(seconds, text, language) of clips 0 .. n_clips-1 of configuration 2 or
    4, without synthesising any audio (the text and duration of clip i are
    those workload() gives it)."""
    return [(sec, *_clip_text(config, i, nw, cjk)[:2])
            for i, (sec, nw, cjk) in enumerate(_spec(config, n_clips))]


def workload_clip(config: int, i: int) -> Clip:
    """Clip i of configuration 2 or 4 alone (the same clip workload() gives)."""
    sec, nw, cjk = _spec(config, i + 1)[i]
    text, lang, seed = _clip_text(config, i, nw, cjk)
    return Clip(synth_audio(sec, seed), text, lang, sec)


def workload(config: int, seed_base: int = None, n_clips: int = None, start: int = 0) -> list:
    """The clips of a BASELINE configuration (0-4), clip i seeded 1000 * config + i.

    ``n_clips`` overrides the configuration's clip count (configs 2 and 4) and
    ``start`` skips the first clips, so shards of a long stream (one per GPU)
    can be generated without synthesising the others."""
    clips = []

    def one(i, seconds, n_words, mix_cjk=False):
        text, lang, seed = _clip_text(config, i, n_words, mix_cjk, seed_base)
        return Clip(synth_audio(seconds, seed), text, lang, seconds)

    if config == 0:
        clips.append(one(0, 10.0, 25))
    elif config == 1:
        clips.append(one(0, 60.0, 180))
    elif config in (2, 4):
        n = (64 if config == 2 else 4096) if n_clips is None else n_clips
        for i, (sec, nw, cjk) in enumerate(_spec(config, start + n)):
            if i >= start:
                clips.append(one(i, sec, nw, mix_cjk=cjk))
    elif config == 3:
        clips.append(one(0, 300.0, 900))
    else:
        raise ValueError(config)
    return clips


def asdict_cfg(cfg: ModelConfig) -> dict:
    return asdict(cfg)
