"""Python mirror of the reference crate's `Aligner` (src/align_inference.rs)
on top of the C ABI of libqa_b200.so.

Same names, argument meaning and error behaviour as the Rust API where it
applies:

* ``Aligner.load_backend_with_dtype(model, half)`` — load weights onto one
  CUDA device in the given 16-bit storage format (``"f16"`` default, ``"bf16"``);
* ``align(path, text, language)`` -> items and ``align_with_raw(path, ...)``
  -> ``(raw_ms, items)`` — a WAV file (src/align_inference.rs:485-511);
* ``align_samples(samples, text, language)`` -> ``(raw_ms, items)`` — one clip
  of 16 kHz mono f32 audio (src/align_inference.rs:521-569); with a Local
  Head loaded and enabled the items are its refined word times;
* ``local_head()``, ``local_head_enabled()``, ``set_local_head_enabled(on)``
  (src/align_inference.rs:571-593);
* ``align_batch([(samples, text, language), ...])`` — many independent clips
  in one device-resident pass (new: the reference aligns one clip per call);
* the tower-boundary stages ``mel``, ``audio_embeds``, ``text_hidden`` and
  ``head`` (src/align_inference.rs:103-181, 737-805) for callers that drive
  the phases themselves.

Every failure of the C ABI raises ``QaError`` carrying the status code
(QA_ERR_SHAPE, QA_ERR_CAP, ...) and the library's message; nothing falls back
to a CPU path.
"""
from __future__ import annotations

import ctypes
import os
import time

import numpy as np

from . import _lib
from . import audio as _audio
from . import local_head as _lh
from . import postprocess
from . import synth


FORCED_ALIGNER_LANGUAGES = ["Chinese", "Cantonese", "English", "French", "German", "Italian",
                            "Japanese", "Korean", "Portuguese", "Russian", "Spanish"]


class Aligner:
    def __init__(self, ctx, cfg: synth.ModelConfig, half: str, builder: synth.InputBuilder):
        self._ctx = ctx
        self.cfg = cfg
        self._half = half
        self.input_builder = builder
        self.timings = None
        self._local_head = None

    # ------------------------------------------------------------ load / close

    @classmethod
    def load_backend_with_dtype(cls, model, half: str = "f16", device: int = 0,
                                cfg: synth.ModelConfig = None, tokenizer=None,
                                local_head=None) -> "Aligner":
        """``model``: a model directory (config.json + model.safetensors, `-hf`
        layout, and the optional local_head/ package) or a dict of name ->
        bf16 bits / (dtype, array) with ``cfg`` (and optionally ``local_head``
        = (tensors, mean, std) of a Local Head package)."""
        half = half.lower()
        if half in ("f16", "fp16", "half"):
            code = _lib.QA_HALF_F16
        elif half in ("bf16", "bfloat16"):
            code = _lib.QA_HALF_BF16
        else:
            raise ValueError(f"unknown 16-bit format {half!r}")
        if isinstance(model, (str, os.PathLike)):
            import json
            with open(os.path.join(model, "config.json")) as f:
                cfg = synth.ModelConfig.from_config_json(json.load(f))
            weights = synth.load_safetensors(os.path.join(model, "model.safetensors"))
            if local_head is None:
                local_head = _lh.load_package(model)
        else:
            if cfg is None:
                raise ValueError("a weights dict needs its ModelConfig")
            weights = model
        L = _lib.lib()
        ctx = ctypes.c_void_p()
        _lib.check(L.qa_open(device, code, ctypes.byref(ctx)))
        tens, keep = _lib.make_tensors(weights)
        qcfg = _lib.make_cfg(cfg)
        rc = L.qa_load(ctx, ctypes.addressof(tens), len(tens), ctypes.addressof(qcfg))
        del keep
        if rc != _lib.QA_OK:
            msg = L.qa_last_error(ctx)
            L.qa_close(ctx)
            raise _lib.QaError(rc, msg.decode() if msg else "")
        try:
            builder = cls._input_builder(model, tokenizer, cfg)
        except Exception:
            L.qa_close(ctx)
            raise
        al = cls(ctx, cfg, "bf16" if code else "f16", builder)
        if local_head is not None:
            try:
                al._local_head = _lh.load_into(al, *local_head)
            except Exception:
                al.close()
                raise
        return al

    @staticmethod
    def _input_builder(model, tokenizer, cfg) -> synth.InputBuilder:
        """The tokenizer as the reference loads it (src/align_inference.rs:
        331-336 -> InputBuilder::load): a model directory's tokenizer.json +
        tokenizer_config.json when there is one; else `tokenizer` (a
        tokenizer.json path, a `tokenizers.Tokenizer`, or None for the
        synthetic tokenizer)."""
        if tokenizer is None and isinstance(model, (str, os.PathLike)) and os.path.exists(
                os.path.join(model, "tokenizer.json")):
            return synth.InputBuilder.load(model, cfg.timestamp_token_id, n_window=cfg.n_window)
        if isinstance(tokenizer, (str, os.PathLike)):
            tokenizer = synth.HFTokenizer.from_file(tokenizer)
        return synth.InputBuilder(tokenizer, n_window=cfg.n_window,
                                  timestamp_token_id=cfg.timestamp_token_id)

    @classmethod
    def load_with_dtype(cls, model, half: str = "f16", **kw) -> "Aligner":
        return cls.load_backend_with_dtype(model, half, **kw)

    @classmethod
    def load(cls, model, **kw) -> "Aligner":
        return cls.load_backend_with_dtype(model, "f16", **kw)

    def close(self) -> None:
        if self._ctx:
            _lib.lib().qa_close(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def half(self) -> str:
        return self._half

    def backend_name(self) -> str:
        return "cuda"

    # ------------------------------------------------------------ Local Head

    def local_head(self):
        """The Local Head this checkpoint ships, if any (a LocalHead handle)."""
        return self._local_head

    def local_head_enabled(self) -> bool:
        """Whether align runs the Local Head."""
        return bool(self._ctx) and _lib.lib().qa_local_head_enabled(self._ctx) == 1

    def set_local_head_enabled(self, enabled: bool) -> None:
        """Turn the Local Head on or off; enabling it on a checkpoint that
        ships none raises (src/align_inference.rs:584-593)."""
        if enabled and self._local_head is None:
            raise ValueError("this checkpoint has no local_head/ package")
        self._check(_lib.lib().qa_set_local_head_enabled(self._ctx, 1 if enabled else 0))

    def set_timeout_ms(self, ms: int) -> None:
        self._check(_lib.lib().qa_set_timeout_ms(self._ctx, int(ms)))

    def _check(self, rc: int) -> None:
        _lib.check(rc, self._ctx)

    # ------------------------------------------------------------ language

    def supported_languages(self) -> list:
        return sorted({s.lower() for s in FORCED_ALIGNER_LANGUAGES})

    def check_language(self, language) -> None:
        if language is None:
            return
        if language.lower() not in self.supported_languages():
            raise ValueError(f"language {language.lower()!r} is not supported by the forced "
                             f"aligner; supported: {self.supported_languages()}")

    # ------------------------------------------------------------ whole path

    def build_input(self, samples: np.ndarray, text: str, language=None):
        self.check_language(language)
        words = synth.split_words(text, language)
        return self.input_builder.build(words, synth.valid_mel_frames(len(samples)))

    def build_inputs(self, clips, host: dict = None) -> list:
        """AlignerInputs of [(samples, text, language)]: every clip's words
        split, then all clips tokenised in one batch call.  Adds the time of
        each part to host["words_ms"] / host["build_ms"] when given."""
        t0 = time.perf_counter()
        words = []
        for _, t, l in clips:
            self.check_language(l)
            words.append(synth.split_words(t, l))
        t1 = time.perf_counter()
        inputs = self.input_builder.build_batch(
            words, [synth.valid_mel_frames(len(s)) for s, _, _ in clips])
        if host is not None:
            host["words_ms"] = host.get("words_ms", 0.0) + (t1 - t0) * 1e3
            host["build_ms"] = host.get("build_ms", 0.0) + (time.perf_counter() - t1) * 1e3
        return inputs

    def align(self, audio, text: str, language=None) -> list:
        """Word items for a WAV file (src/align_inference.rs:485-492): the file is
        decoded, downmixed and, if it is not 16 kHz, resampled
        (audio.load_audio_wav), then aligned as align_samples does."""
        return self.align_with_raw(audio, text, language)[1]

    def align_with_raw(self, audio, text: str, language=None):
        """(raw_ms, items) for a WAV file (src/align_inference.rs:501-511)."""
        self.check_language(language)
        t0 = time.perf_counter()
        samples = _audio.load_audio_wav(audio)
        wav_ms = (time.perf_counter() - t0) * 1e3
        out = self.align_samples(samples, text, language)
        self.timings["wav_ms"] = wav_ms
        return out

    def align_samples(self, samples: np.ndarray, text: str, language=None):
        """(raw_ms, items) for one clip (src/align_inference.rs:521-569)."""
        return self.align_batch([(samples, text, language)])[0]

    def align_batch(self, clips, want_logits: bool = False, want_normed: bool = False):
        """[(samples, text, language)] -> [(raw_ms, items)]; raw_ms is the
        unrepaired argmax stream, items the repaired word times.

        Afterwards ``timings`` holds the device phases of the pass and, as the
        reference's Timings does (src/align_inference.rs:230-251), the host
        phases: words_ms (word split), build_ms (tokenise and assemble the
        input ids) and post_ms (timestamp repair and pairing)."""
        host = {"words_ms": 0.0, "build_ms": 0.0}
        inputs = self.build_inputs(clips, host)
        raws = self.align_inputs([c[0] for c in clips], inputs, want_logits, want_normed)
        t0 = time.perf_counter()
        out = self._items(inputs, raws, want_logits or want_normed)
        host["post_ms"] = (time.perf_counter() - t0) * 1e3
        self.timings = dict(self.timings or {}, **host)
        return out

    @staticmethod
    def _items(inputs, raws, with_extra: bool) -> list:
        """(raw_ms, items[, extra]) per clip: the Local Head's intervals when it
        ran, else the repaired coarse stream paired with the words."""
        out = []
        for (r, extra), inp in zip(raws, inputs):
            iv = extra.get("intervals")
            if iv is not None:
                items = [postprocess.AlignItem(w, float(a), float(b))
                         for w, (a, b) in zip(inp.words, iv)]
            else:
                items = postprocess.pair_words(inp.words, _lib.fix_timestamps(r))
            out.append((r, items, extra) if with_extra else (r, items))
        return out

    def align_stream(self, batches, want_logits: bool = False, want_normed: bool = False):
        """Align an iterable of batches ([(samples, text, language)] each),
        yielding one align_batch result list per batch, in order.

        The host work of neighbouring batches overlaps the device pass:
        while batch k runs on the GPU, batch k+1's words are split and
        tokenised, its audio and ids staged and its pass queued behind batch
        k (the library holds two batches between stage and fetch), and batch
        k-1's timestamps are repaired and paired with words.  Every batch's
        inputs are still copied to the device and its results read back."""
        def build(batch):
            batch = list(batch)
            return batch, self.build_inputs(batch)

        def post(inputs, raws):
            return self._items(inputs, raws, want_logits or want_normed)

        it = iter(batches)
        pending = []  # (inputs, staged) of batches run but not yet fetched, oldest first
        nxt = next(it, None)
        if nxt is None:
            return
        batch, inputs = build(nxt)
        pending.append((inputs, self.stage([c[0] for c in batch], inputs, want_logits, want_normed)))
        self.run()
        while pending:
            nxt = next(it, None)
            if nxt is not None:
                # built and staged while the previous batch runs; its uploads
                # and kernels queue behind that batch's on the stream
                batch, inputs = build(nxt)
                pending.append((inputs, self.stage([c[0] for c in batch], inputs, want_logits,
                                                   want_normed)))
                self.run()
            done_inputs, staged = pending.pop(0)
            raws = self.fetch(staged)
            yield post(done_inputs, raws)  # overlaps the next batch's device pass

    def align_inputs_stream(self, batches):
        """align_stream for batches whose inputs are already built: an iterable
        of (samples_list, inputs) pairs, yielding [(raw_ms, items)] per batch in
        order, with the same two-deep overlap of host work and device passes."""
        it = iter(batches)
        pending = []  # (inputs, staged), oldest first
        nxt = next(it, None)
        if nxt is None:
            return
        pending.append((nxt[1], self.stage(nxt[0], nxt[1])))
        self.run()
        while pending:
            nxt = next(it, None)
            if nxt is not None:
                pending.append((nxt[1], self.stage(nxt[0], nxt[1])))
                self.run()
            done_inputs, staged = pending.pop(0)
            yield self._items(done_inputs, self.fetch(staged), False)

    def align_inputs(self, samples_list, inputs, want_logits=False, want_normed=False):
        """The device-resident batched call on prebuilt inputs: [(raw_ms, extra)]."""
        b = self.stage(samples_list, inputs, want_logits, want_normed)
        self.run()
        return self.fetch(b)

    def stage(self, samples_list, inputs, want_logits=False, want_normed=False):
        """qa_batch_stage: plan the batch and copy its inputs to the device."""
        n = len(inputs)
        L = _lib.lib()
        clips = (_lib.QaClip * n)()
        res = (_lib.QaResult * n)()
        keep, outs = [], []
        lh_on = self.local_head_enabled()
        for i, (s, inp) in enumerate(zip(samples_list, inputs)):
            s = np.ascontiguousarray(s, np.float32)
            ids = np.ascontiguousarray(inp.input_ids, np.uint32)
            n_ts = len(inp.timestamp_positions)
            raw = np.zeros(n_ts, np.int64)
            lg = np.zeros((n_ts, self.cfg.num_labels), np.float32) if want_logits else None
            nm = np.zeros((n_ts, self.cfg.hidden_size), np.float32) if want_normed else None
            iv = np.zeros((n_ts // 2, 2), np.float64) if lh_on else None
            keep += [s, ids]
            clips[i].samples = s.ctypes.data
            clips[i].n_samples = len(s)
            clips[i].input_ids = ids.ctypes.data
            clips[i].seq_len = len(ids)
            res[i].raw_ms = raw.ctypes.data
            res[i].n_ts = n_ts
            res[i].logits = lg.ctypes.data if lg is not None else None
            res[i].normed = nm.ctypes.data if nm is not None else None
            res[i].intervals = iv.ctypes.data if iv is not None else None
            outs.append((raw, {"logits": lg, "normed": nm, "intervals": iv}))
        self._check(L.qa_batch_stage(self._ctx, ctypes.addressof(clips), n,
                                     ctypes.addressof(res)))
        return (clips, res, keep, outs)

    def run(self) -> None:
        """qa_batch_run: enqueue the device pass over the staged batch (no wait)."""
        self._check(_lib.lib().qa_batch_run(self._ctx))

    def fetch(self, staged):
        """qa_batch_fetch: copy the staged batch's results back: [(raw_ms, extra)]."""
        clips, res, keep, outs = staged
        L = _lib.lib()
        self._check(L.qa_batch_fetch(self._ctx, ctypes.addressof(res)))
        t = _lib.QaTimings()
        L.qa_get_timings(self._ctx, ctypes.byref(t))
        self.timings = {k: getattr(t, k) for k, _ in _lib.QaTimings._fields_}
        return outs

    def set_stream(self, stream) -> None:
        """Launch on a caller's cudaStream_t (an int handle; None = own stream)."""
        self._check(_lib.lib().qa_set_stream(self._ctx, stream))

    def set_profile(self, on: bool) -> None:
        self._check(_lib.lib().qa_set_profile(self._ctx, 1 if on else 0))

    def profile(self) -> dict:
        """Per kernel class: launches, total_ms, flops, bytes (qa_get_profile)."""
        L = _lib.lib()
        n = ctypes.c_int(0)
        self._check(L.qa_get_profile(self._ctx, None, 0, ctypes.byref(n)))
        arr = (_lib.QaKernelStat * max(n.value, 1))()
        self._check(L.qa_get_profile(self._ctx, ctypes.addressof(arr), n.value, ctypes.byref(n)))
        return {arr[i].name.decode(): {"launches": arr[i].launches, "total_ms": arr[i].total_ms,
                                       "flops": arr[i].flops, "bytes": arr[i].bytes}
                for i in range(n.value)}

    # ------------------------------------------------------------ stages

    def mel(self, samples: np.ndarray) -> np.ndarray:
        """mel::mel_features: [128, n/160] f32."""
        s = np.ascontiguousarray(samples, np.float32)
        frames = len(s) // 160
        out = np.zeros((128, max(frames, 1)), np.float32)
        nf = ctypes.c_int(0)
        self._check(_lib.lib().qa_mel(self._ctx, s.ctypes.data, len(s), out.ctypes.data,
                                      out.size, ctypes.byref(nf)))
        return out[:, :nf.value] if nf.value != out.shape[1] else out

    def audio_embeds(self, mel: np.ndarray) -> np.ndarray:
        """Backend::audio_embeds: [128, valid] -> [n_audio, 1024] 16-bit bits (uint16)."""
        mel = np.ascontiguousarray(mel, np.float32)
        valid = mel.shape[1]
        na = synth.audio_token_count(valid, self.cfg.n_window)
        out = np.zeros((na, self.cfg.output_dim), np.uint16)
        self._check(_lib.lib().qa_audio_embeds(self._ctx, mel.ctypes.data, mel.shape[0], valid,
                                               out.ctypes.data, out.size))
        return out

    def ensure_capacity(self, need: int) -> int:
        cap = ctypes.c_int(0)
        self._check(_lib.lib().qa_ensure_capacity(self._ctx, int(need), ctypes.byref(cap)))
        return cap.value

    def text_hidden(self, emb_bits: np.ndarray) -> np.ndarray:
        """Backend::text_hidden: [seq, 1024] 16-bit bits -> [seq, 1024] f32."""
        e = np.ascontiguousarray(emb_bits, np.uint16)
        out = np.zeros((e.shape[0], self.cfg.hidden_size), np.float32)
        self._check(_lib.lib().qa_text_hidden(self._ctx, e.ctypes.data, e.shape[0],
                                              out.ctypes.data))
        return out

    def head(self, hidden: np.ndarray, rows, want_logits=True, want_normed=False):
        """Final norm + timestamp head + argmax on `rows` of f32 `hidden`."""
        h = np.ascontiguousarray(hidden, np.float32)
        r = np.ascontiguousarray(rows, np.int32)
        raw = np.zeros(len(r), np.int64)
        lg = np.zeros((len(r), self.cfg.num_labels), np.float32) if want_logits else None
        nm = np.zeros((len(r), self.cfg.hidden_size), np.float32) if want_normed else None
        self._check(_lib.lib().qa_head(self._ctx, h.ctypes.data, h.shape[0], r.ctypes.data,
                                       len(r), raw.ctypes.data,
                                       lg.ctypes.data if lg is not None else None,
                                       nm.ctypes.data if nm is not None else None))
        return raw, lg, nm
