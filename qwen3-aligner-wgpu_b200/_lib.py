"""ctypes binding of libqa_b200.so (the C ABI in include/qa_b200.h and
include/qa_b200_kernels.h).

The library is built in-tree by ``make`` in this directory (see
``__graft_entry__.build``).  There is no fallback: if the shared object is
missing, :func:`lib` raises, so a product path can never silently run on the
CPU.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqa_b200.so")

QA_OK = 0
QA_ERR_SHAPE = 1
QA_ERR_CAP = 2
QA_ERR_CUDA = 3
QA_ERR_OOM = 4
QA_ERR_TIMEOUT = 5
QA_ERR_STATE = 6
QA_ERR_WEIGHTS = 7
QA_ERR_ARG = 8

ERR_NAMES = {
    QA_ERR_SHAPE: "QA_ERR_SHAPE",
    QA_ERR_CAP: "QA_ERR_CAP",
    QA_ERR_CUDA: "QA_ERR_CUDA",
    QA_ERR_OOM: "QA_ERR_OOM",
    QA_ERR_TIMEOUT: "QA_ERR_TIMEOUT",
    QA_ERR_STATE: "QA_ERR_STATE",
    QA_ERR_WEIGHTS: "QA_ERR_WEIGHTS",
    QA_ERR_ARG: "QA_ERR_ARG",
}

QA_HALF_F16 = 0
QA_HALF_BF16 = 1
QA_DTYPE_F32 = 0
QA_DTYPE_F16 = 1
QA_DTYPE_BF16 = 2

EPI_STORE16 = 0
EPI_RESID16 = 1
EPI_RESID32 = 2
EPI_SWIGLU16 = 3
EPI_STORE32 = 4
EPI_ARGMAX = 5
ACT_NONE = 0
ACT_GELU = 1

# Every symbol the two public headers declare; tests check each is exported.
EXPORTED = [
    "qa_open", "qa_load", "qa_close", "qa_last_error", "qa_set_timeout_ms", "qa_half",
    "qa_get_timings", "qa_mel", "qa_audio_embeds", "qa_ensure_capacity", "qa_text_hidden",
    "qa_head", "qa_align_batch", "qa_batch_stage", "qa_batch_run", "qa_batch_fetch",
    "qa_set_stream", "qa_set_profile", "qa_get_profile", "qa_fix_timestamps",
    "qa_decode_wav", "qa_resampled_length", "qa_resample",
    "qa_head_noalloc", "qa_probe_timeout", "qa_local_head_load", "qa_set_local_head_enabled",
    "qa_local_head_enabled", "qa_local_head_refine",
    "qa_k_gemm", "qa_k_conv3x3s2", "qa_k_causal_attention", "qa_k_window_attention",
    "qa_k_conv1", "qa_k_gemm_qkv_rope",
]

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_ll = ctypes.c_longlong


class QaTensor(ctypes.Structure):
    """qa_tensor (include/qa_b200.h)."""
    _fields_ = [("name", ctypes.c_char_p), ("dtype", c_int), ("ndim", c_int),
                ("shape", ctypes.c_int64 * 4), ("data", c_void_p)]


class QaCfg(ctypes.Structure):
    """qa_cfg (include/qa_b200.h)."""
    _fields_ = [(n, c_int) for n in (
        "d_model", "encoder_layers", "encoder_heads", "encoder_ffn_dim", "num_mel_bins",
        "downsample_hidden", "max_source_positions", "n_window", "n_window_infer", "output_dim",
        "vocab_size", "hidden_size", "intermediate_size", "num_layers", "num_heads",
        "num_kv_heads", "head_dim")] + [("rms_norm_eps", ctypes.c_double),
                                       ("rope_theta", ctypes.c_double)] + [
        (n, c_int) for n in ("num_labels", "timestamp_token_id", "audio_token_id")] + [
        ("timestamp_segment_time_ms", ctypes.c_double), ("max_seq", c_int)]


class QaTimings(ctypes.Structure):
    _fields_ = [(n, ctypes.c_double) for n in (
        "h2d_ms", "mel_ms", "enc_ms", "gather_ms", "prefill_ms", "head_ms", "d2h_ms",
        "total_ms")] + [("gpu_launches", ctypes.c_int64), ("h2d_bytes", ctypes.c_int64),
                        ("d2h_bytes", ctypes.c_int64), ("local_ms", ctypes.c_double)]


class QaKernelStat(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", ctypes.c_int64),
                ("total_ms", ctypes.c_double), ("flops", ctypes.c_double),
                ("bytes", ctypes.c_double)]


class QaClip(ctypes.Structure):
    _fields_ = [("samples", c_void_p), ("n_samples", ctypes.c_int64), ("input_ids", c_void_p),
                ("seq_len", c_int)]


class QaResult(ctypes.Structure):
    _fields_ = [("raw_ms", c_void_p), ("n_ts", c_int), ("logits", c_void_p),
                ("normed", c_void_p), ("intervals", c_void_p)]


def make_cfg(mc) -> QaCfg:
    """QaCfg from a synth.ModelConfig-like object."""
    c = QaCfg()
    for name, _ in QaCfg._fields_:
        setattr(c, name, getattr(mc, name))
    return c


def make_tensors(weights: dict):
    """(QaTensor array, keepalive) from name -> (dtype, np array) or bf16 bits."""
    import numpy as np
    items = []
    for name, v in weights.items():
        if isinstance(v, tuple):
            dt, arr = v
        else:
            dt, arr = "BF16", v
        code = {"BF16": QA_DTYPE_BF16, "F16": QA_DTYPE_F16, "F32": QA_DTYPE_F32}[dt]
        arr = np.ascontiguousarray(arr)
        items.append((name.encode(), code, arr))
    arr_t = (QaTensor * len(items))()
    for i, (nm, code, a) in enumerate(items):
        arr_t[i].name = nm
        arr_t[i].dtype = code
        arr_t[i].ndim = a.ndim
        for d in range(a.ndim):
            arr_t[i].shape[d] = a.shape[d]
        arr_t[i].data = a.ctypes.data
    return arr_t, items


class QaError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, code: int, msg: str = ""):
        self.code = code
        super().__init__(f"{ERR_NAMES.get(code, code)}: {msg}")


_lock = threading.Lock()
_lib = None


def lib_exists() -> bool:
    return os.path.exists(LIB_PATH)


def lib() -> ctypes.CDLL:
    """Load (once) and return the shared library; raise if it was not built."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `make` in {_HERE} "
                    "(or __graft_entry__.build()); there is no CPU fallback")
            L = ctypes.CDLL(LIB_PATH)
            _declare(L)
            _lib = L
        return _lib


def _declare(L: ctypes.CDLL) -> None:
    L.qa_k_gemm.argtypes = [c_void_p, c_ll, c_void_p, c_ll, c_int, c_int, c_int, c_int, c_int,
                            c_int, c_void_p, c_ll, c_void_p, c_void_p, c_void_p, c_int, c_void_p,
                            c_void_p, c_int, c_void_p]
    L.qa_k_gemm.restype = c_int
    L.qa_k_conv3x3s2.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_int,
                                 c_int, c_int, c_int, c_void_p, c_ll, c_void_p, c_void_p, c_void_p]
    L.qa_k_gemm_qkv_rope.argtypes = [c_void_p, c_ll, c_void_p, c_ll, c_int, c_int, c_int, c_int,
                                     c_void_p, c_ll, c_void_p, c_void_p, c_void_p, c_int,
                                     c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     ctypes.c_float, c_int, c_int, c_void_p, c_int, c_void_p]
    L.qa_k_conv1.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p,
                             c_int, c_void_p]
    L.qa_k_causal_attention.argtypes = [c_void_p, c_ll, c_ll, c_int, c_int, c_void_p, c_int,
                                        c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p,
                                        c_int, c_void_p, c_void_p]
    L.qa_k_window_attention.argtypes = [c_void_p, c_ll, c_int, c_int, c_void_p, c_int, c_int,
                                        c_void_p, c_int, c_void_p, c_void_p]
    if hasattr(L, "qa_open"):
        L.qa_open.argtypes = [c_int, c_int, ctypes.POINTER(c_void_p)]
        L.qa_load.argtypes = [c_void_p, c_void_p, c_int, c_void_p]
        L.qa_close.argtypes = [c_void_p]
        L.qa_last_error.argtypes = [c_void_p]
        L.qa_last_error.restype = ctypes.c_char_p
        L.qa_set_timeout_ms.argtypes = [c_void_p, c_int]
        L.qa_half.argtypes = [c_void_p]
        L.qa_get_timings.argtypes = [c_void_p, c_void_p]
        L.qa_mel.argtypes = [c_void_p, c_void_p, ctypes.c_int64, c_void_p, ctypes.c_int64,
                             ctypes.POINTER(c_int)]
        L.qa_audio_embeds.argtypes = [c_void_p, c_void_p, c_int, c_int, c_void_p, ctypes.c_int64]
        L.qa_ensure_capacity.argtypes = [c_void_p, c_int, ctypes.POINTER(c_int)]
        L.qa_text_hidden.argtypes = [c_void_p, c_void_p, c_int, c_void_p]
        L.qa_head.argtypes = [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                              c_void_p]
        L.qa_align_batch.argtypes = [c_void_p, c_void_p, c_int, c_void_p]
        L.qa_batch_stage.argtypes = [c_void_p, c_void_p, c_int, c_void_p]
        L.qa_fix_timestamps.argtypes = [c_void_p, c_int, c_void_p]
        L.qa_decode_wav.argtypes = [c_void_p, ctypes.c_int64, c_void_p, ctypes.c_int64,
                                    ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(c_int),
                                    ctypes.POINTER(c_int)]
        L.qa_resampled_length.argtypes = [ctypes.c_int64, c_int, c_int]
        L.qa_resampled_length.restype = ctypes.c_int64
        L.qa_resample.argtypes = [c_void_p, ctypes.c_int64, c_int, c_int, c_void_p,
                                  ctypes.c_int64]
        L.qa_head_noalloc.argtypes = [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p,
                                      c_void_p]
        L.qa_probe_timeout.argtypes = [c_void_p, c_int]
        L.qa_batch_run.argtypes = [c_void_p]
        L.qa_batch_fetch.argtypes = [c_void_p, c_void_p]
        L.qa_set_stream.argtypes = [c_void_p, c_void_p]
        L.qa_set_profile.argtypes = [c_void_p, c_int]
        L.qa_get_profile.argtypes = [c_void_p, c_void_p, c_int, ctypes.POINTER(c_int)]
        L.qa_local_head_load.argtypes = [c_void_p, c_void_p, c_int, c_void_p, c_void_p]
        L.qa_set_local_head_enabled.argtypes = [c_void_p, c_int]
        L.qa_local_head_enabled.argtypes = [c_void_p]
        L.qa_local_head_refine.argtypes = [c_void_p, c_void_p, ctypes.c_int64, c_int, c_void_p,
                                           c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                           c_void_p]


def check(rc: int, ctx=None) -> None:
    if rc != QA_OK:
        msg = ""
        if ctx is not None:
            m = lib().qa_last_error(ctx)
            msg = m.decode() if m else ""
        raise QaError(rc, msg)


def fix_timestamps(raw) -> list:
    """qa_fix_timestamps over an int64 sequence (the compiled LIS repair)."""
    import numpy as np
    a = np.ascontiguousarray(raw, np.int64)
    out = np.empty_like(a)
    if len(a):
        check(lib().qa_fix_timestamps(a.ctypes.data, len(a), out.ctypes.data))
    return out.tolist()


def ptr(t) -> int:
    """Device/host address of a torch tensor (0 for None)."""
    return 0 if t is None else int(t.data_ptr())


def gemm(A, B, out, mode=EPI_STORE16, act=ACT_NONE, bias=None, row_map=None, pe=None,
         pe_period=1, keys=None, status=None, force_bn=0, stream=None):
    """Run the tcgen05 GEMM on torch CUDA tensors: A [M, K], B [N, K]."""
    import torch
    M, K = A.shape
    N = B.shape[0]
    assert B.shape[1] == K and A.dtype == B.dtype
    bf16 = 1 if A.dtype == torch.bfloat16 else 0
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    rc = lib().qa_k_gemm(ptr(A), A.stride(0), ptr(B), B.stride(0), M, N, K, bf16, mode, act,
                         ptr(out), out.stride(0) if out is not None else 0, ptr(bias),
                         ptr(row_map), ptr(pe), pe_period, ptr(keys), ptr(status), force_bn, s)
    check(rc)


def conv3x3s2(x, wt, out, time_major=False, mode=EPI_STORE16, act=ACT_NONE, bias=None,
              status=None, stream=None):
    """Implicit-GEMM conv on torch CUDA tensors: x [n, h, w, c] NHWC, wt [c_out, 9c]."""
    import torch
    n, h, w, c = x.shape
    bf16 = 1 if x.dtype == torch.bfloat16 else 0
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    rc = lib().qa_k_conv3x3s2(ptr(x), n, h, w, c, ptr(wt), wt.shape[0], 1 if time_major else 0,
                              bf16, mode, act, ptr(out), out.stride(0), ptr(bias), ptr(status), s)
    check(rc)


def causal_attention(qkv, nqh, nkvh, tiles, block_tab, kpool, vpool, out, status=None,
                     stream=None, validate=True):
    """Paged causal attention on torch CUDA tensors.

    qkv [T, ldq] 16-bit, tiles int32 [n, 4] (clip, q0, tok0, len), block_tab
    int32 [clips, max_pages], kpool/vpool [pages, nkvh, 64, 128], out [T, nqh*128].
    """
    import torch
    if validate:  # copies tiles and block_tab to the host
        check_attention_args(qkv, nqh, nkvh, tiles, block_tab, kpool, vpool, out)
    bf16 = 1 if qkv.dtype == torch.bfloat16 else 0
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    rc = lib().qa_k_causal_attention(ptr(qkv), qkv.stride(0), qkv.shape[0], nqh, nkvh,
                                     ptr(tiles), tiles.shape[0], ptr(block_tab),
                                     block_tab.shape[1], ptr(kpool), ptr(vpool), kpool.shape[0],
                                     ptr(out), bf16, ptr(status), s)
    check(rc)


def window_attention(qkv, nh, windows, out, status=None, stream=None, max_window=None):
    """Windowed attention on torch CUDA tensors: qkv [T, 3*64*nh] 16-bit,
    windows int32 [n, 2] (first token, length), out [T, 64*nh].  The windows
    are range-checked on the host (a copy to the host) unless `max_window`
    (the longest window) is given, which a caller that checked them passes."""
    import torch
    T = qkv.shape[0]
    dm = 64 * nh
    if (qkv.dim() != 2 or qkv.shape[1] != 3 * dm or tuple(out.shape) != (T, dm)
            or qkv.dtype != out.dtype or windows.dtype != torch.int32 or windows.dim() != 2
            or windows.shape[1] != 2):
        raise ValueError("qkv [T, 3*64*nh], out [T, 64*nh] of one dtype, windows int32 [n, 2]")
    if max_window is None:
        w = windows.cpu()
        if w.numel() and (int(w[:, 0].min()) < 0 or int(w[:, 1].min()) < 1
                          or int((w[:, 0] + w[:, 1]).max()) > T or int(w[:, 1].max()) > 128):
            raise ValueError("window (start, len) out of range")
        max_window = int(w[:, 1].max()) if w.numel() else 1
    bf16 = 1 if qkv.dtype == torch.bfloat16 else 0
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    check(lib().qa_k_window_attention(ptr(qkv), T, dm, nh, ptr(windows), windows.shape[0],
                                      max_window, ptr(out), bf16, ptr(status), s))


def check_attention_args(qkv, nqh, nkvh, tiles, block_tab, kpool, vpool, out) -> None:
    """Host-side shape and range checks for causal_attention (ValueError on failure)."""
    import torch
    T = qkv.shape[0]
    if (tiles.dim() != 2 or tiles.shape[1] != 4 or tiles.dtype != torch.int32
            or block_tab.dim() != 2 or block_tab.dtype != torch.int32):
        raise ValueError("tiles must be int32 [n, 4] and block_tab int32 [clips, max_pages]")
    if tuple(kpool.shape[1:]) != (nkvh, 64, 128) or kpool.shape != vpool.shape:
        raise ValueError("kpool/vpool must be [pages, nkvh, 64, 128]")
    if qkv.dim() != 2 or qkv.shape[1] < (nqh + 2 * nkvh) * 128 or tuple(out.shape) != (
            T, nqh * 128) or not (qkv.dtype == kpool.dtype == vpool.dtype == out.dtype):
        raise ValueError("qkv [T, >= (nqh + 2 nkvh) 128], out [T, nqh 128], one 16-bit dtype")
    t = tiles.cpu()
    bt = block_tab.cpu()
    if t.numel() and (int(t[:, 0].min()) < 0 or int(t[:, 0].max()) >= bt.shape[0]
                      or int(t[:, 1].min()) < 0 or int((t[:, 1] - t[:, 3]).max()) >= 0
                      or int((t[:, 2] + t[:, 3]).max()) > T
                      or int(t[:, 3].max()) > 64 * bt.shape[1]):
        raise ValueError("tile (clip, q0, tok0, len) out of range")
    if bt.numel() and (int(bt.min()) < 0 or int(bt.max()) >= kpool.shape[0]):
        raise ValueError("block_tab names a page outside the pools")


def conv1(mel, wt, bias, out, stream=None):
    """conv1 + bias + GELU on torch CUDA tensors: mel [n, h, w] f32 -> out [n*ho*wo, c_out]."""
    import torch
    n, h, w = mel.shape
    bf16 = 1 if out.dtype == torch.bfloat16 else 0
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    check(lib().qa_k_conv1(ptr(mel), n, h, w, ptr(wt), ptr(bias), wt.shape[0], ptr(out), bf16, s))


def gemm_qkv_rope(A, B, q_out, pos_of, clip_of, block_tab, kc, vc, cos_t, sin_t, qn, kn, eps,
                  nq, nkv, status=None, force_bn=0, stream=None):
    """The fused decoder QKV GEMM on torch CUDA tensors (see qa_k_gemm_qkv_rope)."""
    import torch
    M, K = A.shape
    N = B.shape[0]
    bf16 = 1 if A.dtype == torch.bfloat16 else 0
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    check(lib().qa_k_gemm_qkv_rope(ptr(A), A.stride(0), ptr(B), B.stride(0), M, N, K, bf16,
                                   ptr(q_out), q_out.stride(0), ptr(pos_of), ptr(clip_of),
                                   ptr(block_tab), block_tab.shape[1], ptr(kc), ptr(vc),
                                   ptr(cos_t), ptr(sin_t), ptr(qn), ptr(kn), eps, nq, nkv,
                                   ptr(status), force_bn, s))
