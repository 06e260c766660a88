"""The audio tower's windowed attention kernel against a torch fp32 reference.

src/audio_encoder.rs:574-627: the packed audio tokens are cut into windows of
at most 104 tokens (the last window of a clip is short); every query attends to
every key of its own window with a full softmax of q·kᵀ / sqrt(64), per head
(14 heads of 64).  The kernel runs on the tcgen05 tensor cores with S and P in
TMEM.  The cases cover windows of 1 token, short last windows, exactly 104
tokens, the 128-token maximum, a window ending at the last row of the buffer,
and the checkpoint's 16-head width, in f16 and bf16.
"""
import numpy as np
import pytest

from conftest import cuda_ok, pkg

HD = 64
TOL = 2e-2  # max-abs error relative to the largest reference value (16-bit output)


def _windows(clip_tokens, window):
    """(start, len) windows of consecutive clips packed back to back."""
    out, t0 = [], 0
    for n in clip_tokens:
        for st in range(0, n, window):
            out.append((t0 + st, min(window, n - st)))
        t0 += n
    return out, t0


def _reference(qkv, nh, windows):
    import torch
    T = qkv.shape[0]
    dm = nh * HD
    x = qkv.float()
    out = torch.zeros(T, dm, device=qkv.device)
    for st, n in windows:
        q = x[st:st + n, :dm].reshape(n, nh, HD).permute(1, 0, 2)
        k = x[st:st + n, dm:2 * dm].reshape(n, nh, HD).permute(1, 0, 2)
        v = x[st:st + n, 2 * dm:].reshape(n, nh, HD).permute(1, 0, 2)
        p = torch.softmax(q @ k.transpose(1, 2) / np.sqrt(HD), dim=-1)
        out[st:st + n] = (p @ v).permute(1, 0, 2).reshape(n, dm)
    return out


CASES = [
    (14, [1, 13, 104, 105, 208, 250], 104),   # 1-token clip, short tails, exact windows
    (14, [1300, 37], 104),                    # many full windows + a short tail
    (16, [500, 3], 104),                      # the checkpoint's 16-head tower
    (14, [256, 129], 128),                    # the 128-token maximum
]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype_name", ["f16", "bf16"])
@pytest.mark.parametrize("nh,clips,window", CASES)
def test_window_attention_matches_fp32(dtype_name, nh, clips, window):
    if not cuda_ok():
        pytest.skip("no CUDA device")
    import torch
    L = pkg()._lib
    dtype = torch.float16 if dtype_name == "f16" else torch.bfloat16
    wins, T = _windows(clips, window)
    g = torch.Generator().manual_seed(T + nh)
    qkv = (torch.randn(T, 3 * nh * HD, generator=g) * 2.0).to(dtype).cuda()
    w = torch.tensor(wins, dtype=torch.int32).cuda()
    out = torch.full((T, nh * HD), float("nan"), dtype=dtype, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.window_attention(qkv, nh, w, out, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = _reference(qkv, nh, wins).cpu()
    o = out.float().cpu()
    assert torch.isfinite(o).all(), "rows left unwritten or non-finite"
    err = (o - ref).abs().max().item() / ref.abs().max().item()
    assert err <= TOL, f"rel err {err:.3e}"
    # every row is its own window's: a window of one token returns its own v row
    for st, n in wins:
        if n == 1:
            v = qkv[st, 2 * nh * HD:].float().cpu()
            assert torch.allclose(o[st], v, rtol=1e-2, atol=1e-2)


@pytest.mark.gpu
def test_window_attention_skips_rows_outside_windows():
    """Rows that no window names are left as they were (the kernel writes only
    the rows of its windows, whatever its 128-row tiles read)."""
    if not cuda_ok():
        pytest.skip("no CUDA device")
    import torch
    L = pkg()._lib
    nh, T = 14, 300
    qkv = torch.randn(T, 3 * nh * HD).half().cuda()
    wins = [(10, 104), (150, 40)]
    w = torch.tensor(wins, dtype=torch.int32).cuda()
    out = torch.full((T, nh * HD), 7.0, dtype=torch.float16, device="cuda")
    L.window_attention(qkv, nh, w, out)
    torch.cuda.synchronize()
    o = out.float().cpu()
    keep = torch.ones(T, dtype=torch.bool)
    for st, n in wins:
        keep[st:st + n] = False
    assert (o[keep] == 7.0).all()
    ref = _reference(qkv, nh, wins).cpu()
    assert (o[~keep] - ref[~keep]).abs().max().item() / ref.abs().max().item() <= TOL


def test_window_attention_host_checks():
    """CPU: malformed windows and shapes are refused before any launch."""
    import torch
    L = pkg()._lib
    nh, T = 14, 64
    qkv = torch.zeros(T, 3 * nh * HD, dtype=torch.float16)
    out = torch.zeros(T, nh * HD, dtype=torch.float16)
    for bad in ([(0, 65)], [(60, 10)], [(0, 0)], [(-1, 4)], [(0, 129)]):
        with pytest.raises(ValueError):
            L.window_attention(qkv, nh, torch.tensor(bad, dtype=torch.int32), out)
    with pytest.raises(ValueError):
        L.window_attention(qkv, nh, torch.tensor([(0, 8)], dtype=torch.int32), out[:, :64])
