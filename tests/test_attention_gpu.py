"""Paged causal GQA attention kernels against a torch fp32 reference.

The decoder prefill's attention (src/cpu_decoder.rs:327-412): for each clip,
query position p and head h, softmax(q·kᵀ / sqrt(128)) over keys 0..=p of the
same clip, times v, with K/V head h // 2 (16 query heads, 8 K/V heads).  K/V
live in 64-token pages named by a per-clip block table.  The persistent
tcgen05/TMEM kernel is checked on ragged clip lengths (1, one page minus one, exactly one page, one page plus one, many
pages) with the pages shuffled and the rows past each clip's end holding
finite garbage.
"""
import numpy as np
import pytest

from conftest import cuda_ok, pkg

NQ, NKV, HD, PAGE = 16, 8, 128, 64
TOL = 2e-2  # max-abs error relative to the largest reference value (16-bit output)


def _tiles(lens, step):
    tiles, tok0 = [], 0
    for c, n in enumerate(lens):
        for q0 in range(0, n, step):
            tiles.append((c, q0, tok0, n))
        tok0 += n
    tiles.sort(key=lambda t: -t[1])
    import torch
    return torch.tensor(tiles, dtype=torch.int32)


def _case(lens, dtype, seed):
    import torch
    g = torch.Generator().manual_seed(seed)
    T = sum(lens)
    ldq = (NQ + 2 * NKV) * HD
    qkv = (torch.randn(T, ldq, generator=g) * 2.0).to(dtype)
    pages_per = [(n + PAGE - 1) // PAGE for n in lens]
    n_pages = sum(pages_per) + 3
    perm = torch.randperm(n_pages, generator=g)
    kpool = (torch.randn(n_pages, NKV, PAGE, HD, generator=g) * 2.0).to(dtype)
    vpool = torch.randn(n_pages, NKV, PAGE, HD, generator=g).to(dtype)
    max_pages = max(pages_per)
    bt = torch.zeros(len(lens), max_pages, dtype=torch.int32)
    k = 0
    for c, n in enumerate(lens):
        for i in range(pages_per[c]):
            bt[c, i] = int(perm[k])
            k += 1
    return qkv, kpool, vpool, bt, _tiles(lens, 64), lens


def _reference(qkv, kpool, vpool, bt, lens):
    import torch
    q_all = qkv.float()
    out = torch.zeros(qkv.shape[0], NQ * HD, device=qkv.device)
    tok0 = 0
    for c, n in enumerate(lens):
        pages = bt[c, : (n + PAGE - 1) // PAGE].long()
        k = kpool[pages].float().permute(1, 0, 2, 3).reshape(NKV, -1, HD)[:, :n]
        v = vpool[pages].float().permute(1, 0, 2, 3).reshape(NKV, -1, HD)[:, :n]
        q = q_all[tok0: tok0 + n, : NQ * HD].reshape(n, NQ, HD).permute(1, 0, 2)
        kk = k.repeat_interleave(NQ // NKV, dim=0)
        vv = v.repeat_interleave(NQ // NKV, dim=0)
        s = q @ kk.transpose(1, 2) / np.sqrt(HD)
        s = s.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool, device=s.device), 1), float("-inf"))
        o = torch.softmax(s, dim=-1) @ vv
        out[tok0: tok0 + n] = o.permute(1, 0, 2).reshape(n, NQ * HD)
        tok0 += n
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("dtype_name", ["f16", "bf16"])
@pytest.mark.parametrize("lens", [[1, 63, 64, 65], [130, 700, 2100], [4097]])
def test_paged_attention_matches_fp32(dtype_name, lens):
    if not cuda_ok():
        pytest.skip("no CUDA device")
    import torch
    L = pkg()._lib
    dtype = torch.float16 if dtype_name == "f16" else torch.bfloat16
    qkv, kpool, vpool, bt, tiles, lens = _case(lens, dtype, seed=len(lens) * 7 + sum(lens))
    dev = torch.device("cuda:0")
    d = [t.to(dev) for t in (qkv, kpool, vpool, bt)]
    ref = _reference(d[0], d[1], d[2], bt, lens).cpu()
    t = _tiles(lens, 128).to(dev)
    out = torch.full((qkv.shape[0], NQ * HD), float("nan"), dtype=dtype, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    L.causal_attention(d[0], NQ, NKV, tiles=t, block_tab=d[3], kpool=d[1], vpool=d[2],
                       out=out, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    o = out.float().cpu()
    assert torch.isfinite(o).all(), "rows left unwritten or non-finite"
    err = (o - ref).abs().max().item() / ref.abs().max().item()
    assert err <= TOL, f"rel err {err:.3e}"


@pytest.mark.parametrize("lens", [[1, 63, 64, 65], [130, 700, 2100], [4097]])
def test_attention_cases_pass_host_checks(lens):
    """CPU: the cases above are well formed, and swapped or out-of-range ones are not."""
    import torch
    L = pkg()._lib
    qkv, kpool, vpool, bt, tiles, lens = _case(lens, torch.float16, seed=1)
    out = torch.empty(qkv.shape[0], NQ * HD, dtype=torch.float16)
    L.check_attention_args(qkv, NQ, NKV, tiles, bt, kpool, vpool, out)
    with pytest.raises(ValueError):
        L.check_attention_args(qkv, NQ, NKV, bt, tiles, kpool, vpool, out)
    bad = bt.clone()
    bad[0, 0] = kpool.shape[0]
    with pytest.raises(ValueError):
        L.check_attention_args(qkv, NQ, NKV, tiles, bad, kpool, vpool, out)
    bad_t = tiles.clone()
    bad_t[0, 2] = qkv.shape[0]
    with pytest.raises(ValueError):
        L.check_attention_args(qkv, NQ, NKV, bad_t, bt, kpool, vpool, out)


@pytest.mark.gpu
def test_attention_rejects_bad_arguments():
    if not cuda_ok():
        pytest.skip("no CUDA device")
    import torch
    L = pkg()._lib
    dev = torch.device("cuda:0")
    qkv = torch.zeros(4, 4096, dtype=torch.float16, device=dev)
    pool = torch.zeros(1, NKV, PAGE, HD, dtype=torch.float16, device=dev)
    bt = torch.zeros(1, 1, dtype=torch.int32, device=dev)
    tiles = torch.tensor([[0, 0, 0, 4]], dtype=torch.int32, device=dev)
    out = torch.zeros(4, NQ * HD, dtype=torch.float16, device=dev)
    # a GQA group other than two is refused by the kernel's launcher
    out8 = torch.zeros(4, NKV * HD, dtype=torch.float16, device=dev)
    with pytest.raises(L.QaError):
        L.causal_attention(qkv, NKV, NKV, tiles=tiles, block_tab=bt, kpool=pool, vpool=pool,
                           out=out8, validate=False)
    # swapped tiles / block table are caught on the host, before any launch
    with pytest.raises(ValueError):
        L.causal_attention(qkv, NQ, NKV, tiles=bt, block_tab=tiles, kpool=pool, vpool=pool,
                           out=out)
