"""Kernel micro-benchmarks of the alignment path, on synthetic data on cuda:0.

    python qwen3-aligner-wgpu_b200/kbench.py gemm --m 16384 --n 6144 --k 1024 --mode swiglu
    python qwen3-aligner-wgpu_b200/kbench.py gemm --m 16384 --n 1024 --k 3072 --mode resid16
    python qwen3-aligner-wgpu_b200/kbench.py attention --clips 64
    python qwen3-aligner-wgpu_b200/kbench.py window --tokens 13813
    python qwen3-aligner-wgpu_b200/kbench.py conv --n 256 --h 64 --w 50 --c 480
    python qwen3-aligner-wgpu_b200/kbench.py conv1 --n 256 --h 128 --w 100 --c 480
    python qwen3-aligner-wgpu_b200/kbench.py qkv --clips 64
    python qwen3-aligner-wgpu_b200/kbench.py pass --clips 16 --iters 2

Each run times `--iters` launches with CUDA events on the launching stream
(after `--warmup` launches) and prints one JSON line with the mean launch time
and the achieved TFLOP/s.  Used for the ncu captures under profiles/ (one
kernel, a handful of launches, inputs larger than L2).

`attention` runs one decoder layer's paged causal attention over `--clips`
clips whose lengths are drawn uniformly from [--min-len, --max-len] tokens
(the batched 30 s workload's decoder clips average about 400 tokens), 16 query
and 8 K/V heads of 128, pages shuffled; FLOP/s counts the exact causal work.
"""
import argparse
import importlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["gemm", "attention", "window", "conv", "conv1", "qkv", "pass"])
    ap.add_argument("--h", type=int, default=64)
    ap.add_argument("--w", type=int, default=50)
    ap.add_argument("--c", type=int, default=480)
    ap.add_argument("--cout", type=int, default=0, help="conv output channels (0 = --c)")
    ap.add_argument("--time-major", action="store_true")
    ap.add_argument("--clips", type=int, default=64)
    ap.add_argument("--tokens", type=int, default=13813, help="window: packed audio tokens")
    ap.add_argument("--heads", type=int, default=14, help="window: heads of 64")
    ap.add_argument("--min-len", type=int, default=130)
    ap.add_argument("--max-len", type=int, default=750)
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=6144, help="gemm N, or images for conv")
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--act", default="none", choices=["none", "gelu"])
    ap.add_argument("--bn", type=int, default=0,
                    help="gemm tile: 0 = library choice, -1 = CTA-pair 256x256, >0 = one CTA, that width")
    ap.add_argument("--mode", default="store16",
                    choices=["store16", "resid16", "swiglu", "resid32", "store32", "argmax"])
    ap.add_argument("--dtype", default="f16", choices=["f16", "bf16"])
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()

    import torch
    qa = importlib.import_module("qwen3-aligner-wgpu_b200")
    L = qa._lib
    dt = torch.float16 if a.dtype == "f16" else torch.bfloat16
    if a.kernel == "attention":
        return attention(a, L, dt)
    if a.kernel == "window":
        return window(a, L, dt)
    if a.kernel == "pass":
        return whole_pass(a, qa)
    if a.kernel == "conv":
        return conv(a, L, dt)
    if a.kernel == "conv1":
        return conv1(a, L, dt)
    if a.kernel == "qkv":
        return qkv(a, L, dt)
    g = torch.Generator(device="cuda").manual_seed(0)
    A = (torch.randn(a.m, a.k, device="cuda", generator=g) * 0.5).to(dt)
    B = (torch.randn(a.n, a.k, device="cuda", generator=g) * 0.05).to(dt)
    mode = {"store16": L.EPI_STORE16, "resid16": L.EPI_RESID16, "swiglu": L.EPI_SWIGLU16,
            "resid32": L.EPI_RESID32, "store32": L.EPI_STORE32, "argmax": L.EPI_ARGMAX}[a.mode]
    out_cols = a.n // 2 if a.mode == "swiglu" else a.n
    out_dt = torch.float32 if a.mode in ("resid32", "store32", "argmax") else dt
    out = torch.zeros(a.m, out_cols, device="cuda", dtype=out_dt)
    keys = torch.zeros(a.m, dtype=torch.int64, device="cuda") if a.mode == "argmax" else None
    bn = a.bn
    act = L.ACT_GELU if a.act == "gelu" else L.ACT_NONE
    for _ in range(a.warmup):
        L.gemm(A, B, out, mode=mode, keys=keys, force_bn=bn, act=act)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        L.gemm(A, B, out, mode=mode, keys=keys, force_bn=bn, act=act)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.iters
    flops = 2.0 * a.m * a.n * a.k
    print(json.dumps({"kernel": "gemm_tc", "m": a.m, "n": a.n, "k": a.k, "mode": a.mode, "act": a.act, "bn": a.bn,
                      "dtype": a.dtype, "ms": ms, "tflops": flops / ms / 1e9,
                      "algorithmic_bytes": (a.m * a.k + a.n * a.k) * 2 + a.m * out_cols * out.element_size()}))


def attention(a, L, dt):
    import numpy as np
    import torch
    nq, nkv, hd, page = 16, 8, 128, 64
    rng = np.random.default_rng(0)
    lens = [int(x) for x in rng.integers(a.min_len, a.max_len + 1, a.clips)]
    T = sum(lens)
    pages_per = [(n + page - 1) // page for n in lens]
    n_pages = sum(pages_per)
    perm = rng.permutation(n_pages)
    bt = np.zeros((len(lens), max(pages_per)), dtype=np.int32)
    tiles, k, tok0 = [], 0, 0
    step = 128
    for c, n in enumerate(lens):
        bt[c, : pages_per[c]] = perm[k: k + pages_per[c]]
        k += pages_per[c]
        tiles += [(c, q0, tok0, n) for q0 in range(0, n, step)]
        tok0 += n
    # the runtime's order: longest clip first, a clip's blocks adjacent
    tiles.sort(key=lambda t: (-t[3], t[0], -t[1]))
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = (torch.randn(T, (nq + 2 * nkv) * hd, device=dev, generator=g)).to(dt)
    kpool = torch.randn(n_pages, nkv, page, hd, device=dev, generator=g).to(dt)
    vpool = torch.randn(n_pages, nkv, page, hd, device=dev, generator=g).to(dt)
    out = torch.empty(T, nq * hd, device=dev, dtype=dt)
    t = torch.tensor(tiles, dtype=torch.int32, device=dev)
    btd = torch.from_numpy(bt).to(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    L.check_attention_args(qkv, nq, nkv, t, btd, kpool, vpool, out)
    run = lambda: L.causal_attention(qkv, nq, nkv, tiles=t, block_tab=btd, kpool=kpool,
                                     vpool=vpool, out=out, status=status,
                                     validate=False)
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        run()
    e1.record()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ms = e0.elapsed_time(e1) / a.iters
    flops = sum(4.0 * hd * nq * 0.5 * n * (n + 1) for n in lens)
    print(json.dumps({"kernel": "causal_attention", "clips": a.clips,
                      "tokens": T, "items": len(tiles) * nkv, "dtype": a.dtype, "ms": ms,
                      "tflops": flops / ms / 1e9}))


def whole_pass(a, qa):
    """--iters batched passes (qa_batch_run) over the first --clips clips of
    BASELINE config 2 on the seeded model, staged once (for profiling the
    pass's kernels: the launches of pass k follow those of pass k-1)."""
    cfg = qa.synth.ModelConfig()
    al = qa.Aligner.load_backend_with_dtype(qa.synth.random_weights(cfg), a.dtype, cfg=cfg)
    clips = qa.synth.workload(2, n_clips=a.clips)
    inps = al.build_inputs([(c.samples, c.text, c.language) for c in clips])
    st = al.stage([c.samples for c in clips], inps)
    for _ in range(a.iters):
        al.run()
    al.fetch(st)
    print(json.dumps({"kernel": "pass", "clips": a.clips, "passes": a.iters,
                      "decoder_tokens": sum(i.seq_len() for i in inps),
                      "audio_tokens": sum(i.n_audio_tokens for i in inps),
                      "launches_per_pass": al.timings["gpu_launches"]}))
    al.close()


def window(a, L, dt):
    """The tower's windowed attention over `--tokens` packed audio tokens cut
    into clips of U(65, 390) tokens (5-30 s) and windows of 104, as the bench
    batch is.  Algorithmic bytes: the qkv rows read once and the output written
    once (L2 is flushed between launches by a 256 MiB write outside the timed
    events)."""
    import numpy as np
    import torch
    rng = np.random.default_rng(0)
    wins, t0 = [], 0
    while t0 < a.tokens:
        n = min(int(rng.integers(65, 391)), a.tokens - t0)
        for st in range(0, n, 104):
            wins.append((t0 + st, min(104, n - st)))
        t0 += n
    T, nh = a.tokens, a.heads
    dev = torch.device("cuda:0")
    qkv = torch.randn(T, 3 * 64 * nh, device=dev).to(dt)
    out = torch.empty(T, 64 * nh, device=dev, dtype=dt)
    w = torch.tensor(wins, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    L.window_attention(qkv, nh, w, out, status=status)  # checks the windows once
    run = lambda: L.window_attention(qkv, nh, w, out, status=status, max_window=104)
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(a.iters):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run()
        e1.record()
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    assert int(status.item()) == 0
    ms = tot / a.iters
    flops = sum(4.0 * n * n * 64 * nh for _, n in wins)
    nbytes = T * 4 * 64 * nh * qkv.element_size()
    print(json.dumps({"kernel": "window_attention", "tokens": T, "windows": len(wins),
                      "dtype": a.dtype, "ms": ms, "tflops": flops / ms / 1e9,
                      "gbs": nbytes / ms / 1e6}))


def conv(a, L, dt):
    """3x3 / stride 2 / pad 1 conv (+bias, GELU) over NHWC [n, h, w, c] -> c outputs."""
    import torch
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    co = a.cout or a.c
    x = (torch.randn(a.n, a.h, a.w, a.c, device=dev, generator=g) * 0.5).to(dt)
    wk = (torch.randn(co, 9 * a.c, device=dev, generator=g) * 0.02).to(dt)
    bias = torch.randn(co, device=dev, generator=g) * 0.1
    ho, wo = (a.h - 1) // 2 + 1, (a.w - 1) // 2 + 1
    out = torch.empty(a.n * ho * wo, co, device=dev, dtype=dt)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    run = lambda: L.conv3x3s2(x, wk, out, time_major=a.time_major, act=L.ACT_GELU, bias=bias,
                              status=st)
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        run()
    e1.record()
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    ms = e0.elapsed_time(e1) / a.iters
    flops = 2.0 * a.n * ho * wo * co * 9 * a.c
    print(json.dumps({"kernel": "conv3x3s2", "n": a.n, "h": a.h, "w": a.w, "c": a.c, "cout": co,
                      "time_major": a.time_major, "dtype": a.dtype, "ms": ms,
                      "tflops": flops / ms / 1e9}))


def conv1(a, L, dt):
    """First conv level: mel [n, h, w] f32 -> GELU(conv 1 -> c) NHWC 16-bit."""
    import torch
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    mel = torch.randn(a.n, a.h, a.w, device=dev, generator=g)
    wt = torch.randn(a.c, 9, device=dev, generator=g) * 0.3
    bias = torch.randn(a.c, device=dev, generator=g) * 0.1
    ho, wo = (a.h - 1) // 2 + 1, (a.w - 1) // 2 + 1
    out = torch.empty(a.n * ho * wo, a.c, device=dev, dtype=dt)
    run = lambda: L.conv1(mel, wt, bias, out)
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.iters
    nbytes = out.numel() * out.element_size() + mel.numel() * 4
    print(json.dumps({"kernel": "conv1", "n": a.n, "h": a.h, "w": a.w, "c": a.c, "dtype": a.dtype,
                      "ms": ms, "gbs": nbytes / ms / 1e6,
                      "outputs_per_s": out.numel() / ms * 1e3}))


def qkv(a, L, dt):
    """The decoder's fused QKV GEMM (q/k RMSNorm + RoPE + paged K/V append) over
    --clips clips of U(--min-len, --max-len) tokens, 16 q / 8 kv heads."""
    import numpy as np
    import torch
    nq, nkv, hd, H, page = 16, 8, 128, 1024, 64
    rng = np.random.default_rng(0)
    lens = [int(x) for x in rng.integers(a.min_len, a.max_len + 1, a.clips)]
    T = sum(lens)
    pages_per = [(n + page - 1) // page for n in lens]
    perm = rng.permutation(sum(pages_per))
    bt = np.zeros((len(lens), max(pages_per)), dtype=np.int32)
    pos = np.concatenate([np.arange(n) for n in lens]).astype(np.int32)
    clip = np.concatenate([np.full(n, c) for c, n in enumerate(lens)]).astype(np.int32)
    k = 0
    for c in range(len(lens)):
        bt[c, : pages_per[c]] = perm[k: k + pages_per[c]]
        k += pages_per[c]
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    A = torch.randn(T, H, device=dev, generator=g).to(dt)
    B = (torch.randn((nq + 2 * nkv) * hd, H, device=dev, generator=g) * 0.03).to(dt)
    q = torch.empty(T, (nq + 2 * nkv) * hd, device=dev, dtype=dt)
    kc = torch.zeros(sum(pages_per), nkv, page, hd, device=dev, dtype=dt)
    vc = torch.zeros_like(kc)
    ang = torch.arange(8192, device=dev)[:, None] * (1e6 ** (-torch.arange(64, device=dev) / 64))[None]
    cos_t, sin_t = torch.cos(ang).to(dt), torch.sin(ang).to(dt)
    qn = torch.rand(hd, device=dev, generator=g) + 0.5
    kn = torch.rand(hd, device=dev, generator=g) + 0.5
    t = lambda x: torch.from_numpy(x).to(dev)
    pos_d, clip_d, bt_d = t(pos), t(clip), t(bt)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    run = lambda: L.gemm_qkv_rope(A, B, q, pos_d, clip_d, bt_d, kc, vc, cos_t, sin_t, qn, kn, 1e-6,
                                  nq, nkv, status=st, force_bn=a.bn)
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        run()
    e1.record()
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    ms = e0.elapsed_time(e1) / a.iters
    flops = 2.0 * T * (nq + 2 * nkv) * hd * H
    print(json.dumps({"kernel": "gemm_qkv_rope", "tokens": T, "bn": a.bn, "dtype": a.dtype,
                      "ms": ms, "tflops": flops / ms / 1e9}))


if __name__ == "__main__":
    main()
