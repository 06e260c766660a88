"""Kernel micro-benchmarks of the alignment path, on synthetic data on cuda:0.

    python qwen3-aligner-wgpu_b200/kbench.py gemm --m 16384 --n 6144 --k 1024 --mode swiglu
    python qwen3-aligner-wgpu_b200/kbench.py gemm --m 16384 --n 1024 --k 3072 --mode resid16

Each run times `--iters` launches with CUDA events on the launching stream
(after `--warmup` launches) and prints one JSON line with the mean launch time
and the achieved TFLOP/s.  Used for the ncu captures under profiles/ (one
kernel, a handful of launches, inputs larger than L2).
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
    ap.add_argument("kernel", choices=["gemm"])
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=6144)
    ap.add_argument("--k", type=int, default=1024)
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
    g = torch.Generator(device="cuda").manual_seed(0)
    A = (torch.randn(a.m, a.k, device="cuda", generator=g) * 0.5).to(dt)
    B = (torch.randn(a.n, a.k, device="cuda", generator=g) * 0.05).to(dt)
    mode = {"store16": L.EPI_STORE16, "resid16": L.EPI_RESID16, "swiglu": L.EPI_SWIGLU16,
            "resid32": L.EPI_RESID32, "store32": L.EPI_STORE32, "argmax": L.EPI_ARGMAX}[a.mode]
    out_cols = a.n // 2 if a.mode == "swiglu" else a.n
    out_dt = torch.float32 if a.mode in ("resid32", "store32", "argmax") else dt
    out = torch.zeros(a.m, out_cols, device="cuda", dtype=out_dt)
    keys = torch.zeros(a.m, dtype=torch.int64, device="cuda") if a.mode == "argmax" else None
    bn = 256 if a.mode == "swiglu" else 0
    for _ in range(a.warmup):
        L.gemm(A, B, out, mode=mode, keys=keys, force_bn=bn)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        L.gemm(A, B, out, mode=mode, keys=keys, force_bn=bn)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.iters
    flops = 2.0 * a.m * a.n * a.k
    print(json.dumps({"kernel": "gemm_tc", "m": a.m, "n": a.n, "k": a.k, "mode": a.mode,
                      "dtype": a.dtype, "ms": ms, "tflops": flops / ms / 1e9,
                      "algorithmic_bytes": (a.m * a.k + a.n * a.k) * 2 + a.m * out_cols * out.element_size()}))


if __name__ == "__main__":
    main()
