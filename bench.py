#!/usr/bin/env python
"""Benchmark of the B200 alignment path: aligned audio-seconds per second.

Workload (per GPU): 64 independent clips, durations
U(5, 30) s, 2.5-3.5 words/s, English pseudo-words mixed with CJK characters,
f16 storage, on the seeded random-init Qwen3-ForcedAligner-0.6B architecture.
One step = one pass of the whole path over the batch: samples -> log-mel ->
audio tower -> embedding gather / audio scatter -> 28-layer causal prefill
over the paged K/V cache -> timestamp head -> argmax.

* value   — device time of the batched pass with its inputs already in HBM
            (qa_batch_stage once, then qa_batch_run per step on this stream),
            L2 flushed between steps; whole job = audio seconds of all ranks /
            the slowest rank's time (weak scaling: every GPU runs its own shard
            of clips; no data-path collective).
* e2e     — the same metric through the public API (Aligner.align_stream over
            the timed steps' batches: word split + tokenize + host->device
            copy from pinned staging + device pass + device->host read of
            raw_ms + timestamp repair for every batch; the host work of one
            batch overlaps the device pass of its neighbour).
* roofline — the tcgen05 GEMM kernel (the dominant kernel) timed live with CUDA
            events around every launch on its stream during the timed region.
* cpu_baseline — the CPU restatement of the reference's --device cpu path
            (oracle/) on a bounded sample, rank 0 at N=1 only.

`--impl reference` times that CPU path alone on the same workload (the
reference crate is Rust and cannot be built here; the oracle restates it).

`--workload 4` runs BASELINE config 4's clip distribution instead (U(5, 60) s
English clips at 3 words/s) with the Local Head on: every step also refines
each word's interval on the device, and the CPU baseline runs the oracle's
Local Head after its head.
"""
import argparse
import datetime
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "aligned audio-sec/sec per B200 at 1/2/4/8 GPUs; prefill tok/s; % TC/HBM peak"
UNIT = "audio-s/s"
L2_FLUSH_BYTES = 256 << 20
WORKLOADS = {
    0: "BASELINE config 0: one 10 s clip, 25 English words, f16",
    1: "BASELINE config 1: one 60 s clip, 180 English words, f16",
    2: "BASELINE config 2: 64 clips/GPU, U(5,30) s, 2.5-3.5 words/s, English + CJK, f16",
    4: "BASELINE config 4 (per-GPU shard): clips U(5,60) s, English, 3 words/s, f16, "
       "Local Head on (seed-0 random-init 405k-parameter head)",
    3: "BASELINE config 3: one 300 s clip, 900 English words, bf16 storage",
}
# CPU-baseline sample per workload (clips); config 3's one clip is minutes of
# CPU work, so it has none
CPU_SAMPLE = {0: 1, 1: 1, 2: 12, 3: 0, 4: 3}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--clips", type=int, default=64, help="clips per GPU per step")
    ap.add_argument("--workload", type=int, default=2, choices=[0, 1, 2, 3, 4],
                    help="BASELINE config: 2 = U(5,30) s English+CJK clips (the headline); "
                         "4 = U(5,60) s English clips at 3 words/s with the Local Head on; "
                         "0, 1, 3 = its single clip (10 s, 60 s, 300 s) per step and GPU")
    ap.add_argument("--half", default=None, help="f16 | bf16 (default: bf16 for config 3, "
                                                  "else f16)")
    ap.add_argument("--cpu-sample-clips", type=int, default=None,
                    help="clips of the CPU baseline's sample (default: about 15 s of CPU "
                         "work, 12 clips of config 2 or 3 of config 4)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true",
                    help="BASELINE config 4 as a whole set: --sweep-clips clips split across the "
                         "ranks by LPT and aligned through sweep.py (strong scaling)")
    ap.add_argument("--sweep-clips", type=int, default=4096)
    ap.add_argument("--token-budget", type=int, default=65536)
    args = ap.parse_args()
    if args.half is None:
        args.half = "bf16" if args.workload == 3 else "f16"
    return args


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


def model_flops(cfg, inp, n_samples) -> float:
    """Algorithmic FLOPs of one clip's pass (2 per multiply-add): the conv stem
    per 100-frame chunk (a padded tail chunk counted whole), conv_out, the
    tower layers' dense projections and windowed attention, the projector,
    the decoder's dense projections and exact causal attention, and the
    timestamp head on the 2W slot rows."""
    def down(x):
        return (x - 1) // 2 + 1  # conv 3x3, stride 2, pad 1
    cs = 2 * cfg.n_window
    frames = n_samples // 160
    chunks = -(-frames // cs)
    c, mel = cfg.downsample_hidden, cfg.num_mel_bins
    h1, w1 = down(mel), down(cs)
    h2, w2 = down(h1), down(w1)
    h3, w3 = down(h2), down(w2)
    conv = 2.0 * (9 * c * h1 * w1 + 9 * c * c * h2 * w2 + 9 * c * c * h3 * w3)
    d, na = cfg.d_model, inp.n_audio_tokens
    tower = chunks * conv + na * 2.0 * (c * h3 * d)                       # conv_out
    tower += cfg.encoder_layers * na * 2.0 * d * (3 * d + d + 2 * cfg.encoder_ffn_dim)
    win = w3 * (cfg.n_window_infer // cs)
    ws = [win] * (na // win) + ([na % win] if na % win else [])
    tower += cfg.encoder_layers * sum(4.0 * w * w * d for w in ws)
    tower += na * 2.0 * d * (d + cfg.output_dim)                           # proj1, proj2
    H, L = cfg.hidden_size, inp.seq_len()
    qd, kvd = cfg.num_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim
    dense = 2.0 * H * (qd + 2 * kvd) + 2.0 * qd * H + 2.0 * H * 2 * cfg.intermediate_size \
        + 2.0 * cfg.intermediate_size * H
    attn = cfg.num_heads * 4.0 * cfg.head_dim * L * (L + 1) / 2
    dec = cfg.num_layers * (dense * L + attn)
    head = 2.0 * H * cfg.num_labels * len(inp.timestamp_positions)
    return tower + dec + head


def build_inputs(qa, clips, builder):
    words = [qa.synth.split_words(c.text, c.language) for c in clips]
    return builder.build_batch(words, [qa.synth.valid_mel_frames(len(c.samples)) for c in clips])


def cpu_sample(args, clips):
    """The clips both CPU legs time (the reference arm and cpu_baseline): the
    first k clips of the workload."""
    k = args.cpu_sample_clips or CPU_SAMPLE[args.workload] or 1
    return list(range(min(k, len(clips))))


def cpu_align(orc, om, lh, c, inp):
    """One clip through the CPU restatement: the whole path, and with `lh`
    (an oracle LocalHead) the refinement of its word intervals as well."""
    r = om.align_raw(c.samples, inp.input_ids, inp.timestamp_positions)
    if lh is not None:
        _, logits, normed, _ = om.head(r["hidden"], inp.timestamp_positions, want_normed=True)
        lh.refine(c.samples, logits, normed)


def cpu_reference(qa, orc, cfg, weights, clips, inps, threads, lh_pkg=None):
    """The oracle (CPU restatement of the reference's --device cpu path) over
    `clips`: audio-seconds per wall second, whole path per clip."""
    orc.set_threads(threads)
    om = orc.Model(weights, cfg)
    lh = orc.LocalHead(*lh_pkg) if lh_pkg is not None else None
    t0 = time.perf_counter()
    audio = 0.0
    for c, inp in zip(clips, inps):
        cpu_align(orc, om, lh, c, inp)
        audio += len(c.samples) / 16000.0
    dt = time.perf_counter() - t0
    return audio / dt, audio, dt


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    qa = importlib.import_module("qwen3-aligner-wgpu_b200")
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    orc.build()
    cfg = qa.synth.ModelConfig()
    weights = qa.synth.random_weights(cfg)
    clips = qa.synth.workload(args.workload, n_clips=args.clips)
    inps = build_inputs(qa, clips, qa.synth.InputBuilder())
    threads = os.cpu_count() or 1
    orc.set_threads(threads)
    om = orc.Model(weights, cfg)
    lh = orc.LocalHead(*qa.synth.random_local_head(0)) if args.workload == 4 else None
    sample = cpu_sample(args, clips)  # the same clips as our arm's cpu_baseline
    per_step = min(2, len(sample))
    audio = 0.0
    total = 0.0
    for step in range(args.warmup + args.steps):
        idx = [sample[(step * per_step + k) % len(sample)] for k in range(per_step)]
        t0 = time.perf_counter()
        a = 0.0
        for i in idx:
            cpu_align(orc, om, lh, clips[i], inps[i])
            a += len(clips[i].samples) / 16000.0
        dt = time.perf_counter() - t0
        if step >= args.warmup:
            audio += a
            total += dt
    value = audio / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded audio/transcripts, random-init weights)",
        "config": {"workload": WORKLOADS[args.workload],
                   "sample": f"the first {len(sample)} clips of the workload (as cpu_baseline), "
                             f"{per_step} per step, cycled"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps x {per_step} clips ({audio:.1f} audio-s); "
                                   "C++/OpenMP restatement of the reference's --device cpu path"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


class _Length:
    """Stands in for the samples of a clip another rank aligns: sweep.py reads
    only their count."""

    def __init__(self, n):
        self.n = n

    def __len__(self):
        return self.n


def _gen_config4_audio(i):
    qa = importlib.import_module("qwen3-aligner-wgpu_b200")
    return qa.synth.workload_clip(4, i).samples


def run_sweep(args):
    """BASELINE config 4 as a whole set through sweep.py: every rank computes
    the same LPT shares from the clips' durations and words, synthesises the
    audio of its own share only (a process pool, before the GPU work), warms
    up on a few of its clips, then aligns its share (Local Head on) between a
    barrier and a device synchronisation.  Reported: the whole set's audio
    seconds over the slowest rank's time, and every rank's time."""
    import concurrent.futures as cf
    import multiprocessing as mp
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    qa = importlib.import_module("qwen3-aligner-wgpu_b200")
    texts = qa.synth.workload_texts(4, args.sweep_clips)
    n_samples = [int(round(sec * 16000)) for sec, _, _ in texts]
    words = [qa.synth.split_words(t, l) for _, t, l in texts]
    costs = [qa.sweep.estimate_cost(n, w) for n, w in zip(n_samples, words)]
    mine = qa.sweep.rank_share(costs, rank, world)
    t0 = time.perf_counter()
    workers = max(1, (os.cpu_count() or 2) // world - 1)
    with cf.ProcessPoolExecutor(workers, mp_context=mp.get_context("spawn")) as ex:
        audio = dict(zip(mine, ex.map(_gen_config4_audio, mine, chunksize=4)))
    gen_s = time.perf_counter() - t0
    clips = [(audio[i] if i in audio else _Length(n), t, l)
             for i, (n, (_, t, l)) in enumerate(zip(n_samples, texts))]

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = qa.synth.ModelConfig()
    al = qa.Aligner.load_backend_with_dtype(qa.synth.random_weights(cfg), "f16", device=local,
                                            cfg=cfg, local_head=qa.synth.random_local_head(0))
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    al.set_stream(stream.cuda_stream)
    # warm-up: the grow-only workspaces of a full pass
    warm = sorted(mine, key=lambda i: -n_samples[i])[:48]
    qa.sweep.sweep(al, [clips[i] for i in warm], token_budget=args.token_budget)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    out = qa.sweep.sweep(al, clips, token_budget=args.token_budget, rank=rank, world=world)
    e1.record(stream)
    barrier()
    ms = e0.elapsed_time(e1)
    assert sorted(out) == sorted(mine)
    per_rank = torch.zeros(world, dtype=torch.float64, device=dev)
    per_rank[rank] = ms
    mine_audio = torch.zeros(world, dtype=torch.float64, device=dev)
    mine_audio[rank] = sum(n_samples[i] for i in mine) / 16000.0
    if world > 1:
        dist.all_reduce(per_rank)
        dist.all_reduce(mine_audio)
    per_rank, mine_audio = per_rank.cpu().tolist(), mine_audio.cpu().tolist()
    total_audio = sum(n_samples) / 16000.0
    value = total_audio / (max(per_rank) / 1e3)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": 1,
            "warmup": 1, "ms_per_step": max(per_rank), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded audio/transcripts, random-init weights)",
            "config": {"workload": f"BASELINE config 4 whole set: {args.sweep_clips} clips "
                                   "U(5,60) s, English, 3 words/s, Local Head on, through "
                                   "sweep.py (LPT shares, token-budget passes, two in flight)",
                       "clips": args.sweep_clips, "audio_s": total_audio,
                       "token_budget": args.token_budget,
                       "parallelism": f"clip-sharded x{world} by LPT, no collectives"},
            "rank_ms": per_rank, "rank_audio_s": mine_audio,
            "imbalance_max_over_mean": max(per_rank) / (sum(per_rank) / world),
            "e2e": {"value": value, "unit": UNIT,
                    "h2d_bytes_per_step": int(sum(n_samples) * 4),
                    # raw_ms (8 B per slot) and the refined intervals (2 x 8 B per word)
                    "d2h_bytes_per_step": int(sum(32 * len(w) for w in words)),
                    "includes": "word split + tokenisation + staging + H2D + device passes + "
                                "Local Head + D2H + repair, for the whole set"},
            "audio_synthesis_s_rank0": gen_s,
        }), flush=True)
    al.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.sweep:
        return run_sweep(args)

    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    qa = importlib.import_module("qwen3-aligner-wgpu_b200")
    cfg = qa.synth.ModelConfig()
    weights = qa.synth.random_weights(cfg)
    lh_pkg = qa.synth.random_local_head(0) if args.workload == 4 else None
    al = qa.Aligner.load_backend_with_dtype(weights, args.half, device=local, cfg=cfg,
                                            local_head=lh_pkg)
    if args.workload in (2, 4):
        clips = qa.synth.workload(args.workload, n_clips=args.clips, start=rank * args.clips)
    else:  # one clip: every rank aligns its own copy
        clips = qa.synth.workload(args.workload)
    inps = build_inputs(qa, clips, al.input_builder)
    samples = [c.samples for c in clips]
    audio_s = sum(len(s) for s in samples) / 16000.0
    T_d = sum(i.seq_len() for i in inps)
    T_a = sum(i.n_audio_tokens for i in inps)
    flops_step = sum(model_flops(cfg, i, len(s)) for i, s in zip(inps, samples))

    # One created stream for everything timed: the library's kernels, the L2
    # flush and the CUDA events (the legacy default stream has handle 0, which
    # qa_set_stream reads as "the library's own stream").
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    al.set_stream(stream.cuda_stream)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    # every clip alone, once, untimed: the timed batch must reproduce these
    # raw_ms bit for bit (a row's arithmetic does not depend on its batch)
    single = [al.align_inputs([s], [i])[0][0] for s, i in zip(samples, inps)]

    # ---- value: device pass on HBM-resident inputs
    staged = al.stage(samples, inps)
    for _ in range(args.warmup):
        al.run()
    barrier()

    def timed_steps():
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        n_launch = 0
        barrier()
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            al.run()
            e1.record(stream)
            n_launch += al_launches(al, qa)
        barrier()
        return sum(e0.elapsed_time(e1) for e0, e1 in evs), n_launch

    # value: K steps with no per-launch instrumentation
    with ClockSampler(local) as clk:
        dev_ms, launches = timed_steps()
    # the per-kernel breakdown and the roofline: the same K steps again with a
    # CUDA event pair recorded around every launch on the launching stream
    al.set_profile(True)
    prof_ms, _ = timed_steps()
    prof = al.profile()
    al.set_profile(False)
    raw_check = al.fetch(staged)
    mismatched = [k for k, ((r, _), r1) in enumerate(zip(raw_check, single))
                  if not np.array_equal(r, r1)]
    if mismatched:
        raise SystemExit(f"timed batch differs from single-clip passes on clips {mismatched}")
    ms_max = max_over_ranks(dev_ms)
    prof_ms_max = max_over_ranks(prof_ms)  # every rank takes the same collectives
    audio_all = sum_over_ranks(audio_s)
    value = audio_all * args.steps / (ms_max / 1e3)

    # ---- e2e through the public API (host buffers, copies inside)
    texts = [(c.samples, c.text, c.language) for c in clips]
    for _ in al.align_stream([texts, texts]):  # warm both batch slots' staging buffers
        pass
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in al.align_stream(texts for _ in range(args.steps)):
        pass
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = audio_all * args.steps / (e2e_ms / 1e3)
    t = al.timings
    # host input building of one batch (word split + tokenisation + ids), the
    # host work each e2e step overlaps with the previous batch's device pass
    host = {}
    for _ in range(5):
        h = {}
        al.build_inputs(texts, h)
        for k, v in h.items():
            host[k] = min(host.get(k, v), v)

    # ---- roofline of the dominant kernel (tcgen05 GEMM), from live events
    hbm, tf_burst, tf_sus, src = peaks()
    # every GEMM launch (classes "gemm:<projection>") is the dominant kernel
    gemms = [v for k, v in prof.items() if k.startswith("gemm")]
    g = {"launches": sum(v["launches"] for v in gemms), "total_ms": sum(v["total_ms"] for v in gemms),
         "flops": sum(v["flops"] for v in gemms)}
    gemm_tflops = g["flops"] / (g["total_ms"] / 1e3) / 1e12 if g["total_ms"] else 0.0
    total_prof_ms = sum(v["total_ms"] for v in prof.values()) or 1.0
    kernels = {k: {"launches": v["launches"], "ms_per_step": v["total_ms"] / args.steps,
                   "share": v["total_ms"] / total_prof_ms,
                   **({"tflops": v["flops"] / (v["total_ms"] / 1e3) / 1e12} if v["flops"] else {}),
                   **({"gbs": v["bytes"] / (v["total_ms"] / 1e3) / 1e9,
                       "hbm_frac": v["bytes"] / (v["total_ms"] / 1e3) / 1e9 / hbm}
                      if v["bytes"] and not v["flops"] else {})}
               for k, v in sorted(prof.items(), key=lambda kv: -kv[1]["total_ms"])}
    # DRAM bytes per GEMM launch: not measurable in this run (no profiler);
    # read from the committed ncu summary of the same shapes
    traffic, traffic_src = None, None
    tr = os.path.join(ROOT, "profiles", "gemm_traffic.json")
    if os.path.exists(tr):
        tj = json.load(open(tr))
        traffic = tj.get("bytes_per_launch")
        traffic_src = "static: " + tj.get("source", "profiles/gemm_traffic.json")

    out = None
    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": args.half,
            "data": "synthetic (seeded audio/transcripts, random-init weights)",
            "config": {"workload": WORKLOADS[args.workload] + ", one device pass per step",
                       "clips_per_gpu": len(clips), "audio_s_per_gpu_step": audio_s,
                       "decoder_tokens_per_gpu_step": T_d, "audio_tokens_per_gpu_step": T_a,
                       "l2": "flushed between timed steps (256 MiB write, outside the events)",
                       "parallelism": f"clip-sharded x{world}, no collectives"},
            "realtime_factor_per_gpu": value / world,
            "model_flops_per_gpu_step": flops_step,
            # the whole pass's algorithmic FLOPs over its device time, against
            # the measured sustained bf16 peak (HBM-bound kernels included)
            "tensor_frac_whole_pass": flops_step / (ms_max / args.steps / 1e3) / (tf_sus * 1e12),
            "prefill_tok_s": T_d * world * args.steps / (ms_max / 1e3),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(t["h2d_bytes"]) * world,
                    "d2h_bytes_per_step": int(t["d2h_bytes"]) * world,
                    "includes": "split_words + tokenize + pinned staging + H2D + device pass + "
                                "D2H raw_ms + LIS repair"
                                + (" + Local Head intervals (device) + D2H" if lh_pkg else "")},
            "gpu_launches": launches,
            "profiled_ms_per_step": prof_ms_max / args.steps,
            "roofline": {"bound": "tensor", "kernel": "gemm_pair_kernel + gemm_tc_kernel (tcgen05, all GEMM launches)",
                         "measured": "CUDA events around every GEMM launch on its stream, in a second "
                                     "pass of the K timed steps",
                         "achieved": gemm_tflops, "peak": tf_sus, "unit": "TFLOP/s",
                         "frac": gemm_tflops / tf_sus, "peak_kind": f"{src} sustained bf16",
                         "traffic": traffic, "traffic_source": traffic_src,
                         "launches_per_step": g["launches"] / args.steps,
                         "flops_per_launch": g["flops"] / max(g["launches"], 1)},
            "kernels": kernels,
            "phases_ms": {k: t[k] for k in ("mel_ms", "enc_ms", "gather_ms", "prefill_ms", "head_ms",
                                            "local_ms")},
            "host_build_ms_per_batch": {**host, "cores": os.cpu_count()},
            "clocks": clk.summary(),
        }
    # ---- CPU baseline (rank 0 at N=1 only; after the GPU phase)
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not CPU_SAMPLE[args.workload] \
            and not args.cpu_sample_clips:
        out["cpu_baseline"] = None
        out["cpu_baseline_note"] = "none for config 3: its one 300 s clip is minutes of CPU work"
    elif rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as orc
        orc.build()
        k = len(cpu_sample(args, clips))
        threads = os.cpu_count() or 1
        v, a, dt = cpu_reference(qa, orc, cfg, weights, clips[:k], inps[:k], threads, lh_pkg)
        out["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                               "sample": f"the first {k} clips of the workload ({a:.1f} audio-s "
                                         f"in {dt:.1f} s), whole path per clip; the reference "
                                         f"arm cycles through the same clips"}
    if rank == 0:
        print(json.dumps(out), flush=True)
    al.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def al_launches(al, qa):
    """Kernels the library launched in the last qa_batch_run."""
    import ctypes
    t = qa._lib.QaTimings()
    qa._lib.lib().qa_get_timings(al._ctx, ctypes.byref(t))
    return int(t.gpu_launches)


if __name__ == "__main__":
    sys.exit(main())
