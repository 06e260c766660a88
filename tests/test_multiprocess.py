"""Multi-rank host logic on CPU: world_size 2 `gloo` ranks run the same
sharding and timing reductions bench.py runs over NCCL on GPUs."""
import os
import socket

import pytest

from conftest import pkg


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, per_rank, q):
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    shard = importlib.import_module("qwen3-aligner-wgpu_b200.shard")
    g = shard.RankGroup(backend="gloo", timeout_s=60)
    mine = list(shard.contiguous_shard(g.rank, g.world, per_rank))
    g.barrier()
    t_max = g.max(10.0 + rank)        # slowest rank's time
    n_sum = g.sum(float(len(mine)))   # whole-job units
    q.put((rank, mine, t_max, n_sum))
    g.close()


def test_two_gloo_ranks_shard_and_reduce():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, 5, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    assert res[0][1] == list(range(0, 5)) and res[1][1] == list(range(5, 10))
    assert all(r[2] == 11.0 for r in res)   # max over ranks
    assert all(r[3] == 10.0 for r in res)   # sum over ranks


def _crash_main(rank, world, port, q):
    """Step 1 on both ranks; then rank 1 dies between steps (no collective in
    flight) and rank 0's next reduction must fail within the group's timeout."""
    import importlib
    import sys
    import time
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    shard = importlib.import_module("qwen3-aligner-wgpu_b200.shard")
    g = shard.RankGroup(backend="gloo", timeout_s=5)
    g.barrier()
    first = g.sum(1.0)
    if rank == 1:
        os._exit(3)  # a worker crash between steps
    t0 = time.monotonic()
    try:
        g.max(2.0)
        q.put((rank, first, "completed", time.monotonic() - t0))
    except Exception as e:  # the dead peer surfaces as an error, not a hang
        q.put((rank, first, type(e).__name__, time.monotonic() - t0))
    os._exit(0)


def test_worker_crash_between_steps_is_reported():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_crash_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, first, outcome, waited = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and first == 2.0
    assert outcome != "completed" and waited < 60.0
    assert procs[1].exitcode == 3 and procs[0].exitcode == 0


def test_lpt_balances_and_covers():
    shard = pkg().shard
    import random
    rnd = random.Random(0)
    secs = [rnd.uniform(5, 60) for _ in range(200)]
    costs = [shard.clip_flops(int(13 * s), int(13 * s + 3 * s * 4.2), int(6 * s), int(s) + 1)
             for s in secs]
    for n in (1, 2, 4, 8):
        parts = shard.lpt_assign(costs, n)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(costs)))
        loads = [sum(costs[i] for i in p) for p in parts]
        assert max(loads) <= sum(costs) / n + max(costs)  # LPT bound
        assert max(loads) / (sum(costs) / n) < 1.02


def test_contiguous_shard_rejects_bad_rank():
    shard = pkg().shard
    with pytest.raises(ValueError):
        shard.contiguous_shard(2, 2, 4)
