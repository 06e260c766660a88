"""qa_head_noalloc — the timestamp head for callers that cannot allocate
device memory (a host whose GPU memory belongs to its own pool, or a
latency-bound caller that must not stall on cudaMalloc/cudaFree) — against
the allocating entry point qa_head on the same inputs.

Both run the same kernels, so the bars are those of the head test: raw_ms
identical, logits within 1e-4 max-abs relative error.  Two calls in a row with
different inputs check that the shared scratch carries nothing from one call
to the next.  This file is named to be collected last.
"""
import numpy as np
import pytest

from conftest import cuda_ok

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not cuda_ok():
        pytest.skip("no CUDA device")
    import pipeline_env as E
    return E


def _noalloc(E, al, hidden, rows, want_logits=True):
    import torch
    lib = E.qa._lib
    h = torch.from_numpy(np.ascontiguousarray(hidden, np.float32)).cuda()
    r = torch.from_numpy(np.ascontiguousarray(rows, np.int32)).cuda()
    raw = torch.zeros(len(rows), dtype=torch.int64, device="cuda")
    lg = (torch.zeros(len(rows), al.cfg.num_labels, dtype=torch.float32, device="cuda")
          if want_logits else None)
    torch.cuda.synchronize()  # inputs written on torch's stream; the call uses the context's
    rc = lib.lib().qa_head_noalloc(al._ctx, h.data_ptr(), h.shape[0], r.data_ptr(), len(rows),
                                   raw.data_ptr(), lg.data_ptr() if lg is not None else None)
    lib.check(rc, al._ctx)
    return raw.cpu().numpy(), (lg.cpu().numpy() if lg is not None else None)


def test_head_noalloc_matches_head_twice(env):
    E = env
    al = E.gpu_aligner()
    rng = np.random.default_rng(17)
    cases = [(300, rng.choice(300, 50, replace=False)), (700, rng.choice(700, 333, replace=False))]
    for seq, rows in cases:
        hidden = (rng.standard_normal((seq, al.cfg.hidden_size)) * 3.0).astype(np.float32)
        raw_ref, lg_ref, _ = al.head(hidden, rows)
        raw, lg = _noalloc(E, al, hidden, rows)
        assert np.array_equal(raw, raw_ref)
        assert E.rel_err(lg, lg_ref) <= 1e-4


def test_head_noalloc_rejects_rows_beyond_its_scratch(env):
    E = env
    al = E.gpu_aligner()
    hidden = np.zeros((3000, al.cfg.hidden_size), np.float32)
    with pytest.raises(E.qa.QaError) as ei:
        _noalloc(E, al, hidden, np.arange(2049), want_logits=False)
    assert ei.value.code == E.qa._lib.QA_ERR_CAP  # QA_NOALLOC_HEAD_MAX_ROWS = 2048


def test_head_noalloc_rejects_rows_outside_hidden(env):
    """A row index at or past `seq` (or below 0) is never read: the call
    returns QA_ERR_SHAPE as qa_head does, and the context keeps working.
    The hidden buffer holds more rows than the `seq` passed, so even an
    unguarded read of the bad index would stay inside valid memory."""
    E = env
    al = E.gpu_aligner()
    rng = np.random.default_rng(23)
    seq = 64
    hidden = (rng.standard_normal((seq + 16, al.cfg.hidden_size))).astype(np.float32)
    import torch
    lib = E.qa._lib
    h = torch.from_numpy(hidden).cuda()
    raw = torch.zeros(3, dtype=torch.int64, device="cuda")
    for bad in ([0, seq, 5], [3, -1, 7]):
        r = torch.tensor(bad, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        rc = lib.lib().qa_head_noalloc(al._ctx, h.data_ptr(), seq, r.data_ptr(), 3,
                                       raw.data_ptr(), None)
        assert rc == lib.QA_ERR_SHAPE, rc
    rows = np.array([0, seq - 1, 9])
    raw_ref, _, _ = al.head(hidden[:seq], rows)
    raw_ok, _ = _noalloc(E, al, hidden[:seq], rows, want_logits=False)
    assert np.array_equal(raw_ok, raw_ref)
