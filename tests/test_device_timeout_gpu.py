"""A bounded device wait that runs out, end to end (GPU).

Every tcgen05 kernel of the library waits on mbarriers that TMA copies and
MMA commits complete, and every such wait is bounded by %globaltimer; one
that runs out sets the timeout bit of the context's status word and the host
call returns QA_ERR_TIMEOUT (the reference reports a lost device after each
submit, src/decoder.rs:1670-1672).  qa_probe_timeout runs that path on
purpose: a kernel waits, with a short limit, on a barrier nothing completes.
The test checks the error code and the time it took, and that the same
context then aligns exactly as before.  Nothing faults: the kernel issues no
copy and holds no tensor memory, and it returns once the wait gives up.
"""
import time

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


def test_wait_timeout_reports_and_context_survives(env):
    E = env
    al = E.gpu_aligner()
    lib = E.qa._lib
    clip = E.qa.synth.workload(0)[0]
    inp = al.build_input(clip.samples, clip.text, clip.language)
    [(before, _)] = al.align_inputs([clip.samples], [inp])
    t0 = time.perf_counter()
    rc = lib.lib().qa_probe_timeout(al._ctx, 20)
    dt = time.perf_counter() - t0
    assert rc == lib.QA_ERR_TIMEOUT, rc
    assert b"wait ran out" in lib.lib().qa_last_error(al._ctx)
    assert 0.015 <= dt < 5.0, dt  # the 20 ms limit, not the 2 s default
    # the context keeps working: the same clip gives the same timestamps
    [(after, _)] = al.align_inputs([clip.samples], [inp])
    assert np.array_equal(before, after)
    assert lib.lib().qa_probe_timeout(al._ctx, 0) == lib.QA_ERR_ARG
