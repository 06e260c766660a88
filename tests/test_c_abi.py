"""The C-ABI library without a GPU: it loads, exports every symbol the public
headers declare, and rejects bad arguments with status codes instead of
aborting.  (No compute call is made here.)"""
import ctypes
import os
import re

import pytest

from conftest import ROOT, cuda_ok, pkg


def _declared():
    names = []
    for h in ("qa_b200.h", "qa_b200_kernels.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        names += re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(qa_\w+)\s*\(", src, re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    L = pkg()._lib.lib()
    declared = _declared()
    assert len(declared) >= 14
    missing = [n for n in declared if not hasattr(L, n)]
    assert not missing, missing
    assert sorted(pkg()._lib.EXPORTED) == declared


def test_null_and_bad_arguments():
    lib = pkg()._lib
    L = lib.lib()
    assert L.qa_close(None) == lib.QA_ERR_ARG
    assert L.qa_last_error(None) == b"null context"
    assert L.qa_half(None) == -1
    assert L.qa_open(0, 7, None) == lib.QA_ERR_ARG
    out = ctypes.c_void_p()
    assert L.qa_open(0, 5, ctypes.byref(out)) == lib.QA_ERR_ARG
    # host-only entry points: argument checks, no device needed
    n, sr, ch = ctypes.c_int64(0), ctypes.c_int(0), ctypes.c_int(0)
    assert L.qa_decode_wav(None, 10, None, 0, ctypes.byref(n), ctypes.byref(sr),
                           ctypes.byref(ch)) == lib.QA_ERR_ARG
    junk = (ctypes.c_uint8 * 64)()
    assert L.qa_decode_wav(junk, 64, None, 0, ctypes.byref(n), ctypes.byref(sr),
                           ctypes.byref(ch)) == lib.QA_ERR_SHAPE
    assert L.qa_resampled_length(100, 0, 16000) == -1
    assert L.qa_resampled_length(44100, 44100, 16000) == 16000
    buf = (ctypes.c_float * 16)()
    assert L.qa_resample(buf, 16, 44100, 16000, buf, 5) == lib.QA_ERR_SHAPE
    assert L.qa_resample(None, 16, 44100, 16000, buf, 6) == lib.QA_ERR_ARG
    assert L.qa_fix_timestamps(None, 3, None) == lib.QA_ERR_ARG


@pytest.mark.skipif(cuda_ok(), reason="checks the no-device path")
def test_open_without_a_device_fails_cleanly():
    lib = pkg()._lib
    out = ctypes.c_void_p()
    assert lib.lib().qa_open(0, lib.QA_HALF_F16, ctypes.byref(out)) == lib.QA_ERR_CUDA
    assert not out.value


def test_library_has_no_cpu_fallback_symbols():
    """The product library exports only the qa_ ABI (no oracle code linked in)."""
    import subprocess
    so = pkg()._lib.LIB_PATH
    syms = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in syms.splitlines() if " T " in l}
    assert not any(s.startswith("or_") for s in exported)
