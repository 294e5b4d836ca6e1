"""CPU checks of the C-ABI library: it loads, exports every entry point that
include/vcpm_b200.h declares, its host-side helpers reproduce the reference's
known answers, and failures come back as status codes (never aborts)."""
import ctypes as C
import json
import os
import re
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
import vcpm_b200 as vb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vcpm_b200.h")
KAT = json.load(open(os.path.join(ROOT, "tests", "golden", "reference_kat.json")))


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(vb_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    L = vb.lib()
    names = declared_functions()
    assert len(names) > 40
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/vcpm_b200.h but not exported"
    # the ctypes binding declares a signature for every entry point
    assert sorted(vb.SIGNATURES) == names


def test_exports_match_nm():
    out = subprocess.run(["nm", "-D", "--defined-only", vb.LIB_PATH], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T vb_" in l}
    assert set(declared_functions()) <= exported


def test_host_sway_schedule_and_zero_star():
    k = KAT["cfm_schedule"]
    got = [vb.lib().vb_cfm_sway_t_bf16(s, 10) for s in range(11)]
    assert got == [np.float32(v) for v in k["sway_t"]]
    assert vb.lib().vb_cfm_zero_star_steps(10) == 1


def test_host_noise_matches_oracle():
    x = np.zeros(256, np.float32)
    vb.lib().vb_cfm_noise(42, 3, x.ctypes.data, 256)
    assert np.array_equal(x, O.cfm_noise(42, 3, 256))


def test_host_cache_capacity():
    for req, mx, want in KAT["cache_capacity"]["cases"]:
        assert vb.lib().vb_round_cache_capacity(req, mx) == want


def test_null_arguments_are_rejected_without_a_device():
    L = vb.lib()
    assert L.vb_create(0, None) == vb.VB_ERR_INVALID_ARG
    assert L.vb_sync(None) == vb.VB_ERR_INVALID_ARG
    assert L.vb_matmul(None, None, None, 1, None, 0) == vb.VB_ERR_INVALID_ARG
    assert L.vb_lm_forward(None, None, None, 1, None, None, 1, None, None) == vb.VB_ERR_INVALID_ARG
    assert L.vb_last_error(None) == b"null context"


def test_no_device_is_a_status_not_a_crash():
    n = vb.device_count()
    if n > 0:
        pytest.skip("a CUDA device is present")
    h = C.c_void_p()
    assert vb.lib().vb_create(0, C.byref(h)) == vb.VB_ERR_BACKEND
    with pytest.raises(vb.VBError):
        vb.Context(0)


def test_fault_injection_alloc_runs_in_child():
    """VB_FAULT=alloc makes context creation fail with OOM before any device
    call (host-side failure injection)."""
    code = ("import sys; sys.path.insert(0, %r); import ctypes as C, vcpm_b200 as vb; "
            "h = C.c_void_p(); print(vb.lib().vb_create(0, C.byref(h)))" % os.path.join(ROOT, "voxcpm-cpp_b200"))
    env = dict(os.environ, VB_FAULT="alloc")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == str(vb.VB_ERR_OOM)
