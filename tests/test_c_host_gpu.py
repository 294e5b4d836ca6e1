"""The C11 host driver replays the generation loop through the C ABI on the
device: prompt, per-patch generation with the stop predictor, the streaming
AudioVAE decode, and per-utterance termination (vb_gen_retire) -- the
reference's loop (src/gen_run.c:166-215) driven from C."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "voxcpm-cpp_b200")
sys.path.insert(0, PKG)

import build as B  # noqa: E402

pytestmark = pytest.mark.gpu


def run(*args):
    exe = B.build_host()
    r = subprocess.run([exe, "run", *map(str, args)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("batch,max_len,min_len", [(4, 12, 2), (3, 8, 5), (1, 6, 0)])
def test_generation_loop_from_c(batch, max_len, min_len):
    out = run(batch, max_len, min_len, 1234)
    assert out["device_error"] == 0 and out["finite"]
    assert out["batch"] == batch and 1 <= out["steps"] <= max_len
    # a stop counts once n_patches > min_len + 1 (src/gen_run.c:195-197)
    floor = min(max_len, min_len + 2)
    assert all(floor <= n <= max_len for n in out["patches"]), out["patches"]
    assert max(out["patches"]) == out["steps"]
    assert out["audio_abs_sum"] > 0.0


def test_c_driver_is_deterministic():
    a, b = run(4, 10, 2, 99), run(4, 10, 2, 99)
    assert a["patches"] == b["patches"]
    assert a["audio_abs_sum"] == b["audio_abs_sum"]
