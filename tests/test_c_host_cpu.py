"""The C11 host driver (voxcpm-cpp_b200/host/vcpm_gen_run.c) compiles
against include/vcpm_b200.h alone with -std=c11 -Wall -Wextra -Werror
-pedantic and links libvcpm_b200.so; the public structs' layouts as C sees
them equal the Python binding's ctypes layouts (no device needed)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "voxcpm-cpp_b200")
sys.path.insert(0, PKG)

import build as B  # noqa: E402
import vcpm_b200 as vb  # noqa: E402


@pytest.fixture(scope="module")
def layout():
    if not os.path.exists(B.LIB):
        pytest.skip("libvcpm_b200.so is not built")
    exe = B.build_host()
    r = subprocess.run([exe, "layout"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    return json.loads(r.stdout)


@pytest.mark.parametrize("c_name,py_cls", [
    ("vb_lm_config", vb.LMConfig), ("vb_layer_host", vb.LayerHost), ("vb_dit_config", vb.DiTConfig),
    ("vb_dit_host", vb.DiTHost), ("vb_gemv_op", vb.GemvOp), ("vb_gen_parts", vb.GenParts),
    ("vb_vae_config", vb.VAEConfig),
])
def test_struct_layouts_match_ctypes(layout, c_name, py_cls):
    import ctypes
    assert layout[c_name] == ctypes.sizeof(py_cls)
    checked = 0
    for key, off in layout.items():
        if key.startswith(c_name + "."):
            field = key.split(".", 1)[1]
            assert getattr(py_cls, field).offset == off, key
            checked += 1
    assert checked > 0


def test_vae_slot_count(layout):
    assert layout["VB_VAE_N_SLOTS"] == vb.VAE_N_SLOTS


def test_usage_errors(layout):
    exe = B.HOST_BIN
    assert subprocess.run([exe], capture_output=True, timeout=60).returncode == 2
    assert subprocess.run([exe, "run", "0"], capture_output=True, timeout=60).returncode == 2
