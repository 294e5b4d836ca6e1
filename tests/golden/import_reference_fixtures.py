#!/usr/bin/env python3
"""Imports the reference's golden vectors for this path into tests/golden/.

Run where the voxcpm-cpp tree is available (default ../../../reference or
$VCPM_REFERENCE_DIR).  It copies data only:

* tests/fixtures/{rms_norm_plain,rms_norm_weighted,mlp,attention}_*.bin and
  *_meta.txt -- raw float32 arrays written by the reference's numpy generator
  (tests/fixtures/gen_op_fixtures.py); gated in the reference at cos >= 0.9999
  and RMSE <= 0.01 (tests/test_fixture_parity.c:201,240,315,399).
* the expected values of tests/test_cfm_schedule.c:7-35 (sway schedule and
  CFG-Zero* known answers), parsed from the C source text into JSON.
* the cache-capacity known answers of tests/test_generation_memory.c:14-17.

A sha256 manifest lets tests confirm the copies still match the reference.
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "ref_fixtures")

FIXTURES = [
    "rms_norm_plain_input.bin", "rms_norm_plain_output.bin", "rms_norm_plain_meta.txt",
    "rms_norm_weighted_input.bin", "rms_norm_weighted_output.bin", "rms_norm_weighted_weight.bin",
    "rms_norm_weighted_meta.txt",
    "mlp_input.bin", "mlp_output.bin", "mlp_gate_weight.bin", "mlp_up_weight.bin", "mlp_down_weight.bin",
    "mlp_meta.txt",
    "attention_input.bin", "attention_output.bin", "attention_q_weight.bin", "attention_k_weight.bin",
    "attention_v_weight.bin", "attention_o_weight.bin", "attention_meta.txt",
]


def _floats(text: str) -> list[float]:
    return [float(v.rstrip("f")) for v in re.findall(r"-?\d+\.\d+f?", text)]


def parse_cfm_schedule(src: str) -> dict:
    sched = re.search(r"expected\[11\]\s*=\s*\{(.*?)\};", src, re.S).group(1)
    pos = re.search(r"positive\[4\]\s*=\s*\{(.*?)\};", src, re.S).group(1)
    neg = re.search(r"negative\[4\]\s*=\s*\{(.*?)\};", src, re.S).group(1)
    vel = re.search(r"expected_velocity\[4\]\s*=\s*\{(.*?)\};", src, re.S).group(1)
    scale = re.search(r"scale != ([0-9.]+)f", src).group(1)
    cfg = re.search(r"vcpm_cfm_cfg_zero_star\(negative, positive, 4, ([0-9.]+)f\)", src).group(1)
    return {
        "source": "tests/test_cfm_schedule.c",
        "n_steps": 10,
        "sway_t": _floats(sched),
        "positive": _floats(pos),
        "negative": _floats(neg),
        "cfg_value": float(cfg),
        "expected_velocity": _floats(vel),
        "expected_st_star": float(scale),
    }


def parse_cache_capacity(src: str) -> list[list[int]]:
    cases = re.findall(r"vcpm_gen_round_cache_capacity\((\d+),\s*(\d+)\)\s*==\s*(\d+)", src)
    return [[int(a), int(b), int(c)] for a, b, c in cases]


def main(ref_dir: str) -> int:
    fx = os.path.join(ref_dir, "tests", "fixtures")
    os.makedirs(OUT, exist_ok=True)
    manifest = {}
    for name in FIXTURES:
        shutil.copyfile(os.path.join(fx, name), os.path.join(OUT, name))
        with open(os.path.join(OUT, name), "rb") as f:
            manifest[name] = hashlib.sha256(f.read()).hexdigest()
    with open(os.path.join(ref_dir, "tests", "test_cfm_schedule.c")) as f:
        cfm = parse_cfm_schedule(f.read())
    with open(os.path.join(ref_dir, "tests", "test_generation_memory.c")) as f:
        cap = parse_cache_capacity(f.read())
    kat = {"cfm_schedule": cfm,
           "cache_capacity": {"source": "tests/test_generation_memory.c", "cases": cap},
           "rms_norm_1234": {"source": "tests/test_minicpm4.c", "x": [1.0, 2.0, 3.0, 4.0], "eps": 1e-6, "tol": 2e-3},
           "mlp_identity": {"source": "tests/test_minicpm4.c", "x": [0.5, 1.0, -0.5, 0.0], "hidden": 4, "ffn": 8,
                            "tol": 1e-3},
           "fsq": {"source": "tests/test_phase5.c", "x": [0.0, 0.2, -0.2, 3.0], "scale": 9.0,
                   "expected": [0.0, 2.0 / 9.0, -2.0 / 9.0, 1.0], "tol": 1e-5}}
    with open(os.path.join(HERE, "reference_kat.json"), "w") as f:
        json.dump(kat, f, indent=1)
    with open(os.path.join(OUT, "MANIFEST.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print(f"imported {len(FIXTURES)} fixtures and {len(kat)} known-answer sets into {HERE}")
    return 0


if __name__ == "__main__":
    ref = os.environ.get("VCPM_REFERENCE_DIR") or (sys.argv[1] if len(sys.argv) > 1 else
                                                   os.path.normpath(os.path.join(HERE, "..", "..", "..",
                                                                                 "reference")))
    sys.exit(main(ref))
