"""The reference arm of bench.py on the CPU: `--impl reference` times the
CPU restatement of ggml's Q8_0 GEMV on the host cores and prints one JSON
line on the headline metric and config (no GPU involved), and under
torchrun only rank 0 works and prints."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    return r


def test_reference_arm_prints_the_contract_line():
    r = _run({"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "Q8_0 GEMV GB/s" and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 3
    assert d["value"] > 0 and d["value"] == d["cpu_baseline"]["value"] == d["e2e"]["value"]
    base = d["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["unit"] == "GB/s" and base["sample"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["arm"].startswith("oracle port")
    assert d["config"]["M"] == 1 and d["config"]["layers"] == 28 and len(d["config"]["shapes"]) == 7


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]
