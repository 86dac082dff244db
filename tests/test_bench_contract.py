"""bench.py's output contract, checked on the CPU through its reference arm (the reference's own AVX
kernel, or the oracle's restatement where it is not built): one JSON line with the keys the runner
reads, the default workload, and the CPU baseline block."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REQUIRED = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
            "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e")


def run_bench(*args):
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], capture_output=True, text=True, timeout=600,
                       cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_prints_one_contract_line():
    d = run_bench("--impl", "reference", "--steps", "2", "--warmup", "1")
    if "unavailable" in d:
        pytest.skip(d["unavailable"])
    for key in REQUIRED:
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 2 and d["warmup"] == 1
    assert d["metric"] == "ffn_tokens_per_s" and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["config"]["workload"].startswith("cfg4") and d["config"]["m"] == 8192 and d["config"]["layers"] == 80
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] > 0 and cb["cores"] >= 1 and cb["kind"] in ("reference", "port") and cb["sample"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0


def test_help_lists_the_workloads():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--help"], capture_output=True, text=True, cwd=REPO)
    assert r.returncode == 0
    for w in ("cfg0", "cfg1", "cfg2", "cfg3", "cfg4"):
        assert w in r.stdout
