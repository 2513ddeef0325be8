"""bench.py's reference arm (the oracle on the host cores) prints one JSON line with the contract's keys, for the
decode, prefill and LM-head workloads; CPU only, bounded samples."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e")


@pytest.mark.parametrize("extra", [[], ["--mode", "prefill"], ["--mode", "lmhead"]], ids=["decode", "prefill", "lmhead"])
def test_reference_arm_json_line(extra):
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1", *extra],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in KEYS:
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["unit"] == ("us" if "lmhead" in extra else "TOPS")
    assert d["higher_is_better"] is ("lmhead" not in extra)
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    assert "workload" in d["config"]
