"""CPU: the reference arm of bench.py (the oracle timed on the host cores) runs
and prints one JSON line in the contract's shape, for the decode step, the KV
hand-off and the prefill KV write. One or two short steps each."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(*args):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *args],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


@pytest.mark.parametrize("args", [["--steps", "1", "--warmup", "0"],
                                  ["--op", "handoff", "--steps", "1", "--warmup", "0"],
                                  ["--op", "prefill", "--steps", "2", "--warmup", "1"]])
def test_reference_arm_line(args):
    j = run_bench(*args)
    assert j["impl"] == "reference" and j["unit"] == "GB/s" and j["value"] > 0
    assert j["higher_is_better"] is True and j["n_gpus"] == 1
    cb = j["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == pytest.approx(j["value"], rel=1e-3)
    assert j["e2e"]["h2d_bytes_per_step"] == 0 and j["e2e"]["d2h_bytes_per_step"] == 0
