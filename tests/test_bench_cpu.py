"""The bench contract of the reference arm (no GPU): `bench.py --impl reference` times the CPU
restatement of the reference's training path and prints one JSON line with the same metric,
unit and config as the GPU arm, a cpu_baseline describing the sample, and an e2e object with no
host-device traffic."""
import json
import os
import subprocess
import sys

from tests.conftest import ROOT


def test_reference_arm_prints_one_contract_line(oracle):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "samples/s"
    # the driver divides the two arms only when their metric strings are identical
    sys.path.insert(0, ROOT)
    import bench
    assert d["metric"] == bench.HEADLINE_METRIC and d["higher_is_better"] is True
    assert d["config"]["workload"] == "config1_train_1024sq_8ch"
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
