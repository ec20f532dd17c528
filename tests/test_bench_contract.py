"""bench.py's reference arm runs on the host cores, so its JSON line (the
contract the harness reads) can be checked without a GPU."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("workload", ["config2", "config4", "config2d64"])
def test_reference_arm_json_line(workload):
    extra = ["--ref-config1"] if workload == "config2" else []
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", workload,
                        "--steps", "1", "--warmup", "1", "--ref-seqs", "2", *extra], cwd=ROOT, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["higher_is_better"] is True
    # the reference's own ref_attention when baseline/_ref holds the install, else the oracle port
    ref_installed = os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "fskernels"))
    assert line["cpu_baseline"]["kind"] == ("reference" if ref_installed else "port")
    assert line["cpu_baseline"]["cores"] >= 1 and line["config"]["same_config"] is False
    if workload == "config2" and ref_installed:
        c1 = line["config1_full"]
        assert c1["ms_per_call"] > 0 and len(c1["lens"]) == 4
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["config"]["workload"].startswith("config")
