"""bench.py's reference arm (`--impl reference`: the reference's own CPU path on the host cores)
run the way the benchmark driver runs it, in a fresh interpreter, on the small synthetic
package: it must print one JSON line with the contract's keys and a positive rate. (The arm
once failed at import in a fresh interpreter while every in-process test passed.)"""
import json
import os
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_prints_its_line(tmp_path):
    env = dict(os.environ, XQ_BENCH_DIR=str(tmp_path))
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--preset", "small",
                        "--steps", "1", "--warmup", "1"], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "tok/s" and line["higher_is_better"]
    assert line["value"] > 0 and line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] in ("reference", "port") and line["cpu_baseline"]["cores"] >= 1
    assert "small preset" in line["config"]["workload"]
