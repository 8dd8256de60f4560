"""The reference arm of bench.py on CPU: `bench.py --impl reference` times the
reference's own CLI build (oracle/_ref, compiled from its sources) on the host
cores and prints one JSON line in the same contract as the GPU arm. Run here on
a tiny synthetic model so it takes seconds; the driver runs it on the full
Qwen3 shape."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


@pytest.mark.skipif(bench.reference_binary() is None, reason="oracle/_ref was not built on this machine")
def test_reference_arm_prints_the_contract_line():
    # run the arm, then list the shared objects its process mapped: none of this
    # repository's libraries may be among them (the arm times the reference alone)
    driver = ("import runpy, sys; sys.argv = %r; runpy.run_path(%r, run_name='__main__'); "
              "maps = open('/proc/self/maps').read(); "
              "print('MAPPED', sorted({l.split()[-1] for l in maps.splitlines() if '.so' in l}))"
              % (["bench.py", "--impl", "reference", "--config", "tiny-qwen3", "--steps", "2",
                  "--warmup", "3", "--tokens", "32", "--depth", "64"], os.path.join(ROOT, "bench.py")))
    out = subprocess.run([sys.executable, "-c", driver], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert "workload" in d["config"]
    mapped = [l for l in out.stdout.splitlines() if l.startswith("MAPPED")]
    assert mapped and "libember_b200" not in mapped[0] and "liboracle" not in mapped[0], mapped
    # the same workload object as this library's arm, so the two lines compare
    assert d["config"] == bench._workload_config(
        type("A", (), {"config": "tiny-qwen3", "tokens": 32, "depth": 64, "kv_fp16": False})(), 1)
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
