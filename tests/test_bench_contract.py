"""bench.py's reference arm on the CPU: the JSON line the driver reads (metric, value, unit, config, impl,
cpu_baseline, e2e with no host-device bytes), rank 0 only, and no product library loaded in its process
(its dataset comes from the oracle library's copy of the scene renderer)."""
import json
import os
import pathlib
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]

# Runs the reference arm in this process, then reports whether libnerf_b200.so was ever mapped.
RUNNER = r"""
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0", "--reference-seconds", "1",
            "--skip-reference-cuda", "--views", "2"]
runpy.run_path("bench.py", run_name="__main__")
maps = open("/proc/self/maps").read()
print("MAPPED_PRODUCT_LIB", "libnerf_b200.so" in maps)
"""


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, "-c", RUNNER], cwd=str(ROOT), env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout


def test_reference_arm_line_and_no_product_library():
    out = _run({"RANK": "0", "WORLD_SIZE": "1"})
    lines = [json.loads(x) for x in out.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference"
    assert d["metric"] == "train samples/s (config 2, steady state)" and d["unit"] == "samples/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["steps"] == 1 and d["warmup"] == 0 and d["data"] == "synthetic"
    assert d["config"]["workload"].startswith("config2 bounded training")
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["unit"] == "samples/s"
    assert cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "MAPPED_PRODUCT_LIB False" in out


def test_reference_arm_prints_nothing_on_other_ranks():
    out = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert not [x for x in out.splitlines() if x.startswith("{")]
