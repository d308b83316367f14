"""bench.py's command line and its CPU reference arm, without a GPU: the arm times the
reference's host implementation of the headline workload and prints one JSON line on
rank 0 with the GPU arm's metric and unit; every other rank exits 0 without work."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BENCH = os.path.join(ROOT, "bench.py")


def run(args, **env):
    e = dict(os.environ, **env)
    return subprocess.run([sys.executable, BENCH] + args, cwd=ROOT, env=e, capture_output=True, text=True,
                          timeout=300)


def test_help_lists_the_workloads():
    r = run(["--help"])
    assert r.returncode == 0, r.stderr
    for w in ("decode", "prefill", "moe", "hadamard"):
        assert w in r.stdout


def test_reference_arm_prints_one_line():
    sys.path.insert(0, ROOT)
    import bench
    r = run(["--impl", "reference", "--steps", "1", "--warmup", "3"], RANK="0")
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_do_nothing():
    r = run(["--impl", "reference", "--steps", "1", "--warmup", "3"], RANK="1")
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""
