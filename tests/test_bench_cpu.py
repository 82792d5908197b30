"""bench.py's reference arm runs on host cores only, so its JSON line can be
checked here: the keys the benchmark contract names, a positive throughput,
and the rule that under torchrun only rank 0 runs and prints (the other ranks
exit 0 without work). Uses the small gmm100k-d128 workload (its graph is built
on the host on first use and cached).
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env=None, timeout=600):
    env = dict(os.environ)
    env.update(extra_env or {})
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "gmm100k-d128",
           "--steps", "2", "--warmup", "1", "--batch", "600"]
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    r = _run()
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["steps"] == 2 and line["warmup"] == 1 and line["n_gpus"] == 1
    assert line["higher_is_better"] is True and line["unit"] == "queries/s"
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert "gmm100k-d128" in line["config"]["workload"] and line["config"]["ef"] == 50
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == line["value"] and cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_silently():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_cpu_baseline_fields_and_bound():
    """The CPU baseline of the GPU arm: median of its rounds, a one-thread rate,
    the CPU model, and a wall time close to the budget it is given."""
    import time
    import types

    sys.path.insert(0, ROOT)
    import bench

    args = types.SimpleNamespace(workload="gmm100k-d128", batch=1000, build_device=None, quant="sq4", k=10, ef=50,
                                 rr=8)
    base, qs, g = bench.load_workload(args, 0)
    t0 = time.perf_counter()
    cb = bench.cpu_baseline(args, base, g, qs, 0, budget_s=2.0, rounds=5)
    wall = time.perf_counter() - t0
    assert cb["kind"] == "port" and cb["unit"] == "queries/s" and cb["cores"] == cb["nproc"] >= 1
    assert len(cb["rounds_qps"]) == 5 and cb["rounds_qps"] == sorted(cb["rounds_qps"])
    assert cb["value"] > 0 and abs(cb["value"] - cb["rounds_qps"][2]) <= 0.05
    assert cb["single_thread_qps"] > 0 and cb["cpu_model"]
    assert wall < 30


def test_reference_arm_never_loads_the_engine_library():
    """The reference arm times the oracle port only: the engine's CUDA library
    is never mapped into its process (the index is read by the oracle's own
    ANNX reader and, when missing, built by oracle/_build/libhostbuild.so)."""
    code = (
        "import sys, io, contextlib\n"
        f"sys.path.insert(0, {ROOT!r})\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'gmm100k-d128', '--steps', '1', '--warmup', '0',"
        " '--batch', '200']\n"
        "import bench\n"
        "with contextlib.redirect_stdout(io.StringIO()):\n"
        "    assert bench.main() == 0\n"
        "maps = open('/proc/self/maps').read()\n"
        "assert 'liboracle.so' in maps\n"
        "print('libraven_gpu.so' in maps)\n"
    )
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().splitlines()[-1] == "False"
