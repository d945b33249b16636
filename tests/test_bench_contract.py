"""bench.py's output contract, on the CPU through its reference arm: stdout is exactly one
JSON line carrying the keys a driver reads (metric, value, unit, n_gpus, steps, warmup,
ms_per_step, higher_is_better, config.workload, impl, cpu_baseline, e2e). The b200 arm
prints the same keys plus roofline, clocks and gpu_launches; it needs a GPU."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "impl",
        "cpu_baseline", "e2e")


def _run(*args):
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                        "--steps", "3", "--warmup", "3", "--cpu-seconds", "1", *args],
                       cwd=REPO, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout[-2000:]
    return json.loads(lines[0])


@pytest.mark.parametrize("workload", ["kda_prefill", "moe"])
def test_reference_arm_prints_one_json_line(workload):
    d = _run("--workload", workload)
    for k in KEYS:
        assert k in d, k
    assert d["impl"] == "reference" and d["n_gpus"] == 1
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["workload"]


def test_reference_arm_threads_ignore_launcher_omp_setting():
    """torchrun exports OMP_NUM_THREADS=1; the CPU arm sets its own thread count (one per
    physical core it may run on), so the figure at N > 1 is taken like the one at N = 1."""
    import psutil
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                        "--workload", "moe", "--steps", "3", "--warmup", "3", "--cpu-seconds", "1"],
                       cwd=REPO, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])
    aff = len(os.sched_getaffinity(0))
    want = max(1, min(aff, psutil.cpu_count(logical=False) or aff))
    assert d["cpu_baseline"]["cores"] == want


def test_stack_mode_selection():
    """--gpus N at batch 1 (the driver's scaling run) keeps Mode R; a batch that splits
    over the ranks takes Mode A under --ep-mode auto; one that does not is refused."""
    import argparse
    sys.path.insert(0, REPO)
    import bench

    def args(batch, mode="auto"):
        return argparse.Namespace(batch=batch, ep_mode=mode)

    assert not bench.stack_mode_a(args(1), 8)
    assert not bench.stack_mode_a(args(64), 1)
    assert bench.stack_mode_a(args(64), 2)
    assert not bench.stack_mode_a(args(64, "r"), 2)
    assert bench.stack_mode_a(args(8, "a"), 8)
    with pytest.raises(SystemExit):
        bench.stack_mode_a(args(3), 2)
