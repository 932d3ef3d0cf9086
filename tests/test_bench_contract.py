"""The benchmark's reference arm prints the driver's one-line JSON contract
(run here on the CPU at a small size; the GPU arm is exercised on a GPU box)."""
from __future__ import annotations

import json
import subprocess
import sys

from conftest import REPO


def _run(*args):
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), *args], cwd=REPO, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_reference_arm_contract():
    d = _run("--impl", "reference", "--n", "1024", "--steps", "1", "--warmup", "1")
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "TFLOPS" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["steps"] == 1
    assert d["config"]["m"] == d["config"]["n"] == d["config"]["k"] == 1024
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("reference", "port") and cb["sample"]


def test_workload_configs():
    sys.path.insert(0, str(REPO))
    import argparse

    import bench

    a = argparse.Namespace(config=3, n=16384, phi=1.0)
    assert bench.problem_shape(a) == (131072, 8192, 8192)
    c = bench.workload_config(a, 25, 8, "ce")
    assert c["m"] == 131072 and c["k"] == 8192 and "ce transport" in c["parallelism"] and "phi" not in c
    a = argparse.Namespace(config=2, n=16384, phi=1.0)
    c = bench.workload_config(a, 25, 1)
    assert (c["m"], c["n"], c["k"], c["phi"], c["parallelism"]) == (16384, 16384, 16384, 1.0, "single GPU")
