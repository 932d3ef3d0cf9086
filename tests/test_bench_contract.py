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
    assert set(c["pieces"]) == {"chain_per_chunk", "ring_per_strip"}
    a = argparse.Namespace(config=2, n=16384, phi=1.0)
    c = bench.workload_config(a, 25, 1)
    assert (c["m"], c["n"], c["k"], c["phi"], c["parallelism"]) == (16384, 16384, 16384, 1.0, "single GPU")
    assert "pieces" not in c


def _gate_worker(rank, world, port, plant, q):
    import os
    import traceback

    try:
        import numpy as np
        import torch
        import torch.distributed as dist

        sys.path.insert(0, str(REPO))
        import bench
        from oracle import ozaki_oracle as oo

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(3)
        m, k, n = 40, 96, 70
        A = (rng.random((world * m, k)) - 0.5) * np.exp(rng.standard_normal((world * m, k)))
        B = (rng.random((k, n)) - 0.5) * np.exp(rng.standard_normal((k, n)))
        A_local = A[rank * m:(rank + 1) * m]
        C = oo.ozaki2_matmul(A_local, B)
        if plant and rank == world - 1:
            C[-1, -1] = np.nextafter(C[-1, -1], np.inf)  # one ulp off in the last row and column
        try:
            res = bench.parity_gate(torch, dist, torch.from_numpy(A_local),
                                    torch.from_numpy(B) if rank == 0 else None, torch.from_numpy(C), n, k,
                                    world, rank, 0, torch.device("cpu"))
            q.put((rank, "ok", res["status"]))
        except RuntimeError as exc:
            q.put((rank, "raised", str(exc)))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def _run_gate(plant, world=2):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s_:
        s_.bind(("127.0.0.1", 0))
        port = s_.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gate_worker, args=(r, world, port, plant, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict((r, (st, msg)) for r, st, msg in (q.get(timeout=120) for _ in range(world)))
    for p in procs:
        p.join(timeout=30)
    return out


def test_parity_gate_passes_on_correct_shards_and_raises_everywhere_on_one_ulp():
    """The bench's post-timing gate on 2 gloo ranks: exact shards pass; one ulp
    planted in the last rank's last row and column makes every rank raise."""
    good = _run_gate(plant=False)
    assert all(st == "ok" and msg == "bit-exact" for st, msg in good.values()), good
    bad = _run_gate(plant=True)
    assert all(st == "raised" for st, _ in bad.values()), bad


def test_host_buffer_numa_placement_helpers():
    """The e2e loop's NUMA placement: cpulist parsing, and a GPU with no node in
    sysfs (or no such PCI device here) leaves the affinity untouched."""
    import os

    sys.path.insert(0, str(REPO))
    import bench

    assert bench._cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert bench._cpulist("") == set()

    class Props:
        pci_domain_id, pci_bus_id, pci_device_id = 0xFFFF, 0xFF, 0x1F

    class FakeTorch:
        class cuda:
            @staticmethod
            def get_device_properties(dev):
                return Props()

    before = os.sched_getaffinity(0)
    placement = bench.near_gpu(FakeTorch, 0)
    with placement:
        assert os.sched_getaffinity(0) == before
    assert placement.describe() == {"node": None, "cpus": 0}
    assert os.sched_getaffinity(0) == before
