#!/usr/bin/env python
"""Benchmark: emulated FP64 TFLOPS (2mnk/t) of Ozaki scheme II at n = 16384.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE.json config 2 at its n = 16384 point): square FP64 A, B with
entries (U(0,1) - 0.5) * exp(phi * N(0,1)), phi = 1, seeded synthetic data,
n_mod = 25 (the reference's choice for k = 16384).  A step is one full
emulated product: split A, split B, fused INT8 GEMM + mod + CRT.  Operands are
2 GiB each (larger than L2), so no flush is needed between steps.

With N > 1 (torchrun, one rank per GPU, NCCL) A is row-sharded over the ranks
and B's residues are broadcast from rank 0; the job is the same n = 16384
product (strong scaling).

`value` times the step on resident inputs (CUDA events, max over ranks);
`e2e` times the public op with the operands copied from pinned host memory
and C copied back inside the timed region.  Rank 0 prints one JSON line.

`--impl reference` times the reference's own CPU path (its torch op sequence
and its compiled crt_reconstruct.cpp) on the host cores, one bounded block of
the same product per step, extrapolated to the full product.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (str(REPO / "fp-emulation_b200"), str(REPO)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "emulated FP64 TFLOPS (2mnk/t) at n=16384, 1/2/4/8 B200; INT8 TC util %"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[2, 3, 4, 5], default=2,
                    help="2: square n x n (the metric's workload); 3: m=131072, k=n=8192 with 1%% of A's rows "
                         "x 2^40; 4: convert()'ed 6 x 4096 MLP forward, batch 16384; 5: Chebyshev D@u, D^2@u "
                         "(N = 2048, 4096 fields) and a DT-PINN training step")
    ap.add_argument("--sweep", action="store_true",
                    help="config 2 over n in {1024..16384} x phi in {0.5, 1, 2}, with cuBLAS DGEMM and the "
                         "reference's own CUDA path (n <= 8192) beside every point; one JSON line per point")
    ap.add_argument("--n", type=int, default=16384, help="config 2 size")
    ap.add_argument("--phi", type=float, default=1.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-extras", action="store_true", help="skip DGEMM/cuBLASLt/CPU side numbers")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffer) leg")
    ap.add_argument("--b-layout", choices=["root", "sharded"], default="root",
                    help="N > 1, the timed product: B held by rank 0 (its residues sent to every rank; default) "
                         "or column-sharded (rank q holds columns [q*n/N, (q+1)*n/N) and the residues are "
                         "all-gathered).  The end-to-end leg at N > 1 always uses the column-sharded public op")
    return ap.parse_args()


def problem_shape(args):
    """(M, N, K) of the workload: config 2 is n x n x n, config 3 is 131072 x 8192 x 8192."""
    if args.config == 3:
        return 131072, 8192, 8192
    return args.n, args.n, args.n


def workload_config(args, n_mod, world, transport=None):
    M, N, K = problem_shape(args)
    if args.config == 3:
        desc = ("BASELINE config 3: m=131072, k=n=8192 FP64 GEMM, N(0,1) entries with 1% of A's rows "
                "(seeded choice) scaled by 2^40")
    else:
        desc = f"BASELINE config 2 point n={N}: square FP64 GEMM, entries (U(0,1)-0.5)*exp({args.phi}*N(0,1))"
    return {
        "workload": desc,
        "m": M, "n": N, "k": K, "n_mod": n_mod, **({"phi": args.phi} if args.config == 2 else {}),
        "l2": f"inputs larger than L2 ({8 * M * K / 2**30:.1f} and {8 * K * N / 2**30:.1f} GiB operands); no flush",
        "parallelism": "single GPU" if world == 1 else (
            f"A row-sharded over {world} GPUs, B residues to every GPU over NVLink "
            f"({transport or os.environ.get('FPEMU_TRANSPORT', 'ce')}"
            f"{'' if 'column-sharded' in str(transport) else ' transport, B on rank 0'}, "
            f"{os.environ.get('FPEMU_BCAST', 'residues')})"),
        **({} if world == 1 else {"pieces": {"chain_per_chunk": int(os.environ.get("FPEMU_CE_PIECES", "8")),
                                             "ring_per_strip": int(os.environ.get("FPEMU_RING_PIECES", "1"))}}),
    }


# ---------------------------------------------------------------- clocks ----

class ClockSampler:
    """nvidia-smi samples of one GPU (by UUID) while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.uuid}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, mx, reasons = [], None, set()
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- helpers -----

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _cpulist(text):
    cpus = set()
    for part in text.strip().split(","):
        if part:
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


class near_gpu:
    """Run a block on the CPUs of the GPU's NUMA node, so that host memory the
    block allocates (pinned buffers of the end-to-end loop) is placed on the
    node whose root complex the GPU hangs off: DMA then never crosses the
    socket link.  The caller's affinity is restored on exit; pages keep their
    placement.  Skipped (node None) where sysfs gives no node for the GPU."""

    def __init__(self, torch, dev):
        self.node, self.cpus = None, set()
        try:
            p = torch.cuda.get_device_properties(dev)
            bdf = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            node = int(Path(f"/sys/bus/pci/devices/{bdf}/numa_node").read_text())
            if node >= 0:
                cpus = _cpulist(Path(f"/sys/devices/system/node/node{node}/cpulist").read_text())
                self.cpus = cpus & os.sched_getaffinity(0)
                self.node = node
        except (OSError, ValueError, AttributeError):
            pass

    def __enter__(self):
        self.saved = os.sched_getaffinity(0)
        if self.cpus:
            os.sched_setaffinity(0, self.cpus)
        return self

    def __exit__(self, *exc):
        os.sched_setaffinity(0, self.saved)
        return False

    def describe(self):
        return {"node": self.node, "cpus": len(self.cpus)}


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {}


def gemm_traffic_per_launch(n):
    """Per-launch DRAM traffic of the GEMM kernel from the committed ncu summary."""
    p = REPO / "profiles" / "gemm_crt_traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d.get(str(n))
    except Exception:
        return None


def synth(torch, rows, cols, phi, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    u = torch.rand(rows, cols, dtype=torch.float64, generator=g, device=device)
    e = torch.randn(rows, cols, dtype=torch.float64, generator=g, device=device)
    return (u - 0.5) * torch.exp(phi * e)


def synth_config3_rows(torch, M, r0, r1, K, seed, device):
    """Rows [r0, r1) of config 3's A: N(0,1), with 1 % of all M rows (a seeded
    choice, the same on every rank) scaled by 2^40."""
    g = torch.Generator(device=device).manual_seed(seed)
    A = torch.randn(r1 - r0, K, dtype=torch.float64, generator=g, device=device)
    scaled = torch.randperm(M, generator=torch.Generator().manual_seed(seed + 7))[: M // 100]
    local = scaled[(scaled >= r0) & (scaled < r1)] - r0
    if local.numel():
        A[local.to(device)] *= 2.0 ** 40
    return A


# ---------------------------------------------------------------- ours -----

def run_ours(args):
    os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep NCCL's version banner off stdout
    import torch
    import torch.distributed as dist

    from fp_emulation import _lib
    from fp_emulation.distributed import ozaki2_int8_matmul_allgather, shard_rows
    from fp_emulation.ozaki import _n_moduli, _res_ld, ozaki2_int8_matmul

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    lib = _lib.load()
    M, n, k = problem_shape(args)
    r0, r1 = shard_rows(M, world, rank)
    m = r1 - r0
    bits = 53
    n_mod = _n_moduli(k, bits)
    ld = _res_ld(k)
    root = 0

    sharded = world > 1 and args.b_layout == "sharded"
    if world > 1 and n % world:
        raise SystemExit(f"n = {n} must be a multiple of the GPU count")
    nb = n // world
    # Every rank draws the same B (one seeded generator), so that the column-sharded
    # layouts below hold the root's values; rank 0 keeps all of it.
    if args.config == 3:
        A = synth_config3_rows(torch, M, r0, r1, k, args.seed + 1 + rank, dev)
        B = torch.randn(k, n, dtype=torch.float64, device=dev,
                        generator=torch.Generator(device=dev).manual_seed(args.seed + 1000))
    else:
        A = synth(torch, m, k, args.phi, args.seed + 1 + rank, dev)
        B = synth(torch, k, n, args.phi, args.seed + 1000, dev)
    B_block = B[:, rank * nb:(rank + 1) * nb].contiguous() if world > 1 else None
    if world > 1 and rank != root and not sharded:
        B = None

    a_res = torch.empty((n_mod, m, ld), dtype=torch.int8, device=dev)
    b_res = torch.empty((n_mod, n, ld), dtype=torch.int8, device=dev) if (world == 1 or rank == root) else None
    re = torch.empty((m,), dtype=torch.int32, device=dev)
    ce = torch.empty((n,), dtype=torch.int32, device=dev)
    colmax = torch.empty((n,), dtype=torch.int64, device=dev)
    C = torch.empty((m, n), dtype=torch.float64, device=dev)
    ws_bytes = lib.fpemu_gemm_workspace_size(m, n, n_mod)
    ws = torch.empty((max(ws_bytes, 256),), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)

    n_steps_events = []
    gemm_timing = []
    dist_ops = None
    if world > 1:
        import fp_emulation.distributed as fdist

        use_ce = fdist.BCAST_MODE == "residues" and fdist.TRANSPORT != "nccl"
        dist_ops = fdist._GpuOps(dev, comm_sms=0 if use_ce else None)
        n_chunks = len(fdist.plan_column_chunks(n))
        product = fdist.rowsharded_product_auto

    last_step = {}

    def step_dist(record):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)] if record else None
        dist_ops.timing = gemm_timing if record else None
        first = len(gemm_timing)
        if ev: ev[0].record(stream)
        if sharded:
            last_step["C"] = fdist.rowsharded_product_allgather(A, B_block, k, bits, n_mod, dist_ops)
        else:
            last_step["C"] = product(A, B, n, k, bits, n_mod, dist_ops, root=root)
        if ev:
            ev[1].record(stream)
            n_steps_events.append(ev + [first, len(gemm_timing)])

    def step(record):
        if world > 1:
            return step_dist(record)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record else None
        if ev: ev[0].record(stream)
        _lib.check(lib.fpemu_split(m, k, A.data_ptr(), A.stride(0), A.stride(1), bits, n_mod, a_res.data_ptr(),
                                   ld, m * ld, re.data_ptr(), None, sp), "split A")
        if ev: ev[1].record(stream)
        if rank == root:
            _lib.check(lib.fpemu_split(n, k, B.data_ptr(), B.stride(1), B.stride(0), bits, n_mod,
                                       b_res.data_ptr(), ld, n * ld, ce.data_ptr(), colmax.data_ptr(), sp),
                       "split B")
        if world > 1:
            dist.broadcast(b_res, src=root)
            dist.broadcast(ce, src=root)
        if ev: ev[2].record(stream)
        _lib.check(lib.fpemu_gemm_crt(m, n, k, n_mod, a_res.data_ptr(), b_res.data_ptr(), ld, n * ld,
                                      re.data_ptr(), ce.data_ptr(), bits, C.data_ptr(), n, 0, ws.data_ptr(),
                                      ws.numel(), sp),
                   "gemm_crt")
        if ev:
            ev[3].record(stream)
            n_steps_events.append(ev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    def sum_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return t.item()

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize(dev)
    code = _lib.device_error(clear=True)
    if code[0]:
        raise RuntimeError(f"device-side failure during warm-up: {code}")

    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(uuid) as clk:
        start.record(stream)
        for _ in range(args.steps):
            step(True)
        end.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    elapsed_ms = max_over_ranks(start.elapsed_time(end))
    code = _lib.device_error(clear=True)
    if code[0]:
        raise RuntimeError(f"device-side failure in the timed region: {code}")
    ms_step = elapsed_ms / args.steps
    parity = parity_gate(torch, dist, A, B, last_step.pop("C") if world > 1 else C, n, k, world, rank, root, dev)
    transport_used = None
    if world > 1:
        transport_used = fdist.TRANSPORT if fdist.BCAST_MODE == "residues" else "nccl"
        if sharded:
            transport_used = "column-sharded B, residues all-gathered by the copy-engine ring"
    flops = 2.0 * M * n * k
    value = flops / (ms_step * 1e-3) / 1e12

    if world == 1:
        split_a_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in n_steps_events)
        split_b_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in n_steps_events)
        gemm_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in n_steps_events)
        int8_ops = 2.0 * m * n * k * n_mod
        stages = {"split_a": round(split_a_ms, 3), "split_b": round(split_b_ms, 3), "gemm_crt": round(gemm_ms, 3)}
    else:
        # Per chunk GEMM launches of the pipelined row-sharded product (this rank).
        gemm_ms = statistics.mean(s_.elapsed_time(e_) for s_, e_, _ in gemm_timing)
        int8_ops = statistics.mean(o for _, _, o in gemm_timing)
        # Where each rank's step goes: before its first chunk GEMM (A's split and the
        # first chunk's transfer), GEMMs, waits between GEMMs, and after the last.
        br = {"fill": [], "gemm": [], "gaps": [], "tail": []}
        for e0, e1, i0, i1 in n_steps_events:
            g = gemm_timing[i0:i1]
            br["fill"].append(e0.elapsed_time(g[0][0]))
            br["gemm"].append(sum(a.elapsed_time(b) for a, b, _ in g))
            br["gaps"].append(sum(g[j - 1][1].elapsed_time(g[j][0]) for j in range(1, len(g))))
            br["tail"].append(g[-1][1].elapsed_time(e1))
        mine = {key: round(statistics.mean(v), 3) for key, v in br.items()}
        mine["step"] = round(statistics.mean(e0.elapsed_time(e1) for e0, e1, _, _ in n_steps_events), 3)
        per_rank = [None] * world
        dist.all_gather_object(per_rank, mine)
        stages = {"gemm_crt_per_chunk": round(gemm_ms, 3), "chunks": n_chunks, "per_rank": per_rank}
    achieved = int8_ops / (gemm_ms * 1e-3) / 1e12
    peaks = measured_peaks()
    # MEASURED_PEAKS.json has no INT8 figure; B200's dense INT8 rate is twice its dense
    # BF16 rate, so the primary denominator is 2x the measured burst cuBLAS bf16 rate.
    # The sustained bf16 figure (measured at the clock a seconds-long bf16 loop holds
    # under the 1 kW cap) sits below what INT8 work reaches -- INT8 draws less power
    # per operation and holds a higher clock -- so it is reported beside it only.
    # When the side numbers run, the fraction of cuBLASLt's INT8 rate on one
    # modulus plane of the same shape, measured in the same process, is added.
    if peaks.get("bf16_tflops"):
        peak, peak_src = 2.0 * peaks["bf16_tflops"], "2 x bf16_tflops (burst) of measured"
        peak_sus = 2.0 * peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    else:
        peak, peak_src = 2.0 * 1590.0, "2 x 1.59 PFLOP/s burst bf16 of fallback"
        peak_sus = 2.0 * 1400.0
    # Our kernels per step and rank.  One GPU: split A, split B (column max +
    # split), the GEMM stage (1 kernel fused, 2 in the split form).  Root-split
    # transports (ce, nccl): split A, split B per chunk on the root (2 kernels), the
    # GEMM stage per chunk.  Rings: split A, and per chunk the strip's 2 split
    # kernels and the GEMM stage.
    if world == 1:
        per_rank = 3 + lib.fpemu_gemm_kernels(m, n)
    else:
        cw = [c1 - c0 for c0, c1 in fdist.plan_column_chunks(n)]
        if sharded:
            sw = fdist.allgather_strip_cols(world)
            cw = [world * min(sw, nb - c0) for c0 in range(0, nb, sw)]
        gk = sum(lib.fpemu_gemm_kernels(m, w) for w in cw)
        if sharded or transport_used == "ce-ring":
            per_rank = 1 + 2 * len(cw) + gk
        else:
            per_rank = 1 + gk + (2 * len(cw) if rank == root else 0)
    launches = int(sum_over_ranks(per_rank * args.steps))

    # ---- end to end through the public op, host buffers ------------------
    e2e = None
    if not args.no_e2e:
        # End to end through the public op, host buffers in and out, pipelined the
        # way a caller streaming products would run it: the inputs of step i+1 are
        # copied host->device (pinned) while step i computes, and step i's C is
        # copied device->host behind it.  Every step still moves its full inputs
        # and its full result across PCIe inside the timed region.
        # One GPU: the public op on A and B.  N GPUs: the column-sharded public op,
        # each rank copying in only its rows of A and its block of B's columns
        # (every GPU's PCIe link carries its share; B whole on one rank would put
        # all of B's bytes through the root's link every step).
        numa = near_gpu(torch, dev)
        with numa:
            A_h = A.cpu().pin_memory()
            B_h = (B if world == 1 else B_block).cpu().pin_memory()
            C_h = [torch.empty((m, n), dtype=torch.float64).pin_memory() for _ in range(2)]
        A_d = [torch.empty_like(A) for _ in range(2)]
        B_d = [torch.empty(tuple(B_h.shape), dtype=torch.float64, device=dev) for _ in range(2)]
        del a_res  # give the public op's own workspace room
        h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        loaded = [torch.cuda.Event() for _ in range(2)]
        consumed = [torch.cuda.Event() for _ in range(2)]
        last = {}

        def load(i):
            b = i % 2
            with torch.cuda.stream(h2d):
                h2d.wait_event(consumed[b])          # the previous step using buffer b is done
                A_d[b].copy_(A_h, non_blocking=True)
                B_d[b].copy_(B_h, non_blocking=True)
                loaded[b].record(h2d)

        def run(i):
            b = i % 2
            stream.wait_event(loaded[b])
            if world == 1:
                Cd = ozaki2_int8_matmul(A_d[b], B_d[b])
            else:
                Cd = ozaki2_int8_matmul_allgather(A_d[b], B_d[b])
            consumed[b].record(stream)
            with torch.cuda.stream(d2h):
                d2h.wait_event(consumed[b])
                C_h[b].copy_(Cd, non_blocking=True)
                Cd.record_stream(d2h)
            last["b"] = b

        def e2e_loop(steps):
            h2d.wait_stream(stream)
            load(0)
            for i in range(steps):
                if i + 1 < steps:
                    load(i + 1)
                run(i)
            stream.wait_stream(d2h)

        e2e_steps = max(3, args.steps // 2)
        e2e_loop(max(2, args.warmup))
        torch.cuda.synchronize(dev)
        barrier()
        s2, t2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(stream)
        e2e_loop(e2e_steps)
        t2.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = max_over_ranks(s2.elapsed_time(t2)) / e2e_steps
        h2d_bytes = sum_over_ranks(A_h.numel() * 8 + B_h.numel() * 8)
        d2h_bytes = sum_over_ranks(C_h[0].numel() * 8)
        e2e = {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOPS",
               "h2d_bytes_per_step": int(h2d_bytes), "d2h_bytes_per_step": int(d2h_bytes),
               "ms_per_step": round(e2e_ms, 3),
               "host_buffers": "pinned, allocated on the GPU's NUMA node" if numa.node is not None
                               else "pinned (no NUMA node reported for the GPU)",
               "numa": numa.describe(),
               "method": ("public op per step" if world == 1 else
                          "column-sharded public op (ozaki2_int8_matmul_allgather) per step: each rank copies in "
                          "its rows of A and its column block of B") +
                         "; H2D of step i+1 and D2H of step i overlap step i's compute"}
        # Sanity guard on the last end-to-end result: a row sample against cuBLAS DGEMM.
        if world == 1:
            b = last["b"]
            rows = torch.arange(0, m, max(1, m // 64))
            ref_rows = (A_d[b][rows.to(dev)] @ B_d[b]).cpu()
            got_rows = C_h[b][rows]
            rel = ((got_rows - ref_rows).abs().max() / ref_rows.abs().max()).item()
            if not rel < 1e-12:
                raise RuntimeError(f"sanity check failed: max rel diff vs DGEMM {rel}")

    extras = {}
    if not args.no_extras:
        extras = side_numbers(torch, dev, A, B if rank == root else None, b_res, m, n, k, n_mod, rank, root,
                              world, args)

    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8", "emulated": "f64", "data": "synthetic (seeded, generated on device)",
            "config": workload_config(args, n_mod, world, transport_used),
            "e2e": e2e,
            "roofline": {"bound": "tensor", "kernel": "ozaki_gemm_kernel (fused INT8 GEMM + mod + CRT)",
                         "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "peak_sustained": round(peak_sus, 1), "frac_sustained": round(achieved / peak_sus, 4),
                         "ops_per_launch": int8_ops, "launch_ms": round(gemm_ms, 3),
                         # measured for the single-GPU launch at n = 16384 (profiles/); the
                         # multi-GPU launches are per column chunk, with no capture of their own
                         "traffic": gemm_traffic_per_launch(n) if args.config == 2 and world == 1 else None},
            "int8_tc_util": round(achieved / peak, 4),
            "stages_ms": stages,
            "parity": parity,
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        out.update(extras)
        i8 = extras.get("int8_cublaslt", {}).get("tops_per_modulus_gemm")
        if i8:
            out["roofline"]["frac_of_cublaslt_int8"] = round(achieved / i8, 4)
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def parity_gate(torch, dist, A_local, B_root, C_local, n, k, world, rank, root, dev):
    """Checker, after the timed region: every rank compares a sampled block of
    its rows of the last step's C -- its first, last and two interior rows, by
    64 columns that include the first and the last -- bit for bit with the CPU
    oracle's product of the same rows of A and columns of B (row and column
    exponents span all of K, so the block of the product is exact).  B's
    sampled columns come from the root.  Any mismatch on any rank raises on
    every rank."""
    import numpy as np

    from oracle import ozaki_oracle as oo

    m = C_local.shape[0]
    rows = sorted({0, m // 3, (2 * m) // 3, m - 1}) if m else []
    cols = sorted(set(np.linspace(0, n - 1, min(n, 64)).round().astype(int).tolist()))
    cols_t = torch.tensor(cols, device=dev)
    if rank == root:
        Bc = B_root.index_select(1, cols_t).contiguous()
    else:
        Bc = torch.empty((k, len(cols)), dtype=torch.float64, device=dev)
    if world > 1:
        dist.broadcast(Bc, src=root)
    ok = True
    if rows:
        rows_t = torch.tensor(rows, device=dev)
        got = C_local.index_select(0, rows_t).index_select(1, cols_t).cpu().numpy()
        want = oo.ozaki2_matmul(A_local.index_select(0, rows_t).cpu().numpy(), Bc.cpu().numpy())
        ok = bool(np.array_equal(got.view(np.int64), want.view(np.int64)))
    bad = torch.tensor([0 if ok else 1], dtype=torch.int32, device=dev)
    if world > 1:
        dist.all_reduce(bad, op=dist.ReduceOp.SUM)
    if bad.item():
        raise RuntimeError(f"parity gate: {bad.item()} rank(s) differ from the oracle on the sampled block")
    return {"status": "bit-exact", "checker": "CPU oracle (oracle/ozaki_oracle.py), after the timed region",
            "sampled": {"ranks": world, "rows_per_rank": len(rows), "cols": len(cols),
                        "rows_rank0": rows if rank == 0 else None, "cols_first_last": [cols[0], cols[-1]]}}


def side_numbers(torch, dev, A, B, b_res, m, n, k, n_mod, rank, root, world, args):
    """cuBLAS DGEMM and cuBLASLt INT8 on the same GPU, and the reference's CPU path
    on this host's cores (rank 0, single GPU only)."""
    out = {}
    if rank == root:
        Bm = B
        for _ in range(2):
            torch.matmul(A, Bm)
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 3
        s.record()
        for _ in range(reps):
            torch.matmul(A, Bm)
        e.record()
        torch.cuda.synchronize(dev)
        dg_ms = s.elapsed_time(e) / reps
        out["dgemm_cublas"] = {"tflops": round(2.0 * m * n * k / (dg_ms * 1e-3) / 1e12, 3), "ms": round(dg_ms, 3),
                               "shape": [m, n, k]}
        # cuBLASLt INT8 (the reference's GEMM backend) on one modulus plane, same shape.
        try:
            a8 = torch.randint(0, 101, (m, k), dtype=torch.int8, device=dev)
            b8 = b_res[0][:, :k]
            bT = b8.t()
            for _ in range(2):
                torch._int_mm(a8, bT)
            torch.cuda.synchronize(dev)
            s.record()
            for _ in range(reps):
                torch._int_mm(a8, bT)
            e.record()
            torch.cuda.synchronize(dev)
            i8_ms = s.elapsed_time(e) / reps
            i8 = 2.0 * m * n * k / (i8_ms * 1e-3) / 1e12
            out["int8_cublaslt"] = {"tops_per_modulus_gemm": round(i8, 1), "ms": round(i8_ms, 3),
                                    "effective_fp64_tflops_at_n_mod": round(i8 / n_mod, 3)}
        except Exception as exc:  # torch._int_mm layout limits
            out["int8_cublaslt"] = {"error": str(exc)[:200]}
    if rank == 0 and world == 1:
        out["cpu_baseline"] = cpu_baseline(args, torch)
    return out


def cpu_baseline(args, torch, r=256, c=256):
    """The reference's CPU path on this host's cores (rank 0, one GPU): one
    bounded sample of the workload (reference_sample), its measured throughput."""
    from oracle.reference_path import crt_kind

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    reference_sample(args, 32, 32)  # warm-up (also loads the compiled CRT)
    flops, secs, est = reference_sample(args, r, c)
    M, N, K = workload_gemms(args)[0][:3]
    return {"value": round(flops / secs / 1e12, 9), "unit": "TFLOPS", "cores": cores, "kind": crt_kind(),
            "sample": f"{r}x{c} block of the {M}x{N}x{K} product (full K), {secs:.1f} s wall, through the "
                      f"reference's torch op sequence + crt_reconstruct.cpp compiled from the reference source; "
                      f"the whole product would take {est / 3600:.2f} h at the block model's extrapolation"}


# ---------------------------------------------------------------- sweep ----

def run_sweep(args):
    """Config 2 over n x phi on one GPU: our one-shot product (split A, split B,
    fused GEMM + CRT through fpemu_ozaki2_dgemm, inputs resident), cuBLAS DGEMM,
    and the reference's own CUDA path where its int32 indices allow (n <= 8192),
    whose result block is compared with ours (max ulp apart)."""
    import numpy as np
    import torch

    from fp_emulation import _lib
    from fp_emulation.ozaki import _n_moduli

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    sizes = [1024, 2048, 4096, 8192, 16384]
    phis = [0.5, 1.0, 2.0]
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    block = 64

    def steps_for(n):
        return max(3, min(50, int(2e3 / (n / 1024) ** 3)))

    ref_points = [{"n": n, "phi": phi, "seed_a": args.seed + 1, "seed_b": args.seed + 1000, "warmup": 2,
                   "steps": min(10, steps_for(n)), "block": block} for n in sizes if n <= 8192 for phi in phis]
    ref = {}
    if not args.no_extras and (REPO / "baseline" / "_ref" / "fp_emulation" / "ozaki.py").exists():
        res = subprocess.run([sys.executable, "-m", "oracle.reference_cuda", json.dumps(ref_points)], cwd=REPO,
                             capture_output=True, text=True, timeout=1800)
        if res.returncode == 0:
            for r in json.loads(res.stdout.strip().splitlines()[-1]):
                ref[(r["n"], r["phi"])] = r
        else:
            ref["error"] = res.stderr[-500:]
    dgemm = {}
    for n in sizes:
        A = torch.randn(n, n, dtype=torch.float64, device=dev)
        for _ in range(2):
            A @ A
        torch.cuda.synchronize(dev)
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = steps_for(n)
        s_.record()
        for _ in range(reps):
            A @ A
        e_.record()
        torch.cuda.synchronize(dev)
        dgemm[n] = s_.elapsed_time(e_) / reps
        del A
    for n in sizes:
        n_mod = _n_moduli(n, 53)
        ws = torch.empty((lib.fpemu_workspace_size(n, n, n, n_mod),), dtype=torch.uint8, device=dev)
        for phi in phis:
            A = synth(torch, n, n, phi, args.seed + 1, dev)
            B = synth(torch, n, n, phi, args.seed + 1000, dev)
            C = torch.empty((n, n), dtype=torch.float64, device=dev)

            def once():
                _lib.check(lib.fpemu_ozaki2_dgemm(n, n, n, A.data_ptr(), n, 1, B.data_ptr(), n, 1, C.data_ptr(), n,
                                                  53, n_mod, ws.data_ptr(), ws.numel(), stream), "ozaki2_dgemm")

            for _ in range(3):
                once()
            torch.cuda.synchronize(dev)
            reps = steps_for(n)
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            for _ in range(reps):
                once()
            e_.record()
            torch.cuda.synchronize(dev)
            ms = s_.elapsed_time(e_) / reps
            code = _lib.device_error(clear=True)
            if code[0]:
                raise RuntimeError(f"device-side failure at n={n}: {code}")
            rec = {"sweep": "config 2", "n": n, "phi": phi, "n_mod": n_mod, "steps": reps, "ms": round(ms, 4),
                   "tflops": round(2.0 * n ** 3 / (ms * 1e-3) / 1e12, 3),
                   "dgemm_cublas": {"ms": round(dgemm[n], 4), "tflops": round(2.0 * n ** 3 / (dgemm[n] * 1e-3) / 1e12, 3)}}
            r = ref.get((n, phi))
            if r is not None and "ms" in r:
                mine = C[:block, :block].cpu().numpy().ravel()
                theirs = np.array([float.fromhex(h) for h in r["block"]])
                ulp = np.abs(mine - theirs) / np.spacing(np.maximum(np.abs(theirs), 1e-300))
                rec["reference_cuda"] = {"ms": r["ms"], "tflops": r["tflops"], "speedup": round(r["ms"] / ms, 2),
                                         "max_ulp_vs_ours_on_64x64_block": float(ulp.max()),
                                         "path": "reference ozaki2_int8_matmul on CUDA tensors: torch split + "
                                                 "cuBLASLt batched INT8 + mod_reduce + crt_kernel"}
            elif r is not None:
                rec["reference_cuda"] = {"skipped": r.get("skipped")}
            elif "error" in ref:
                rec["reference_cuda"] = {"error": ref["error"]}
            print(json.dumps(rec), flush=True)
            del A, B, C
        del ws
        torch.cuda.empty_cache()


# ------------------------------------------------------ configs 4 and 5 -----

def cheb_torch(torch, N, device):
    """Chebyshev-Gauss-Lobatto points and first-derivative matrix on N+1 points
    (the construction of the reference's DT-PINN notebook, in float64)."""
    x = torch.cos(torch.pi * torch.arange(N + 1, dtype=torch.float64, device=device) / N)
    c = torch.ones(N + 1, dtype=torch.float64, device=device)
    c[0] = 2.0
    c[N] = 2.0
    c = c * ((-1.0) ** torch.arange(N + 1, dtype=torch.float64, device=device))
    X = x.unsqueeze(1).expand(N + 1, N + 1)
    D = (c.unsqueeze(1) / c.unsqueeze(0)) / (X - X.T + torch.eye(N + 1, dtype=torch.float64, device=device))
    return x, D - torch.diag(D.sum(dim=1))


def _time(torch, dev, fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_.record()
    for _ in range(steps):
        fn()
    e_.record()
    torch.cuda.synchronize(dev)
    return s_.elapsed_time(e_) / steps


def _pipelined_e2e(torch, dev, x_h, run_fn, steps, warmup, numa):
    """Milliseconds per step of `run_fn` fed from host memory the way a caller
    streaming batches runs it: step i+1's input is copied host->device (pinned,
    one stream) while step i computes, and step i's outputs are copied
    device->host (another stream) behind it; two device input buffers and two
    sets of pinned output buffers alternate.  Every step still moves its whole
    input and all its outputs across PCIe inside the timed region.  Returns the
    time and one set of host outputs."""
    stream = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    x_d = [torch.empty(tuple(x_h.shape), dtype=x_h.dtype, device=dev) for _ in range(2)]
    loaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    outs_h = [None, None]

    def load(i):
        b = i % 2
        with torch.cuda.stream(h2d):
            h2d.wait_event(consumed[b])        # the step that last read x_d[b] is done
            x_d[b].copy_(x_h, non_blocking=True)
            loaded[b].record(h2d)

    def run(i):
        b = i % 2
        stream.wait_event(loaded[b])
        res = run_fn(x_d[b])
        res = res if isinstance(res, tuple) else (res,)
        consumed[b].record(stream)
        if outs_h[b] is None:
            with numa:
                outs_h[b] = [torch.empty(r.shape, dtype=r.dtype).pin_memory() for r in res]
        with torch.cuda.stream(d2h):
            d2h.wait_event(consumed[b])
            for o, r in zip(outs_h[b], res):
                o.copy_(r, non_blocking=True)
                r.record_stream(d2h)

    def loop(n):
        h2d.wait_stream(stream)
        load(0)
        for i in range(n):
            if i + 1 < n:
                load(i + 1)
            run(i)
        stream.wait_stream(d2h)

    loop(max(2, warmup))
    torch.cuda.synchronize(dev)
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_.record(stream)
    loop(steps)
    e_.record(stream)
    torch.cuda.synchronize(dev)
    return s_.elapsed_time(e_) / steps, outs_h[0]


def _blocks_equal(got, want):
    import numpy as np

    return bool(np.array_equal(np.asarray(got).view(np.int64), np.asarray(want).view(np.int64)))


def run_model_config(args):
    """Configs 4 and 5 on one GPU per rank (with torchrun, independent replicas:
    weak scaling).  `value` is emulated FP64 TFLOPS of the step through the public
    API; native FP64 (cuBLAS through torch) is timed beside it."""
    import copy

    import numpy as np
    import torch
    import torch.distributed as dist
    from torch import nn

    from fp_emulation import _lib, convert, ozaki2_int8_matmul, prepare_operand
    from oracle import ozaki_oracle as oo

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    torch.backends.cuda.matmul.allow_tf32 = False
    extras, stages = {}, {}
    if args.config == 4:
        width, depth, batch = 4096, 6, 16384
        torch.manual_seed(args.seed)
        layers = []
        for i in range(depth):
            layers.append(nn.Linear(width, width, dtype=torch.float64))
            if i < depth - 1:
                layers.append(nn.Tanh())
        native = nn.Sequential(*layers).to(dev)
        model = convert(copy.deepcopy(native))
        cached = convert(copy.deepcopy(native), cache_weight_residues=True)
        x = torch.randn(batch, width, dtype=torch.float64, device=dev,
                        generator=torch.Generator(device=dev).manual_seed(args.seed + 1))
        flops = depth * 2.0 * batch * width * width
        with torch.no_grad():
            ms = _time(torch, dev, lambda: model(x), args.steps, args.warmup)
            ms_cached = _time(torch, dev, lambda: cached(x), args.steps, args.warmup)
            ms_native = _time(torch, dev, lambda: native(x), max(2, args.steps // 2), 1)
            # Parity: every layer's GEMM + bias on sampled rows of its own (GPU) input.
            rows = torch.tensor(sorted({0, batch // 2, batch - 1, 12345 % batch}), device=dev)
            h, ok = x, True
            for layer in model:
                out = layer(h)
                if isinstance(layer, nn.Linear):
                    want = oo.ozaki2_matmul(h[rows].cpu().numpy(), layer.weight.T.cpu().numpy()) + \
                        layer.bias.cpu().numpy()
                    ok &= _blocks_equal(out[rows].cpu().numpy(), want)
                h = out
        desc = (f"BASELINE config 4: convert()'ed FP64 MLP, {depth} nn.Linear({width}, {width}) with tanh between "
                f"(Kaiming-uniform init, seed {args.seed}), batch {batch} N(0,1) rows; forward under no_grad")
        extras["cached_weight_residues"] = {"ms": round(ms_cached, 3),
                                           "tflops": round(flops / (ms_cached * 1e-3) / 1e12, 3)}
        parity = {"status": "bit-exact" if ok else "MISMATCH",
                  "checker": "CPU oracle per layer on 4 sampled rows of the layer's own input (GEMM + bias)"}
        e2e_in, e2e_run = x, (lambda xin: model(xin))
    else:
        N, cols = 2048, 4096
        xg, D = cheb_torch(torch, N, dev)
        D2 = D @ D
        g = torch.Generator(device=dev).manual_seed(args.seed + 5)
        a = 1.0 + 7.0 * torch.rand(cols, dtype=torch.float64, device=dev, generator=g)
        u = torch.sin(torch.pi * xg[:, None] * a[None, :]) + \
            0.1 * torch.randn(N + 1, cols, dtype=torch.float64, device=dev, generator=g)
        Dp, D2p = prepare_operand(D, "left"), prepare_operand(D2, "left")
        flops = 2 * 2.0 * (N + 1) * (N + 1) * cols
        ms = _time(torch, dev, lambda: (ozaki2_int8_matmul(Dp, u), ozaki2_int8_matmul(D2p, u)), args.steps,
                   args.warmup)
        ms_unprep = _time(torch, dev, lambda: (ozaki2_int8_matmul(D, u), ozaki2_int8_matmul(D2, u)), args.steps,
                          args.warmup)
        ms_native = _time(torch, dev, lambda: (D @ u, D2 @ u), max(2, args.steps // 2), 1)
        Du, D2u = ozaki2_int8_matmul(Dp, u), ozaki2_int8_matmul(D2p, u)
        rows = torch.tensor(sorted({0, 1, N // 2, N}), device=dev)
        cc_ = torch.tensor(sorted(set(np.linspace(0, cols - 1, 48).round().astype(int).tolist())), device=dev)
        uc = u[:, cc_].cpu().numpy()
        ok = _blocks_equal(Du[rows][:, cc_].cpu().numpy(), oo.ozaki2_matmul(D[rows].cpu().numpy(), uc))
        ok &= _blocks_equal(D2u[rows][:, cc_].cpu().numpy(), oo.ozaki2_matmul(D2[rows].cpu().numpy(), uc))
        desc = (f"BASELINE config 5: Chebyshev-Gauss-Lobatto N={N} ({N + 1} points), D and D^2 = D@D (entries up to "
                f"{D.abs().max().item():.3g}), applied to {cols} fields u = sin(pi x a) + 0.1 N(0,1), a ~ U(1,8); "
                f"step = D@u and D^2@u with D, D^2 prepared once")
        extras["unprepared_operators"] = {"ms": round(ms_unprep, 3),
                                          "tflops": round(flops / (ms_unprep * 1e-3) / 1e12, 3)}
        extras["dt_pinn_train_step"] = dt_pinn_step(torch, dev, args)
        parity = {"status": "bit-exact" if ok else "MISMATCH",
                  "checker": "CPU oracle on 4 rows x 48 columns of D@u and D^2@u"}
        e2e_in, e2e_run = u, (lambda uin: (ozaki2_int8_matmul(Dp, uin), ozaki2_int8_matmul(D2p, uin)))
    if parity["status"] != "bit-exact":
        raise RuntimeError(f"parity gate failed: {parity}")
    code = _lib.device_error(clear=True)
    if code[0]:
        raise RuntimeError(f"device-side failure: {code}")

    # End to end: every step's input from pinned host memory, its outputs back to host.
    numa = near_gpu(torch, dev)
    with numa:
        x_h = e2e_in.cpu().pin_memory()
    with torch.no_grad():
        e2e_ms, outs_h = _pipelined_e2e(torch, dev, x_h, e2e_run, max(3, args.steps // 2), 2, numa)
    d2h = sum(t.numel() * t.element_size() for t in outs_h)

    def total(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        return t.item()

    value = total(flops / (ms * 1e-3) / 1e12)
    e2e_v = total(flops / (e2e_ms * 1e-3) / 1e12)
    if rank == 0:
        out = {"metric": f"emulated FP64 TFLOPS (2mnk/t) of BASELINE config {args.config}",
               "value": round(value, 3), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "int8", "emulated": "f64",
               "data": "synthetic (seeded, generated on device)",
               "config": {"workload": desc, "parallelism": "single GPU" if world == 1 else f"{world} replicas",
                          "l2": "operands larger than L2; no flush" if args.config == 4 else
                                "operands about 100 MB, re-read from L2 between steps"},
               "e2e": {"value": round(e2e_v, 3), "unit": "TFLOPS", "h2d_bytes_per_step": int(total(x_h.numel() * 8)),
                       "d2h_bytes_per_step": int(total(d2h)), "ms_per_step": round(e2e_ms, 3),
                       "method": "public op per step; H2D of step i+1 and D2H of step i overlap step i's compute",
                       "numa": numa.describe()},
               "native_fp64_cublas": {"ms": round(ms_native, 3), "tflops": round(flops / (ms_native * 1e-3) / 1e12, 3)},
               "parity": parity, **extras}
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def dt_pinn_step(torch, dev, args, n_steps=20):
    """One DT-PINN training step for Burgers' equation on the reference notebook's
    40 x 40 Chebyshev grid (05_dt_pinn.ipynb: derivative operators by Kronecker
    products, a 2-256-256-256-1 tanh network, PDE + 10 IC + 10 BC loss, Adam):
    forward, backward and optimizer step, with the network convert()'ed and the
    derivative operators applied as prepared emulated products -- timed against
    the same step in native FP64."""
    from torch import nn

    from fp_emulation import convert, ozaki2_int8_matmul, prepare_operand

    Nx = Nt = 39
    xc, Dx = cheb_torch(torch, Nx, dev)
    tc, Dt = cheb_torch(torch, Nt, dev)
    tc, Dt = 0.5 * (tc + 1), 2 * Dt
    I = torch.eye(Nx + 1, dtype=torch.float64, device=dev)
    DX, DT, DXX = torch.kron(Dx, I), torch.kron(I, Dt), torch.kron(Dx @ Dx, I)
    xx, tt = torch.meshgrid(xc, tc, indexing="ij")
    X = torch.stack([xx.reshape(-1), tt.reshape(-1)], dim=1)
    ic = X[:, 1].abs() < 1e-10
    bc = ((X[:, 0] + 1).abs() < 1e-10) | ((X[:, 0] - 1).abs() < 1e-10)
    nu = 0.01 / torch.pi

    def net():
        torch.manual_seed(args.seed)
        return nn.Sequential(nn.Linear(2, 256), nn.Tanh(), nn.Linear(256, 256), nn.Tanh(), nn.Linear(256, 256),
                             nn.Tanh(), nn.Linear(256, 1)).to(dtype=torch.float64, device=dev)

    ops_fp64 = (DX, DT, DXX)
    ops_oz = tuple(prepare_operand(M, "left") for M in ops_fp64)

    # Index tensors instead of boolean masks: a mask index waits for the host to
    # learn its size, which also rules out CUDA-graph capture.
    ic_idx, bc_idx = ic.nonzero().squeeze(1), bc.nonzero().squeeze(1)
    ic_x = torch.sin(torch.pi * X.index_select(0, ic_idx)[:, 0:1])

    def make(emulated, capturable=False):
        model = convert(net()) if emulated else net()
        opt = torch.optim.Adam(model.parameters(), lr=1e-3, capturable=capturable)
        mm = ozaki2_int8_matmul if emulated else torch.matmul
        ops = ops_oz if emulated else ops_fp64

        def step():
            u = model(X)
            u_x, u_t, u_xx = mm(ops[0], u), mm(ops[1], u), mm(ops[2], u)
            loss = (u_t + u * u_x - nu * u_xx).pow(2).mean() + \
                10 * (u.index_select(0, ic_idx) + ic_x).pow(2).mean() + 10 * u.index_select(0, bc_idx).pow(2).mean()
            opt.zero_grad(set_to_none=False)
            loss.backward()
            opt.step()
            return loss

        return step

    def graphed(emulated):
        """The same step captured once in a CUDA graph and replayed: the
        launch-bound inner loop without host work between the kernels."""
        step = make(emulated, capturable=True)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):  # warm-up on the capturing stream: optimizer state, caches
                step()
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        return g.replay

    ms_oz = _time(torch, dev, make(True), n_steps, 3)
    ms_fp = _time(torch, dev, make(False), n_steps, 3)
    out = {"grid": f"{Nx + 1} x {Nt + 1} Chebyshev points, operators {tuple(DX.shape)}",
           "ms_emulated": round(ms_oz, 3), "ms_native_fp64": round(ms_fp, 3),
           "what": "forward + backward + Adam step; emulated: convert()'ed network and prepared DX, DT, DXX"}
    try:
        out["ms_emulated_cuda_graph"] = round(_time(torch, dev, graphed(True), n_steps, 3), 3)
        out["ms_native_fp64_cuda_graph"] = round(_time(torch, dev, graphed(False), n_steps, 3), 3)
    except Exception as exc:  # a capture the runtime refuses is reported, not fatal
        out["cuda_graph_error"] = str(exc)[:300]
    return out


# ---------------------------------------------------------------- reference arm ---

def workload_gemms(args):
    """The emulated products of one step: [(M, N, K, count)]."""
    if args.config == 3:
        return [(131072, 8192, 8192, 1)]
    if args.config == 4:
        return [(16384, 4096, 4096, 6)]
    if args.config == 5:
        return [(2049, 4096, 2049, 2)]
    return [(args.n, args.n, args.n, 1)]


def reference_sample(args, r=128, c=256):
    """One bounded sample of the workload through the reference's CPU path: for
    each product of the step, an r x c block of C (r full rows of A against c
    full columns of B, full K).  Returns (sample_flops, sample_seconds,
    extrapolated_full_step_seconds)."""
    from oracle.reference_path import block_time, synthetic_block

    flops = secs = est = 0.0
    for M, N, K, count in workload_gemms(args):
        A, B = synthetic_block(K, min(r, M), min(c, N), args.phi, args.seed)
        e, blk, _ = block_time(A, B, M, N)
        flops += 2.0 * A.shape[0] * B.shape[1] * K
        secs += blk
        est += count * e
    return flops, secs, est


def run_reference(args):
    """The reference arm: the reference's own CPU implementation of the path (its
    torch op sequence and its compiled crt_reconstruct.cpp) on all host cores.
    A step is one bounded sample of the workload (reference_sample); `value` is
    the sample's measured throughput and `ms_per_step` its wall time, so the
    line describes exactly the work this run did.  The whole-product time
    extrapolated from the sample is reported beside it."""
    world, rank, _ = dist_env()
    if world > 1 and rank != 0:
        return
    import torch

    from oracle.ozaki_oracle import n_moduli
    from oracle.reference_path import crt_kind

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    M, N, K = workload_gemms(args)[0][:3]
    n_mod = n_moduli(K, 53)
    r, c = 128, 256
    for _ in range(args.warmup):
        reference_sample(args, 16, 16)
    samples = [reference_sample(args, r, c) for _ in range(args.steps)]
    flops = statistics.mean(f for f, _, _ in samples)
    secs = statistics.mean(t for _, t, _ in samples)
    est = statistics.mean(e for _, _, e in samples)
    value = flops / secs / 1e12
    shapes = ", ".join(f"{cnt} x {m_}x{n_}x{k_}" for m_, n_, k_, cnt in workload_gemms(args))
    out = {
        "metric": METRIC if args.config in (2, 3) else f"emulated FP64 TFLOPS (2mnk/t) of BASELINE config {args.config}",
        "value": round(value, 9), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(secs * 1e3, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int32", "emulated": "f64",
        "data": "synthetic (seeded)", "impl": "reference",
        "config": workload_config(args, n_mod, world) if args.config in (2, 3) else {"workload": f"config {args.config}: {shapes}"},
        "cpu_baseline": {"value": round(value, 9), "unit": "TFLOPS", "cores": cores, "kind": crt_kind(),
                         "sample": f"per step, an {r}x{c} block (full K) of each product of the step ({shapes}) "
                                   f"through the reference's CPU op sequence + its crt_reconstruct.cpp: "
                                   f"{secs:.1f} s wall per step; the whole step would take {est / 3600:.2f} h "
                                   f"at the block model's extrapolation"},
        "extrapolated_full_step_s": round(est, 1),
        "e2e": {"value": round(value, 9), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.sweep:
        run_sweep(args)
    elif args.config in (4, 5):
        run_model_config(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
