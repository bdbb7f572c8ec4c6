#!/usr/bin/env python
"""Benchmark of the B200 Gram Newton-Schulz path (one JSON line on rank 0).

Headline workload: per GPU, a batch of 64 matrices 1024 x 4096 in bf16, entries
N(0, 1) * 1e-2 (seeded), orthogonalised with the default polar-express
coefficients and a Gram reset at iteration 2. One step is one
``GramNewtonSchulz(ns_backend="b200")`` call over the batch. Inputs are 512 MiB
per GPU, larger than the 126 MB L2, so no flush is needed between steps.

* ``value``: matrices/s over all ranks, inputs resident in HBM, device time
  (CUDA events, max over ranks).
* ``e2e``: the same call through the public API with a pinned-host input copied
  in and the result copied back every step; each step's batch travels in four
  pieces pipelined over copy-in, compute and copy-out streams.
* ``roofline``: algorithmic flops of every tcgen05 GEMM launch / their CUDA-event
  time (measured in a second pass of the same steps), against the measured bf16
  peak.
* ``gpu_comparison``: the reference's torch backend (fp16 ``@`` / ``baddbmm``
  on cuBLAS, newton_schulz.py:107-206 over kernels/torch_ns.py:5-35) restated
  here and timed on the same GPU and batch.
* ``cpu_baseline``: the reference's torch path restated with torch CPU ops
  (oracle/gns_torch_port.py, bit-identical to the reference on the CPU) on a
  bounded sample, all host threads, rank 0, N = 1.
* ``workloads``: the optimizer steps and the latency case, measured at the same
  N (bench_workloads.py): the Llama-3-8B-shaped Muon step (round-robin owners
  across the ranks), the 16 x 4096^2 Dion3 step, the column-sharded 8192 x 65536
  orthogonalisation, at N > 1 a DDP training step with and without Muon's
  momentum communication hook, and the 1 x 128 x 256 latency.

``--impl reference`` times the reference's CPU path (the same torch CPU
restatement) on the host cores and prints its own line with this arm's config.
Multi-GPU: launched with torchrun, one rank per GPU; every rank orthogonalises
its own batch of 64 (the batch-sharded layout, no collective in the timed
region) for ``value``: weak scaling. The workloads' Muon, Dion3 and
column-sharded steps do use collectives across the ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH, ROWS, COLS, SCALE, SEED = 64, 1024, 4096, 1e-2, 0
M_DIM, N_DIM = min(ROWS, COLS), max(ROWS, COLS)
FLOPS_PER_MATRIX = 6 * M_DIM**2 * N_DIM + 14 * M_DIM**3  # algorithmic, symmetry-exploiting
KERNELS_PER_STEP = 1 + 18  # normalisation (1) + tcgen05 GEMMs (18)
E2E_CHUNKS = 4  # pieces per end-to-end step, pipelined over copy-in / compute / copy-out streams
CPU_SAMPLE = 8  # matrices per CPU-baseline step
METRIC = "NS matrices/s"
UNIT = "matrices/s"
WORKLOAD = (
    "batched Gram Newton-Schulz, 64 x (1024 x 4096) bf16 per GPU, N(0,1)*1e-2 seed 0, "
    "polar-express coefficients, reset at iteration 2"
)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None, help="timed steps (default 200; workloads: their own)")
    p.add_argument("--warmup", type=int, default=None, help="warm-up steps (default 10)")
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--e2e-steps", type=int, default=5)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-workloads", action="store_true", help="headline only (no optimizer steps)")
    p.add_argument(
        "--workload",
        choices=("cfg2", "cfg1", "muon8b", "dion3", "colshard", "ddp"),
        default="cfg2",
        help="cfg2 (default): batched GNS matrices/s with every workload attached; cfg1: single "
        "128x256 fp32 GNS latency; muon8b: Muon step on Llama-3-8B shapes; dion3: Dion3 step on "
        "16 x 4096^2 fp32; colshard: one 8192 x 65536 bf16 GNS with its columns split over the ranks; "
        "ddp: backward + Muon.step under DistributedDataParallel with and without the momentum hook (N > 1)",
    )
    args = p.parse_args()
    args.steps_given = args.steps is not None
    args.warmup_given = args.warmup is not None
    if args.steps is None:
        args.steps = 200
    if args.warmup is None:
        args.warmup = 10
    return args


def quiet_nccl_banner() -> None:
    """Keeps NCCL's version banner off stdout, where rank 0 prints its one JSON line."""
    if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
        os.environ["NCCL_DEBUG"] = "WARN"


def load_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text()), "measured"
        except json.JSONDecodeError:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def headline_config(world: int) -> dict:
    """The workload description shared by this arm and the reference arm."""
    return {
        "workload": WORKLOAD,
        "batch_per_gpu": BATCH,
        "rows": ROWS,
        "cols": COLS,
        "input_dtype": "bf16",
        "algorithmic_tflop_per_matrix": FLOPS_PER_MATRIX / 1e12,
        "l2": "inputs (512 MiB per GPU) larger than L2; no flush",
        "parallelism": f"batch-sharded x{world} (no collective in the timed region)",
    }


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons of one GPU while running."""

    FIELDS = (
        "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
        "clocks_event_reasons.sw_power_cap"
    )
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu_index = gpu_index
        self.proc: subprocess.Popen | None = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self) -> "ClockSampler":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.out, stderr=subprocess.DEVNULL,
            )
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc: object) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        self.out.flush()
        rows = []
        for line in Path(self.out.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) != 7:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), float(parts[2]), parts[3:]))
            except ValueError:
                continue
        os.unlink(self.out.name)
        if not rows:
            return None
        loaded = [r for r in rows if r[2] > 200.0] or rows
        reasons = sorted(
            {name for r in loaded for name, flag in zip(self.REASONS, r[3]) if flag.lower().startswith("active")}
        )
        return {
            "sm_mhz": statistics.median(r[0] for r in loaded),
            "sm_max_mhz": max(r[1] for r in rows),
            "power_w_max": max(r[2] for r in rows),
            "samples": len(loaded),
            "reasons": reasons,
        }


# ------------------------------------------------------- CPU reference path
def cpu_reference_sample(count: int):
    """`count` matrices of the headline workload's shape and distribution, bf16, on the CPU."""
    import torch

    gen = torch.Generator().manual_seed(SEED)
    return (torch.randn((count, ROWS, COLS), generator=gen) * SCALE).to(torch.bfloat16)


def cpu_reference_steps(steps: int, warmup: int) -> tuple[float, int]:
    """Seconds for `steps` CPU steps of CPU_SAMPLE matrices each through the
    reference's torch path restated on torch CPU ops; returns (seconds, threads)."""
    import torch

    from oracle import gns_torch_port

    torch.set_num_threads(os.cpu_count() or 1)
    coeffs = gns_torch_port_coefficients()
    x = cpu_reference_sample(CPU_SAMPLE)
    for _ in range(warmup):
        gns_torch_port.orthogonalize(x, coeffs)
    t0 = time.perf_counter()
    for _ in range(steps):
        gns_torch_port.orthogonalize(x, coeffs)
    return time.perf_counter() - t0, torch.get_num_threads()


def gns_torch_port_coefficients():
    from gram_newton_schulz_ampere_b200.coefficients import polar_express_coefficients

    return polar_express_coefficients()


def time_cpu_baseline() -> dict:
    """The CPU baseline beside this arm's number: 2 steps of CPU_SAMPLE matrices."""
    elapsed, threads = cpu_reference_steps(2, 1)
    count = 2 * CPU_SAMPLE
    return {
        "value": count / elapsed,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"{count} matrices (2 steps of {CPU_SAMPLE} of the 1024 x 4096 batch) through the reference's "
        f"torch path on torch CPU ops (oracle/gns_torch_port.py), {threads} threads, {elapsed:.2f} s",
    }


# --------------------------------------------- reference backend on the GPU
def torch_backend_chain(x, coefficients, resets=(2,), epsilon=1e-7):
    """The reference's torch backend restated for a timing comparison on this GPU:
    fp32 normalisation to fp16, then fp16 ``@`` / ``torch.baddbmm`` products on
    cuBLAS in the order of newton_schulz.py:122-200, cast back."""
    import torch

    tall = x.size(-2) > x.size(-1)
    xf = x.float()
    xs = (xf / (xf.norm(dim=(-2, -1), keepdim=True) + epsilon)).half()
    del xf

    def gram(m):
        return m.mT @ m if tall else m @ m.mT

    g = gram(xs)
    eye = torch.eye(g.shape[-1], dtype=xs.dtype, device=x.device).unsqueeze(0).expand(g.shape[0], -1, -1).contiguous()
    q = None
    n = len(coefficients)
    for it, (a, b, c) in enumerate(coefficients):
        if it != 0 and it in resets:
            xs = xs @ q if tall else q @ xs
            g = gram(xs)
            q = None
        p = torch.baddbmm(g, g, g, alpha=float(c), beta=float(b))
        q = p.add(eye, alpha=float(a)) if q is None else torch.baddbmm(q, q, p, beta=float(a))
        if it < n - 1 and it + 1 not in resets:
            gp = torch.baddbmm(g, g, p, beta=float(a))
            g = torch.baddbmm(gp, p, gp, beta=float(a))
    return (xs @ q if tall else q @ xs).to(x.dtype)


def time_gpu_comparison(x, device, steps: int = 5, warmup: int = 2) -> dict:
    import torch

    coeffs = gns_torch_port_coefficients()
    for _ in range(warmup):
        torch_backend_chain(x, coeffs)
    torch.cuda.synchronize(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        torch_backend_chain(x, coeffs)
    stop.record()
    stop.synchronize()
    ms = start.elapsed_time(stop) / steps
    return {
        "value": x.shape[0] / (ms * 1e-3),
        "unit": UNIT,
        "ms_per_step": ms,
        "steps": steps,
        "kind": "the reference's torch backend (fp16 cuBLAS products, newton_schulz.py:107-206 over "
        "kernels/torch_ns.py:5-35) restated in bench.py, same batch, same GPU, inputs resident",
    }


# ---------------------------------------------------------- end to end
def time_e2e(ns, host_in, host_out, steps: int, device, barrier, chunks: int = E2E_CHUNKS) -> float:
    """Milliseconds for `steps` end-to-end steps: every step copies its whole input
    from pinned host memory, orthogonalises it through the public API and copies the
    result back. Each step's batch goes through in `chunks` pieces on three streams
    (host-to-device, compute, device-to-host), so the two PCIe directions and the
    GPU work overlap, as a streaming caller would arrange it."""
    import torch

    n = host_in.shape[0]
    bounds = [(n * c // chunks, n * (c + 1) // chunks) for c in range(chunks)]
    s_in, s_comp, s_out = (torch.cuda.Stream(device) for _ in range(3))
    slots = 2
    dev_in = [torch.empty_like(host_in[: bounds[0][1]], device=device) for _ in range(slots)]
    h2d_done = [torch.cuda.Event() for _ in range(slots)]
    comp_done = [torch.cuda.Event() for _ in range(slots)]
    out_done = [torch.cuda.Event() for _ in range(slots)]

    def run(nsteps: int) -> None:
        items = [(step, c) for step in range(nsteps) for c in range(chunks)]
        for i, (_, c) in enumerate(items):
            lo, hi = bounds[c]
            k = i % slots
            buf = dev_in[k][: hi - lo]
            if i >= slots:
                s_in.wait_event(comp_done[k])  # the compute of item i - slots has read this slot
            with torch.cuda.stream(s_in):
                buf.copy_(host_in[lo:hi], non_blocking=True)
                h2d_done[k].record(s_in)
            s_comp.wait_event(h2d_done[k])
            if i >= slots:
                s_comp.wait_event(out_done[k])
            with torch.cuda.stream(s_comp):
                out = ns(buf)
                comp_done[k].record(s_comp)
            s_out.wait_event(comp_done[k])
            with torch.cuda.stream(s_out):
                host_out[lo:hi].copy_(out, non_blocking=True)
                out.record_stream(s_out)
                out_done[k].record(s_out)

    cur = torch.cuda.current_stream(device)
    for st in (s_in, s_comp, s_out):
        st.wait_stream(cur)
    run(1)
    for st in (s_in, s_comp, s_out):
        cur.wait_stream(st)
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(cur)
    for st in (s_in, s_comp, s_out):
        st.wait_stream(cur)
    run(steps)
    for st in (s_in, s_comp, s_out):
        cur.wait_stream(st)
    stop.record(cur)
    stop.synchronize()
    return start.elapsed_time(stop)


def run_reference(args: argparse.Namespace) -> None:
    """``--impl reference``: the reference's CPU path on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    elapsed, threads = cpu_reference_steps(args.steps, args.warmup)
    value = args.steps * CPU_SAMPLE / elapsed
    sample = (
        f"each step orthogonalises {CPU_SAMPLE} matrices of the 64-matrix 1024 x 4096 batch (same shape, "
        "distribution and coefficients) through the reference's torch path restated with torch CPU ops "
        f"(oracle/gns_torch_port.py; bit-identical to the reference on the CPU), {threads} threads; the "
        "metric is per matrix, so the 8-matrix sample measures the same per-matrix rate"
    )
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * elapsed / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": headline_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def recorded_traffic() -> dict | None:
    """DRAM bytes per GEMM launch of a batch-64 chain from the committed ncu
    summary (profiles/gemm_tc_kernel_cfg2.md), with the commit it was captured at."""
    tfile = ROOT / "profiles" / "gemm_tc_kernel_cfg2.md"
    if not tfile.exists():
        return None
    found: dict[str, str] = {}
    for text_line in tfile.read_text().splitlines():
        for key in ("traffic_bytes_per_launch_batch64", "traffic_capture_commit"):
            if text_line.startswith(key + ":"):
                found[key] = text_line.split(":", 1)[1].strip()
    if "traffic_bytes_per_launch_batch64" not in found:
        return None
    return {
        "bytes": int(found["traffic_bytes_per_launch_batch64"]),
        "source": "ncu dram__bytes_read.sum + dram__bytes_write.sum averaged over the 18 GEMM launches of one "
        f"batch-64 chain, profiles/gemm_tc_kernel_cfg2.md, captured at commit "
        f"{found.get('traffic_capture_commit', 'unknown')} (not measured by this run)",
    }


# ------------------------------------------------------------------- GPU
def main() -> None:
    args = parse_args()
    if args.workload != "cfg2":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the headline workload"}))
            return
        from bench_workloads import run_workload

        run_workload(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")

    import torch
    import torch.distributed as dist

    from gram_newton_schulz_ampere_b200 import GramNewtonSchulz, _native

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        quiet_nccl_banner()
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)

    gen = torch.Generator(device=device).manual_seed(SEED + rank)
    x = (torch.randn((BATCH, ROWS, COLS), generator=gen, device=device) * SCALE).to(torch.bfloat16)
    ns = GramNewtonSchulz(ns_backend="b200")

    def barrier() -> None:
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        out = ns(x)
    barrier()

    # ---- device-timed region (inputs resident)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        time.sleep(1.0)  # nvidia-smi needs a moment before its first sample
        start.record()
        for _ in range(args.steps):
            out = ns(x)
        stop.record()
        stop.synchronize()
    elapsed_ms = start.elapsed_time(stop)
    barrier()

    # ---- the same steps again with a CUDA event pair around every GEMM launch
    # (kernel durations for the roofline; kept out of the timed region above)
    prof_steps = min(args.steps, 50)
    capacity = prof_steps * 24 + 16
    _native.profile_enable(capacity)
    for _ in range(prof_steps):
        out = ns(x)
    launches = _native.profile_collect(capacity)
    barrier()
    status = _native.device_status(clear=True)
    if status != 0:
        raise SystemExit(f"a kernel's bounded wait gave up (device status {status})")
    elapsed = torch.tensor([elapsed_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    elapsed_ms = float(elapsed.item())

    # ---- end-to-end through the public API with host buffers
    host_in = x.cpu().pin_memory()
    host_out = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    e2e_ms = time_e2e(ns, host_in, host_out, args.e2e_steps, device, barrier)
    e2e_ms = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())
    io_bytes = x.numel() * x.element_size()
    del host_in, host_out

    gpu_comparison = time_gpu_comparison(x, device)
    del x, out
    torch.cuda.empty_cache()
    barrier()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = time_cpu_baseline()
    barrier()

    workloads = None
    if not args.no_workloads:
        from bench_workloads import measure_cfg1, measure_colshard, measure_ddp_step, measure_dion3, measure_muon

        workloads = {}
        for name, measure in (("muon_step", measure_muon), ("dion3_step", measure_dion3),
                              ("colshard", measure_colshard), ("ddp_step", measure_ddp_step),
                              ("cfg1_latency", measure_cfg1)):
            workloads[name] = measure(world, rank, local_rank, device)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks, peak_source = load_peaks()
    gemm_ms = sum(m for m, _, _ in launches)
    gemm_flops = sum(f for _, f, _ in launches)
    achieved = gemm_flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else 0.0
    sustained = elapsed_ms > 1000.0
    peak = peaks["bf16_tflops_sustained" if sustained else "bf16_tflops"]
    traffic = recorded_traffic()
    ms_per_step = elapsed_ms / args.steps
    line = {
        "metric": METRIC,
        "value": BATCH * world * args.steps / (elapsed_ms * 1e-3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": headline_config(world),
        "e2e": {
            "value": BATCH * world * args.e2e_steps / (e2e_ms * 1e-3),
            "unit": UNIT,
            "h2d_bytes_per_step": io_bytes,
            "d2h_bytes_per_step": io_bytes,
            "api": "gram_newton_schulz_ampere_b200.GramNewtonSchulz(ns_backend='b200')",
            "pipeline": f"{E2E_CHUNKS} chunks per step over host-to-device, compute and device-to-host streams",
        },
        "gpu_launches": KERNELS_PER_STEP * args.steps,
        "roofline": {
            "bound": "tensor",
            "kernel": "gns::gemm_tc_kernel (all 18 launches per step)",
            "achieved": achieved,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": achieved / peak if peak else None,
            "peak_source": f"{peak_source} {'sustained' if sustained else 'burst'} bf16",
            "gemm_launches": len(launches),
            "profiled_steps": prof_steps,
            "gemm_ms_per_step": gemm_ms / prof_steps,
            "traffic": traffic["bytes"] if traffic else None,
            "traffic_source": traffic["source"] if traffic else None,
            "chain_tflops": BATCH * FLOPS_PER_MATRIX / (ms_per_step * 1e-3) / 1e12,
        },
        "gpu_comparison": gpu_comparison,
        "cpu_baseline": cpu,
        "workloads": workloads,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
