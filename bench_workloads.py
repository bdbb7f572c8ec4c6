"""Secondary benchmark workloads of bench.py (``--workload cfg1|muon8b|dion3|colshard``).

* cfg1: latency of one ``GramNewtonSchulz`` call on a (1, 128, 256) fp32 matrix
  microseconds per call.
* muon8b: one ``Muon.step()`` on a synthetic Llama-3-8B-shaped parameter set
  32 layers x {q, o: 4096x4096, k, v: 1024x4096,
  gate, up: 14336x4096, down: 4096x14336}, bf16 parameters N(0, 0.02), bf16
  gradients N(0, 1e-3) (same seed on every rank: DDP-replicated), lr 3e-3,
  momentum 0.95, Nesterov, spectral-norm lr adjustment. Across N ranks the
  matrices of each shape bucket are round-robined and all-gathered (NCCL).
* dion3: one ``Dion3.step()`` on 16 x (4096 x 4096) fp32 matrices plus 16
  bias vectors in an AdamW group, gradients N(0, 1e-3) times
  a per-row lognormal(sigma = 1) scale, fraction 0.25, momentum 0.95,
  muon_beta2 0.95, weight decay 0.01; replicated across ranks.
* colshard: Gram Newton-Schulz of one 8192 x 65536 bf16 N(0, 1) matrix whose
  columns are split over the N ranks (DTensor ``Shard(1)``):
  the partial-Gram chain (two fp32 all-reduces of the 8192 x 8192 Gram matrix,
  one of the norm). At N = 1 the matrix is whole and goes through the fused
  chain. At N > 1 the line also carries the time of the reference's owner
  scheme (assemble the matrix on one rank with all-to-alls) on the same input.

Each prints one JSON line on rank 0 with device time (CUDA events, barrier and
synchronize on both sides, max over ranks) and, for the optimizer steps, the
live roofline of the tcgen05 GEMM launches inside the timed region.
"""

from __future__ import annotations

import json
import os
import time
from datetime import timedelta

import torch
import torch.distributed as dist

from bench import ClockSampler, load_peaks, quiet_nccl_banner

LLAMA8B = (  # (rows, cols) per layer
    (4096, 4096),   # q
    (4096, 4096),   # o
    (1024, 4096),   # k
    (1024, 4096),   # v
    (14336, 4096),  # gate
    (14336, 4096),  # up
    (4096, 14336),  # down
)
LAYERS = 32


def _gns_flops(rows: int, cols: int) -> float:
    m, n = min(rows, cols), max(rows, cols)
    if m == n:
        return 20.0 * n**3  # standard NS, symmetric products counted as computed
    return 6.0 * m * m * n + 14.0 * m**3


def _setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        quiet_nccl_banner()
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    return world, rank, local, device


def _timed(fn, steps: int, warmup: int, device, world: int, local: int, profile_capacity: int = 0):
    from gram_newton_schulz_ampere_b200 import _native

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    if profile_capacity:
        _native.profile_enable(profile_capacity)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        time.sleep(1.0)
        start.record()
        for _ in range(steps):
            fn()
        stop.record()
        stop.synchronize()
    launches = _native.profile_collect(profile_capacity) if profile_capacity else []
    elapsed = torch.tensor([start.elapsed_time(stop)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    status = _native.device_status(clear=True)
    if status != 0:
        raise SystemExit(f"a kernel's bounded wait gave up (device status {status})")
    return float(elapsed.item()), launches, clocks.summary()


def _roofline(launches, elapsed_ms: float) -> dict | None:
    if not launches:
        return None
    peaks, source = load_peaks()
    sustained = elapsed_ms > 1000.0
    peak = peaks["bf16_tflops_sustained" if sustained else "bf16_tflops"]
    gemm_ms = sum(m for m, _, _ in launches)
    achieved = sum(f for _, f, _ in launches) / (gemm_ms * 1e-3) / 1e12
    return {
        "bound": "tensor",
        "kernel": "gns::gemm_tc_kernel",
        "achieved": achieved,
        "peak": peak,
        "unit": "TFLOP/s",
        "frac": achieved / peak,
        "peak_source": f"{source} {'sustained' if sustained else 'burst'} bf16",
        "gemm_launches": len(launches),
        "gemm_ms_total": gemm_ms,
        "traffic": None,
    }


def _emit(rank: int, line: dict) -> None:
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_cfg1(args, world, rank, local, device) -> None:
    from gram_newton_schulz_ampere_b200 import GramNewtonSchulz

    gen = torch.Generator().manual_seed(0)
    x = torch.randn((1, 128, 256), generator=gen).to(device)
    ns = GramNewtonSchulz()
    steps = max(args.steps, 200)
    elapsed, launches, clocks = _timed(lambda: ns(x), steps, max(args.warmup, 10), device, world, local)
    _emit(rank, {
        "metric": "GNS latency (1 x 128 x 256 fp32)",
        "value": 1e3 * elapsed / steps,
        "unit": "us",
        "n_gpus": world,
        "steps": steps,
        "warmup": max(args.warmup, 10),
        "higher_is_better": False,
        "scaling": "weak",
        "dtype": "f16",
        "data": "synthetic",
        "config": {"workload": "cfg1: GramNewtonSchulz on (1, 128, 256) fp32 N(0,1) seed 0; 2 native launches "
                               "(normalisation + the fused small-matrix chain)"},
        "clocks": clocks,
    })


def _muon_parameters(device, seed: int):
    gen = torch.Generator(device=device).manual_seed(seed)
    params, grads = [], []
    for _ in range(LAYERS):
        for rows, cols in LLAMA8B:
            p = torch.nn.Parameter((torch.randn((rows, cols), generator=gen, device=device) * 0.02).to(torch.bfloat16))
            g = (torch.randn((rows, cols), generator=gen, device=device) * 1e-3).to(torch.bfloat16)
            params.append(p)
            grads.append(g)
    return params, grads


def run_muon8b(args, world, rank, local, device) -> None:
    from gram_newton_schulz_ampere_b200 import Muon

    params, grads = _muon_parameters(device, 1234)
    for p, g in zip(params, grads, strict=True):
        p.grad = g
    opt = Muon(
        params, lr=3e-3, momentum=0.95, nesterov=True, adjust_lr="spectral_norm",
        distributed_mesh=dist.group.WORLD if world > 1 else None,
    )
    steps = args.steps if args.steps <= 20 else 5
    warmup = max(args.warmup, 3) if args.warmup <= 10 else 3
    elapsed, launches, clocks = _timed(opt.step, steps, warmup, device, world, local, profile_capacity=steps * 200)
    ms = elapsed / steps
    ns_tflop = LAYERS * sum(_gns_flops(r, c) for r, c in LLAMA8B) / 1e12
    numel = LAYERS * sum(r * c for r, c in LLAMA8B)
    roof = _roofline(launches, elapsed)
    if roof:
        roof["gemm_ms_per_step"] = roof["gemm_ms_total"] / steps
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    _emit(rank, {
        "metric": "Muon step ms (Llama-3-8B shapes)",
        "value": ms,
        "unit": "ms",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": ms,
        "higher_is_better": False,
        "scaling": "strong",
        "dtype": "f16",
        "data": "synthetic",
        "config": {
            "workload": "cfg3: Muon step, 32 layers x {q,o 4096^2; k,v 1024x4096; gate,up 14336x4096; "
            "down 4096x14336} bf16, lr 3e-3, momentum 0.95, Nesterov, spectral_norm",
            "parameters": numel,
            "parallelism": f"replicated x{world}: round-robin orthogonalisation + all-gather per bucket",
            "ns_algorithmic_tflop_per_step": ns_tflop,
            "ns_tflops_per_gpu": ns_tflop / world / (ms * 1e-3),
        },
        "roofline": roof,
        "clocks": clocks,
    })


def run_dion3(args, world, rank, local, device) -> None:
    from gram_newton_schulz_ampere_b200 import Dion3

    gen = torch.Generator(device=device).manual_seed(4321)
    mats, biases = [], []
    for _ in range(16):
        m = torch.nn.Parameter(torch.randn((4096, 4096), generator=gen, device=device) * 0.02)
        scale = torch.exp(torch.randn((4096, 1), generator=gen, device=device))
        m.grad = torch.randn((4096, 4096), generator=gen, device=device) * 1e-3 * scale
        b = torch.nn.Parameter(torch.zeros(4096, device=device))
        b.grad = torch.randn(4096, generator=gen, device=device) * 1e-3
        mats.append(m)
        biases.append(b)
    opt = Dion3(
        [{"params": mats, "algorithm": "dion3"}, {"params": biases, "algorithm": "adamw"}],
        lr=0.01, fraction=0.25, momentum=0.95, muon_beta2=0.95, weight_decay=0.01,
        distributed_mesh=dist.group.WORLD if world > 1 else None,
    )
    steps = args.steps if args.steps <= 50 else 20
    warmup = max(args.warmup, 3) if args.warmup <= 10 else 3
    elapsed, launches, clocks = _timed(opt.step, steps, warmup, device, world, local, profile_capacity=steps * 40)
    ms = elapsed / steps
    roof = _roofline(launches, elapsed)
    n = 16 * 4096 * 4096
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    _emit(rank, {
        "metric": "Dion3 step ms (16 x 4096^2 fp32)",
        "value": ms,
        "unit": "ms",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": ms,
        "higher_is_better": False,
        "scaling": "strong",
        "dtype": "f32 state, f16 products",
        "data": "synthetic",
        "config": {
            "workload": "cfg4: Dion3 step, 16 x 4096^2 fp32 + 16 bias vectors (AdamW), fraction 0.25, "
            "momentum 0.95, muon_beta2 0.95, wd 0.01, lognormal row scales",
            "state_bytes_per_step": 25 * n,
            "state_gbs_if_state_bound": 25 * n / (ms * 1e-3) / 1e9,
            "parallelism": f"replicated x{world}",
        },
        "roofline": roof,
        "clocks": clocks,
    })


def run_colshard(args, world, rank, local, device) -> None:
    from gram_newton_schulz_ampere_b200 import GramNewtonSchulz
    from gram_newton_schulz_ampere_b200 import distributed_orthogonalization as D

    rows, cols = 8192, 65536
    if cols % world:
        raise SystemExit(f"colshard needs a GPU count dividing {cols}")
    width = cols // world
    gen = torch.Generator(device=device).manual_seed(5)
    # Every rank draws the whole matrix from the same seed and keeps its columns.
    full = torch.randn((rows, cols), generator=gen, device=device).to(torch.bfloat16)
    shard = full[:, rank * width:(rank + 1) * width].contiguous()
    del full
    ns = GramNewtonSchulz()
    group = dist.group.WORLD if world > 1 else None
    if world > 1:
        def step():
            return D.orthogonalize_long_axis_sharded([shard], (rows, cols), ns, group)

        def owner_step():
            return D.orthogonalize_sharded_matrices([shard], (rows, cols), 1, ns, group)
    else:
        def step():
            return ns(shard)

    steps = args.steps if args.steps <= 20 else 10
    warmup = max(args.warmup, 3) if args.warmup <= 10 else 3
    elapsed, launches, clocks = _timed(step, steps, warmup, device, world, local, profile_capacity=steps * 40)
    ms = elapsed / steps
    owner_ms = None
    if world > 1:
        owner_elapsed, _, _ = _timed(owner_step, steps, warmup, device, world, local)
        owner_ms = owner_elapsed / steps
    roof = _roofline(launches, elapsed)
    if roof:
        roof["gemm_ms_per_step"] = roof["gemm_ms_total"] / steps
    m = rows
    total_tflop = (6.0 * m * m * cols + 14.0 * m**3) / 1e12
    per_rank_tflop = (6.0 * m * m * width + 14.0 * m**3) / 1e12
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    _emit(rank, {
        "metric": "column-sharded GNS ms (8192 x 65536 bf16)",
        "value": ms,
        "unit": "ms",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": ms,
        "higher_is_better": False,
        "scaling": "strong",
        "dtype": "f16",
        "data": "synthetic",
        "config": {
            "workload": "cfg5: GramNewtonSchulz of one 8192 x 65536 bf16 N(0,1) matrix, Shard(1) over the ranks",
            "parallelism": f"partial-Gram all-reduce x{world}" if world > 1 else "whole matrix, fused chain",
            "algorithmic_tflop": total_tflop,
            "algorithmic_tflop_per_rank": per_rank_tflop,
            "tflops_per_gpu": per_rank_tflop / (ms * 1e-3),
            "owner_scheme_ms": owner_ms,
            "inputs": "fresh 1 GB shard per rank; L2 (126 MB) holds neither operand nor Gram matrix",
        },
        "roofline": roof,
        "clocks": clocks,
    })


def run_workload(args) -> None:
    world, rank, local, device = _setup()
    runners = {"cfg1": run_cfg1, "muon8b": run_muon8b, "dion3": run_dion3, "colshard": run_colshard}
    runners[args.workload](args, world, rank, local, device)
