"""The optimizer-step and latency workloads that bench.py measures beside its
headline (``workloads`` in its JSON line), and ``bench.py --workload X``'s
standalone lines.

* cfg1: latency of one ``GramNewtonSchulz`` call on a (1, 128, 256) fp32 matrix,
  microseconds per call.
* muon_step: one ``Muon.step()`` on a synthetic Llama-3-8B-shaped parameter set:
  32 layers x {q, o: 4096x4096, k, v: 1024x4096, gate, up: 14336x4096,
  down: 4096x14336}, bf16 parameters N(0, 0.02), bf16 gradients N(0, 1e-3)
  (same seed on every rank: DDP-replicated), lr 3e-3, momentum 0.95, Nesterov,
  spectral-norm lr adjustment. Across N ranks each bucket's matrices are
  round-robined: the owner orthogonalises and applies the update, and each
  bucket's updated parameters are all-gathered.
* dion3_step: one ``Dion3.step()`` on 16 x (4096 x 4096) fp32 matrices plus 16
  bias vectors in an AdamW group, gradients N(0, 1e-3) times a per-row
  lognormal(sigma = 1) scale, fraction 0.25, momentum 0.95, muon_beta2 0.95,
  weight decay 0.01; replicated across ranks, and at N > 1 also as row-sharded
  DTensors (``Shard(0)``, ``row_sharded``).
* colshard: Gram Newton-Schulz of one 8192 x 65536 bf16 N(0, 1) matrix whose
  columns are split over the N ranks (DTensor ``Shard(1)``): the partial-Gram
  chain (fp32 all-reduces of the 8192 x 8192 Gram matrix and of the norm). At
  N = 1 the matrix is whole and goes through the fused chain.

Every measurement is device time (CUDA events, barrier and synchronize on both
sides, max over ranks). GEMM rooflines come from a separate pass of the same
steps with a CUDA event pair around each tcgen05 GEMM launch, after the timed
region. Every rank runs the same collectives in the same order.
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


def gns_flops(rows: int, cols: int) -> float:
    """Algorithmic flops of one orthogonalisation (symmetric products counted as computed)."""
    m, n = min(rows, cols), max(rows, cols)
    if m == n:
        return 20.0 * n**3
    return 6.0 * m * m * n + 14.0 * m**3


def setup_ranks():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1 and not dist.is_initialized():
        quiet_nccl_banner()
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    return world, rank, local, device


def sync_ranks(device, world: int) -> None:
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()


def max_over_ranks(value: float, device, world: int) -> float:
    t = torch.tensor([value], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def check_status() -> None:
    from gram_newton_schulz_ampere_b200 import _native

    status = _native.device_status(clear=True)
    if status != 0:
        raise SystemExit(f"a kernel's bounded wait gave up (device status {status})")


def timed(fn, steps: int, warmup: int, device, world: int, local: int):
    """(ms for `steps` calls, max over ranks; clock summary)."""
    for _ in range(warmup):
        fn()
    sync_ranks(device, world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        time.sleep(1.0)  # nvidia-smi needs a moment before its first sample
        start.record()
        for _ in range(steps):
            fn()
        stop.record()
        stop.synchronize()
    elapsed = max_over_ranks(start.elapsed_time(stop), device, world)
    sync_ranks(device, world)
    check_status()
    return elapsed, clocks.summary()


def profiled_gemms(fn, steps: int, capacity: int, device, world: int):
    """Per-launch (ms, flops, symmetric) of every tcgen05 GEMM in `steps` more calls."""
    from gram_newton_schulz_ampere_b200 import _native

    _native.profile_enable(capacity)
    for _ in range(steps):
        fn()
    launches = _native.profile_collect(capacity)
    sync_ranks(device, world)
    return launches


def gemm_roofline(launches, sustained: bool) -> dict | None:
    if not launches:
        return None
    peaks, source = load_peaks()
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
    }


def hbm(bytes_moved: float, ms: float) -> dict:
    peaks, source = load_peaks()
    gbs = bytes_moved / (ms * 1e-3) / 1e9 if ms > 0 else 0.0
    return {"bytes": bytes_moved, "ms": ms, "achieved_gbs": gbs, "peak_gbs": peaks["hbm_gbs"],
            "frac": gbs / peaks["hbm_gbs"], "peak_source": source}


def phase_breakdown(events) -> dict[str, float]:
    """Milliseconds per stage label (summed over repeats), from a Muon step's
    (label, event) marks: each interval is charged to the label that closes it."""
    totals: dict[str, float] = {}
    for (_, begin), (label, end) in zip(events, events[1:]):
        if label == "start":
            continue
        totals[label] = totals.get(label, 0.0) + begin.elapsed_time(end)
    if events:
        totals["total"] = events[0][1].elapsed_time(events[-1][1])
    return totals


# ---------------------------------------------------------------- cfg1
def measure_cfg1(world, rank, local, device, steps: int = 200, warmup: int = 10) -> dict:
    from gram_newton_schulz_ampere_b200 import GramNewtonSchulz

    gen = torch.Generator().manual_seed(0)
    x = torch.randn((1, 128, 256), generator=gen).to(device)
    ns = GramNewtonSchulz()
    elapsed, clocks = timed(lambda: ns(x), steps, warmup, device, world, local)
    # the same call replayed from a CUDA graph (input copied into the graph's buffer)
    from gram_newton_schulz_ampere_b200.graphs import CapturedOrthogonalizer

    captured = CapturedOrthogonalizer(ns, x)
    graph_elapsed, _ = timed(lambda: captured(x), steps, warmup, device, world, local)
    t0 = time.perf_counter()
    for _ in range(steps):
        ns(x)
    host_eager = (time.perf_counter() - t0) * 1e6 / steps
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for _ in range(steps):
        captured(x)
    host_graph = (time.perf_counter() - t0) * 1e6 / steps
    torch.cuda.synchronize(device)
    return {
        "metric": "GNS latency (1 x 128 x 256 fp32)",
        "value": 1e3 * elapsed / steps,
        "unit": "us",
        "graph_replay_us": 1e3 * graph_elapsed / steps,
        "host_us_per_call": {"eager": host_eager, "graph_replay": host_graph},
        "higher_is_better": False,
        "steps": steps,
        "warmup": warmup,
        "workload": "one GramNewtonSchulz call on (1, 128, 256) fp32 N(0,1) seed 0 per rank: normalisation + "
        "the fused small-matrix chain (2 launches)",
        "algorithmic_mflop": gns_flops(128, 256) / 1e6,
        "clocks": clocks,
    }


# ----------------------------------------------------------- Muon step
def _muon_parameters(device, seed: int):
    gen = torch.Generator(device=device).manual_seed(seed)
    params = []
    for _ in range(LAYERS):
        for rows, cols in LLAMA8B:
            p = torch.nn.Parameter((torch.randn((rows, cols), generator=gen, device=device) * 0.02).to(torch.bfloat16))
            p.grad = (torch.randn((rows, cols), generator=gen, device=device) * 1e-3).to(torch.bfloat16)
            params.append(p)
    return params


def measure_muon(world, rank, local, device, steps: int = 5, warmup: int = 3) -> dict:
    from gram_newton_schulz_ampere_b200 import Muon
    from gram_newton_schulz_ampere_b200.distributed_orthogonalization import gather_owned_tensors, round_robin_owners

    params = _muon_parameters(device, 1234)
    group = dist.group.WORLD if world > 1 else None
    opt = Muon(params, lr=3e-3, momentum=0.95, nesterov=True, adjust_lr="spectral_norm", distributed_mesh=group)
    elapsed, clocks = timed(opt.step, steps, warmup, device, world, local)
    ms = elapsed / steps

    # one more step with stage marks (untimed above)
    opt.phase_events = []
    opt.step()
    torch.cuda.synchronize(device)
    stages = phase_breakdown(opt.phase_events)
    opt.phase_events = None
    sync_ranks(device, world)
    stages = {k: max_over_ranks(v, device, world) for k, v in sorted(stages.items())}

    launches = profiled_gemms(opt.step, 1, 400, device, world)
    roof = gemm_roofline(launches, sustained=True)

    # HBM passes: momentum reads g, m and writes m (+ u for owned matrices);
    # the update pass reads p and O and writes p for owned matrices.
    numel = [p.numel() for p in params]
    owned = [True] * len(params)
    if world > 1:
        owned = [False] * len(params)
        buckets: dict[tuple[int, int], list[int]] = {}
        for i, p in enumerate(params):
            buckets.setdefault(tuple(p.shape), []).append(i)
        for idx in buckets.values():
            for i, o in zip(idx, round_robin_owners(len(idx), world), strict=True):
                owned[i] = o == rank
    # owned matrices: g read, m read/write, u write (8 B); the others (their
    # momentum runs after the last bucket at W > 1): g read, m read/write (6 B)
    mom_bytes = sum(n * 8 for n, own in zip(numel, owned, strict=True) if own)
    other_bytes = sum(n * 6 for n, own in zip(numel, owned, strict=True) if not own)
    app_bytes = sum(n * 6 for n, own in zip(numel, owned, strict=True) if own)
    exchange_alone = None
    if world > 1:
        # the parameter exchange alone (all-gather + copy into place), without
        # compute to hide behind
        by_shape: dict[tuple[int, int], list[int]] = {}
        for i, p in enumerate(params):
            by_shape.setdefault(tuple(p.shape), []).append(i)

        def exchange():
            for idx in by_shape.values():
                gather_owned_tensors([params[i].detach() for i in idx],
                                     round_robin_owners(len(idx), world), group).finish()

        ex_ms, _ = timed(exchange, 2, 1, device, world, local)
        exchange_alone = ex_ms / 2
    staged = None
    if world > 1:
        # the same step with Muon.contiguous_buckets = False (parameters left where
        # they are; each bucket gathered through a staging buffer and copied back)
        opt.contiguous_buckets = False
        flat_ms, flat_clocks = timed(opt.step, steps, warmup, device, world, local)
        opt.phase_events = []
        opt.step()
        torch.cuda.synchronize(device)
        flat_stages = {k: max_over_ranks(v, device, world) for k, v in sorted(phase_breakdown(opt.phase_events).items())}
        opt.phase_events = None
        staged = {"value": flat_ms / steps, "unit": "ms", "stages_ms": flat_stages, "clocks": flat_clocks,
                  "option": "Muon.contiguous_buckets = False"}
    ns_tflop = LAYERS * sum(gns_flops(r, c) for r, c in LLAMA8B) / 1e12
    total_numel = sum(numel)
    del opt, params
    torch.cuda.empty_cache()
    sync_ranks(device, world)
    return {
        "metric": "Muon step ms (Llama-3-8B shapes)",
        "value": ms,
        "unit": "ms",
        "higher_is_better": False,
        "scaling": "strong",
        "steps": steps,
        "warmup": warmup,
        "workload": "Muon.step() on 32 layers x {q,o 4096^2; k,v 1024x4096; gate,up 14336x4096; down 4096x14336} "
        "bf16 (6.98 G parameters), bf16 grads N(0,1e-3), lr 3e-3, momentum 0.95, Nesterov, spectral_norm",
        "parallelism": (f"replicated x{world}: round-robin owners orthogonalise and apply; each bucket's "
                        "updated parameters are all-gathered in place (NCCL, contiguous parameter buckets), "
                        "overlapped with the next bucket")
        if world > 1 else "one GPU",
        "parameters": total_numel,
        "ns_algorithmic_tflop_per_step": ns_tflop,
        "ns_tflops_per_gpu": ns_tflop / world / (ms * 1e-3),
        "stages_ms": stages,
        "momentum_hbm": hbm(mom_bytes, stages.get("momentum", 0.0)),
        "deferred_momentum_hbm": hbm(other_bytes, stages.get("deferred_momentum", 0.0)) if other_bytes else None,
        "apply_hbm": hbm(app_bytes, stages.get("applied", 0.0)),
        "exchange_ms_alone": exchange_alone,
        "staged_exchange": staged,
        "roofline": roof,
        "clocks": clocks,
    }


# ------------------------------------------ DDP training step with Muon
class _MatrixModel(torch.nn.Module):
    """The matrices of `layers` Llama-3-8B layers; loss = sum_i (W_i * C_i).sum(),
    so each gradient is a fixed tensor C_i (the backward pass is one write per
    matrix and DDP's bucketed all-reduce)."""

    def __init__(self, layers: int, device, seed: int) -> None:
        super().__init__()
        gen = torch.Generator(device=device).manual_seed(seed)
        self.weights = torch.nn.ParameterList()
        self.coeffs = []
        for _ in range(layers):
            for rows, cols in LLAMA8B:
                w = (torch.randn((rows, cols), generator=gen, device=device) * 0.02).to(torch.bfloat16)
                self.weights.append(torch.nn.Parameter(w))
                self.coeffs.append((torch.randn((rows, cols), generator=gen, device=device) * 1e-3).to(torch.bfloat16))

    def forward(self, scale: torch.Tensor) -> torch.Tensor:
        return scale * sum((w * c).float().sum() for w, c in zip(self.weights, self.coeffs))


def measure_ddp_step(world, rank, local, device, steps: int = 5, warmup: int = 3, layers: int = 8) -> dict | None:
    """Backward + ``Muon.step()`` under DistributedDataParallel, with the momentum
    pass in ``step()`` and with ``Muon.momentum_comm_hook()`` (momentum runs as
    each gradient bucket's all-reduce lands). Needs W > 1 (DDP's all-reduce is
    what the hook overlaps)."""
    if world == 1:
        return None
    from torch.nn.parallel import DistributedDataParallel

    from gram_newton_schulz_ampere_b200 import Muon

    out = {}
    for hooked in (False, True):
        model = _MatrixModel(layers, device, 77)
        ddp = DistributedDataParallel(model, device_ids=[local], gradient_as_bucket_view=True)
        opt = Muon(list(model.parameters()), lr=3e-3, momentum=0.95, nesterov=True, adjust_lr="spectral_norm",
                   distributed_mesh=dist.group.WORLD)
        if hooked:
            ddp.register_comm_hook(None, opt.momentum_comm_hook())

        one = torch.ones((), device=device)

        def train_step():
            opt.zero_grad(set_to_none=False)
            ddp(one).backward()
            opt.step()

        elapsed, clocks = timed(train_step, steps, warmup, device, world, local)
        out["hook" if hooked else "no_hook"] = {"value": elapsed / steps, "unit": "ms", "clocks": clocks}
        del ddp, opt, model
        torch.cuda.empty_cache()
        sync_ranks(device, world)
    params = layers * sum(r * c for r, c in LLAMA8B)
    return {
        "metric": "DDP training step ms (backward + Muon.step)",
        "value": out["hook"]["value"],
        "unit": "ms",
        "higher_is_better": False,
        "scaling": "strong",
        "steps": steps,
        "warmup": warmup,
        "workload": f"DDP over {layers} Llama-3-8B layers' matrices ({params / 1e9:.2f} G bf16 parameters); loss "
        "sum((W * C).sum()) with fixed C, so backward writes each gradient once; Muon lr 3e-3, momentum 0.95",
        "with_momentum_comm_hook": out["hook"],
        "without_hook": out["no_hook"],
    }


# ---------------------------------------------------------- Dion3 step
def measure_dion3(world, rank, local, device, steps: int = 20, warmup: int = 3) -> dict:
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
    elapsed, clocks = timed(opt.step, steps, warmup, device, world, local)
    ms = elapsed / steps
    launches = profiled_gemms(opt.step, 2, 200, device, world)
    n = 16 * 4096 * 4096
    del opt, mats, biases
    torch.cuda.empty_cache()
    sync_ranks(device, world)
    row_sharded = None
    if world > 1:
        # The same 16 matrices as row-sharded DTensors (Shard(0)): each rank holds
        # 4096 / W rows of every matrix, selects locally, and the selected rows are
        # orthogonalised on owner ranks (reference dion3.py:213-229).
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.tensor import Shard, distribute_tensor

        mesh = init_device_mesh("cuda", (world,))
        gen = torch.Generator(device=device).manual_seed(4321)
        shards = []
        for _ in range(16):
            full = torch.randn((4096, 4096), generator=gen, device=device) * 0.02
            scale = torch.exp(torch.randn((4096, 1), generator=gen, device=device))
            grad = torch.randn((4096, 4096), generator=gen, device=device) * 1e-3 * scale
            p = torch.nn.Parameter(distribute_tensor(full, mesh, [Shard(0)]))
            p.grad = distribute_tensor(grad, mesh, [Shard(0)])
            shards.append(p)
            del full, grad
        opt = Dion3(shards, lr=0.01, fraction=0.25, momentum=0.95, muon_beta2=0.95, weight_decay=0.01,
                    distributed_mesh=mesh)
        sharded_ms, sharded_clocks = timed(opt.step, steps, warmup, device, world, local)
        row_sharded = {
            "value": sharded_ms / steps,
            "unit": "ms",
            "parallelism": f"row-sharded Shard(0) x{world}: local selection of ceil(0.25 * 4096 / {world}) rows "
            "per rank, owner all-to-all orthogonalisation",
            "clocks": sharded_clocks,
        }
        del opt, shards
        torch.cuda.empty_cache()
        sync_ranks(device, world)
    return {
        "metric": "Dion3 step ms (16 x 4096^2 fp32)",
        "value": ms,
        "unit": "ms",
        "higher_is_better": False,
        "scaling": "strong",
        "steps": steps,
        "warmup": warmup,
        "workload": "Dion3.step() on 16 x 4096^2 fp32 + 16 bias vectors (AdamW), fraction 0.25, momentum 0.95, "
        "muon_beta2 0.95, wd 0.01, lognormal row scales",
        "parallelism": f"replicated x{world}" if world > 1 else "one GPU",
        "state_bytes_per_step": 25 * n,
        "state_gbs_if_state_bound": 25 * n / (ms * 1e-3) / 1e9,
        "roofline": gemm_roofline(launches, sustained=False),
        "row_sharded": row_sharded,
        "clocks": clocks,
    }


# ---------------------------------------------------- column-sharded GNS
def measure_colshard(world, rank, local, device, steps: int = 10, warmup: int = 3) -> dict:
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
    else:
        def step():
            return ns(shard)
    elapsed, clocks = timed(step, steps, warmup, device, world, local)
    ms = elapsed / steps
    launches = profiled_gemms(step, 2, 100, device, world)
    m = rows
    per_rank_tflop = (6.0 * m * m * width + 14.0 * m**3) / 1e12
    del shard
    torch.cuda.empty_cache()
    sync_ranks(device, world)
    return {
        "metric": "column-sharded GNS ms (8192 x 65536 bf16)",
        "value": ms,
        "unit": "ms",
        "higher_is_better": False,
        "scaling": "strong",
        "steps": steps,
        "warmup": warmup,
        "workload": "GramNewtonSchulz of one 8192 x 65536 bf16 N(0,1) matrix, columns split over the ranks",
        "parallelism": f"partial-Gram all-reduce x{world}" if world > 1 else "whole matrix, fused chain",
        "algorithmic_tflop": (6.0 * m * m * cols + 14.0 * m**3) / 1e12,
        "algorithmic_tflop_per_rank": per_rank_tflop,
        "tflops_per_gpu": per_rank_tflop / (ms * 1e-3),
        "roofline": gemm_roofline(launches, sustained=False),
        "clocks": clocks,
    }


MEASURES = {"cfg1": measure_cfg1, "muon8b": measure_muon, "dion3": measure_dion3, "colshard": measure_colshard,
            "ddp": measure_ddp_step}


def run_workload(args) -> None:
    """``bench.py --workload X``: one JSON line for workload X alone."""
    world, rank, local, device = setup_ranks()
    kwargs = {}
    if args.steps_given:
        kwargs["steps"] = args.steps
    if args.warmup_given:
        kwargs["warmup"] = max(args.warmup, 3)
    line = MEASURES[args.workload](world, rank, local, device, **kwargs)
    if line is None:
        line = {"workload": args.workload, "unavailable": "needs more than one GPU"}
    line["n_gpus"] = world
    line["data"] = "synthetic"
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
