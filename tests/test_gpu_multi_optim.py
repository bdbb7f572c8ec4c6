"""Muon and Dion3 on two NCCL ranks (skipped with fewer than two GPUs).

Optimizer-level distributed behaviour, following the reference's
tests/test_distributed.py:

* DDP-replicated and plain replicated parameters end identical on every rank;
* DTensor shards along either matrix axis match the single-rank optimizer:
  bit for bit when the shard is the short axis (owner scheme), within the
  whole-chain bar (2e-2 relative Frobenius error) when it is the long axis
  (partial-Gram chain, whose Gram is summed across ranks in a different order);
* momentum and variance state are DTensors with the local shard's shape, and a
  torch.distributed.checkpoint round trip restores them exactly;
* uneven, empty and batched shards step; a column-sharded Dion3 parameter and
  mismatched gradient participation raise the reference's errors.
"""

from __future__ import annotations

import os
import socket
import sys
import traceback
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float() - b.float()).norm() / b.float().norm().clamp(min=1e-8))


def _same_on_all_ranks(dist, tensor: torch.Tensor) -> None:
    gathered = [torch.empty_like(tensor) for _ in range(dist.get_world_size())]
    dist.all_gather(gathered, tensor.detach().contiguous())
    for other in gathered[1:]:
        assert torch.equal(other, gathered[0]), "replicated parameter differs across ranks"


def _muon_checks(dist, mesh, device, rank: int) -> None:
    from torch.distributed.tensor import DTensor, Shard, distribute_tensor
    from torch.nn.parallel import DistributedDataParallel

    from gram_newton_schulz_ampere_b200 import Muon

    gen = torch.Generator(device=device).manual_seed(67)
    model = DistributedDataParallel(torch.nn.Linear(4, 4, bias=False).to(device), device_ids=[rank])
    opt = Muon(model.parameters(), lr=0.02, momentum=0.0, nesterov=False, adjust_lr=None,
               distributed_mesh=dist.group.WORLD)
    inputs = torch.randn(3, 4, generator=gen, device=device) + rank
    model(inputs).square().mean().backward()
    opt.step()
    _same_on_all_ranks(dist, model.module.weight)

    replicated = [torch.nn.Parameter(torch.randn(8, 4, generator=gen, device=device)) for _ in range(3)]
    for p in replicated:
        p.grad = torch.randn(8, 4, generator=gen, device=device)
    Muon(replicated, lr=0.05, momentum=0.0, nesterov=False, adjust_lr=None,
         distributed_mesh=dist.group.WORLD).step()
    for p in replicated:
        _same_on_all_ranks(dist, p)

    # Replicated buckets with Nesterov momentum in bf16: owners orthogonalise,
    # apply and send; every rank ends with the single-rank result bit for bit.
    shapes = [(96, 64)] * 5 + [(64, 200)] * 3 + [(48, 48)]
    start = [(torch.randn(s, generator=gen, device=device) * 0.02).bfloat16() for s in shapes]
    grads = [[(torch.randn(s, generator=gen, device=device) * 1e-3).bfloat16() for s in shapes] for _ in range(2)]

    def run(mesh_or_none, contiguous=True):
        params = [torch.nn.Parameter(t.clone()) for t in start]
        opt = Muon(params, lr=3e-3, momentum=0.95, nesterov=True, weight_decay=0.1, distributed_mesh=mesh_or_none)
        opt.contiguous_buckets = contiguous
        for step_grads in grads:
            for p, g in zip(params, step_grads, strict=True):
                p.grad = g.clone()
            opt.step()
        return params, opt

    single, single_opt = run(None)
    owned, owned_opt = run(dist.group.WORLD)
    for a, b in zip(owned, single, strict=True):
        assert torch.equal(a.detach(), b.detach()), "owner-apply Muon differs from single rank"
        assert torch.equal(owned_opt.state[a]["momentum_buffer"], single_opt.state[b]["momentum_buffer"])
        _same_on_all_ranks(dist, a)
    staged, _ = run(dist.group.WORLD, contiguous=False)  # gathered through a staging buffer
    for a, b in zip(staged, single, strict=True):
        assert torch.equal(a.detach(), b.detach()), "staged-exchange Muon differs from single rank"

    # (shard dim, shape, long axis?): rows of a tall or columns of a wide matrix
    # are its long axis; (0, (1, 5)) leaves rank 1 an empty shard.
    for dim, shape, long_axis in ((0, (5, 4), True), (1, (4, 5), True), (0, (1, 5), False),
                                  (0, (5, 6), False), (1, (6, 5), False), (0, (96, 40), True),
                                  (1, (96, 40), False)):
        full = torch.randn(shape, generator=gen, device=device)
        grad = torch.randn(shape, generator=gen, device=device)
        reference = torch.nn.Parameter(full.clone())
        reference.grad = grad.clone()
        Muon([reference], lr=0.03, momentum=0.0, nesterov=False, adjust_lr=None).step()
        p = torch.nn.Parameter(distribute_tensor(full, mesh, [Shard(dim)]))
        p.grad = distribute_tensor(grad, mesh, [Shard(dim)])
        o = Muon([p], lr=0.03, momentum=0.0, nesterov=False, adjust_lr=None, distributed_mesh=mesh)
        o.step()
        got = p.full_tensor()
        if long_axis:
            err = _rel(full - got, full - reference.detach())
            assert err < 2e-2, f"Muon long-axis shard {dim} {shape}: {err:.3e}"
        else:
            assert torch.equal(got, reference.detach()), f"Muon short-axis shard {dim} {shape} differs"
        momentum = o.state[p]["momentum_buffer"]
        assert isinstance(momentum, DTensor) and momentum.to_local().shape == p.to_local().shape

    regular = torch.nn.Parameter(torch.zeros(3, 2, device=device))
    sharded = torch.nn.Parameter(distribute_tensor(torch.zeros(4, 2, device=device), mesh, [Shard(0)]))
    regular.grad = torch.ones_like(regular)
    sharded_grad = distribute_tensor(torch.ones(4, 2, device=device), mesh, [Shard(0)])
    if rank == 0:
        sharded.grad = sharded_grad
    with pytest.raises(RuntimeError, match="gradient participation"):
        Muon([regular, sharded]).step()


def _dion3_checks(dist, mesh, device, rank: int, checkpoint_dir: str) -> None:
    import torch.distributed.checkpoint as dcp
    from torch.distributed.checkpoint.state_dict import get_optimizer_state_dict, set_optimizer_state_dict
    from torch.distributed.tensor import DTensor, Shard, distribute_tensor

    from gram_newton_schulz_ampere_b200 import Dion3

    gen = torch.Generator(device=device).manual_seed(113)
    replicated = [torch.nn.Parameter(torch.randn(8, 4, generator=gen, device=device)) for _ in range(3)]
    for p in replicated:
        p.grad = torch.randn(8, 4, generator=gen, device=device)
    Dion3(replicated, lr=0.05, fraction=0.5, momentum=0.5, muon_beta2=0.9, weight_decay=0.0,
          adjust_lr=None, distributed_mesh=dist.group.WORLD).step()
    for p in replicated:
        _same_on_all_ranks(dist, p)

    settings = dict(lr=0.03, fraction=1.0, momentum=0.5, muon_beta2=0.9, weight_decay=0.0, adjust_lr=None)
    full = torch.randn(6, 4, generator=gen, device=device)
    grad = torch.randn(6, 4, generator=gen, device=device)
    reference = torch.nn.Parameter(full.clone())
    reference.grad = grad.clone()
    Dion3([reference], **settings).step()
    p = torch.nn.Parameter(distribute_tensor(full, mesh, [Shard(0)]))
    p.grad = distribute_tensor(grad, mesh, [Shard(0)])
    opt = Dion3([p], distributed_mesh=mesh, **settings)
    opt.step()
    got = p.full_tensor()
    want_update = full - reference.detach()
    got_update = full - got
    assert _rel(got_update, want_update) < 0.2
    assert torch.nn.functional.cosine_similarity(got_update.flatten(), want_update.flatten(), dim=0) > 0.99
    momentum = opt.state[p]["momentum_buffer"]
    variance = opt.state[p]["variance_neuron"]
    assert isinstance(momentum, DTensor) and isinstance(variance, DTensor)
    assert variance.to_local().shape == (*momentum.to_local().shape[:-1], 1)

    model = torch.nn.Module()
    model.register_parameter("matrix", p)
    saved = get_optimizer_state_dict(model, opt)
    resumed_p = torch.nn.Parameter(distribute_tensor(got.detach(), mesh, [Shard(0)]))
    resumed_model = torch.nn.Module()
    resumed_model.register_parameter("matrix", resumed_p)
    resumed = Dion3([resumed_p], distributed_mesh=mesh, **settings)
    dist.barrier()
    dcp.save({"optimizer": saved}, checkpoint_id=checkpoint_dir)
    loaded = get_optimizer_state_dict(resumed_model, resumed)
    dcp.load({"optimizer": loaded}, checkpoint_id=checkpoint_dir)
    set_optimizer_state_dict(resumed_model, resumed, loaded)
    for key, original in (("momentum_buffer", momentum), ("variance_neuron", variance)):
        restored = resumed.state[resumed_p][key]
        assert isinstance(restored, DTensor)
        assert torch.equal(restored.to_local(), original.to_local()), f"{key} not restored"
    dist.barrier()

    mixed = [torch.nn.Parameter(distribute_tensor(torch.randn(s, generator=gen, device=device), mesh, [Shard(0)]))
             for s in ((6, 4), (5, 4))]
    local_shapes = tuple(m.to_local().shape for m in mixed)
    for m in mixed:
        m.grad = torch.ones_like(m)
    Dion3(mixed, fraction=1.0, adjust_lr=None, distributed_mesh=mesh).step()
    assert tuple(m.to_local().shape for m in mixed) == local_shapes

    batched = [torch.nn.Parameter(torch.randn(s, generator=gen, device=device)) for s in ((2, 4, 3), (2, 4, 5))]
    for b in batched:
        b.grad = torch.ones_like(b)
    Dion3(batched, fraction=0.5, adjust_lr=None, distributed_mesh=dist.group.WORLD).step()
    assert all(torch.isfinite(b).all() for b in batched)

    batched_shard = torch.nn.Parameter(distribute_tensor(torch.randn(2, 5, 4, generator=gen, device=device),
                                                         mesh, [Shard(1)]))
    batched_shard.grad = torch.ones_like(batched_shard)
    Dion3([batched_shard], fraction=0.5, adjust_lr=None, distributed_mesh=mesh).step()
    assert torch.isfinite(batched_shard.to_local()).all()

    column = torch.nn.Parameter(distribute_tensor(full, mesh, [Shard(1)]))
    column.grad = distribute_tensor(grad, mesh, [Shard(1)])
    with pytest.raises(NotImplementedError, match="row-sharded"):
        Dion3([column], fraction=0.5, distributed_mesh=mesh).step()


def _worker(rank: int, port: int, result_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    status = "ok"
    try:
        import torch.distributed as dist
        from torch.distributed.device_mesh import init_device_mesh

        from gram_newton_schulz_ampere_b200 import _native

        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
        dist.init_process_group(
            "nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=120), device_id=device
        )
        mesh = init_device_mesh("cuda", (WORLD,), mesh_dim_names=("shard",))
        _muon_checks(dist, mesh, device, rank)
        _dion3_checks(dist, mesh, device, rank, str(Path(result_dir, "dcp")))
        torch.cuda.synchronize(device)
        code = _native.device_status(clear=True)
        assert code == 0, f"device status {code}"
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        status = traceback.format_exc()
    Path(result_dir, f"rank{rank}.txt").write_text(status)


@pytest.mark.skipif(
    not torch.cuda.is_available() or torch.cuda.device_count() < WORLD, reason="needs two GPUs"
)
def test_two_rank_optimizers_match_single_rank(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, port, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("an NCCL rank did not finish")
    for r in range(WORLD):
        result = (tmp_path / f"rank{r}.txt").read_text()
        assert result == "ok", f"rank {r}: {result}"
