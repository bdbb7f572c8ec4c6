"""Multi-rank orchestration on the CPU: two gloo ranks (spawned processes).

Covers the distributed layer with a CPU orthogonaliser (the numpy oracle), as the
reference's torchrun tests do with NCCL (tests/test_distributed.py:40-160):
replicated round-robin + all-gather gives every rank the single-rank result,
Shard(0) / Shard(1) DTensor updates (uneven shapes included) equal the
single-rank result on each shard, batch-sharded buckets stay local, and a
gradient-participation mismatch raises on every rank.
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

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_orthogonalizer(calls: list):
    import numpy as np

    from oracle import gns_oracle

    def orth(matrix: torch.Tensor) -> torch.Tensor:
        calls.append(tuple(matrix.shape))
        out = gns_oracle.orthogonalize(matrix.detach().float().numpy())
        return torch.from_numpy(np.ascontiguousarray(out)).to(matrix.dtype)

    return orth


def _worker(rank: int, world: int, port: int, result_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Shard, distribute_tensor

    from gram_newton_schulz_ampere_b200 import distributed_orthogonalization as D

    status = "ok"
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        group = dist.group.WORLD
        calls: list = []
        orth = _oracle_orthogonalizer(calls)
        gen = torch.Generator().manual_seed(1234)
        # --- replicated buckets: 5 x (8, 4) and 3 x (6, 10); ranks hold identical data
        params = [torch.nn.Parameter(torch.randn(8, 4, generator=gen)) for _ in range(5)]
        params += [torch.nn.Parameter(torch.randn(6, 10, generator=gen)) for _ in range(3)]
        updates = [torch.randn(p.shape, generator=gen) for p in params]
        shapes = [tuple(p.shape) for p in params]
        out = D.orthogonalize_parameter_updates(params, updates, shapes, orth, group, False)
        single = D.orthogonalize_parameter_updates(params, updates, shapes, _oracle_orthogonalizer([]), None, False)
        for a, b in zip(out, single, strict=True):
            assert torch.equal(a, b), "replicated result differs from single rank"
        # each rank orthogonalised ceil(n/W) matrices per bucket
        assert sorted(calls) == sorted([(3, 8, 4), (2, 6, 10)]), calls
        gathered = [torch.empty_like(out[0]) for _ in range(world)]
        dist.all_gather(gathered, out[0])
        assert all(torch.equal(g, gathered[0]) for g in gathered)

        # --- DTensor shards along either matrix axis, even and uneven
        mesh = init_device_mesh("cpu", (world,))
        for dim, shape in ((0, (5, 4)), (1, (4, 5)), (0, (1, 5)), (1, (6, 5)), (1, (3, 7))):
            full_update = torch.randn(shape, generator=gen)
            full_param = torch.randn(shape, generator=gen)
            param = torch.nn.Parameter(distribute_tensor(full_param, mesh, [Shard(dim)]))
            local_update = distribute_tensor(full_update, mesh, [Shard(dim)]).to_local()
            got = D.orthogonalize_parameter_updates([param], [local_update], [shape], orth, mesh, False)[0]
            expected = distribute_tensor(orth(full_update.unsqueeze(0))[0], mesh, [Shard(dim)]).to_local()
            assert got.shape == local_update.shape
            assert torch.equal(got, expected), f"shard dim {dim} shape {shape}"

        # --- batch-sharded bucket is purely local
        batched = torch.nn.Parameter(distribute_tensor(torch.randn(4, 3, 6, generator=gen), mesh, [Shard(0)]))
        layout = D.parameter_layout(batched, mesh, False)
        assert layout.batch_sharded and layout.sharded_tensor_dimension == 0

        # --- participation mismatch raises on every rank
        a = torch.nn.Parameter(torch.zeros(3, 2))
        b = torch.nn.Parameter(torch.zeros(3, 2))
        a.grad = torch.ones(3, 2)
        if rank == 0:
            b.grad = torch.ones(3, 2)
        try:
            D.validate_gradient_participation([a, b], group, False)
            status = "participation mismatch not detected"
        except RuntimeError as exc:
            assert "gradient participation" in str(exc)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # report to the parent test
        status = traceback.format_exc()
    Path(result_dir, f"rank{rank}.txt").write_text(status)


def test_two_gloo_ranks(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a gloo rank did not finish")
    for r in range(2):
        result = (tmp_path / f"rank{r}.txt").read_text()
        assert result == "ok", f"rank {r}: {result}"
