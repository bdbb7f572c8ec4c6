"""Muon's DDP communication hook (momentum pass during backward).

With ``ddp.register_comm_hook(None, opt.momentum_comm_hook())`` each gradient
bucket's momentum runs as soon as its all-reduce lands; the parameters after
several steps must equal, bit for bit, those of the same model and data
stepped without the hook (momentum inside ``step()``). Run as NCCL ranks in
spawned processes: one rank on one GPU, and two ranks when two GPUs exist.
"""

from __future__ import annotations

import copy
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


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, result_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    status = "ok"
    try:
        import torch.distributed as dist
        from torch.nn.parallel import DistributedDataParallel

        from gram_newton_schulz_ampere_b200 import Muon, _native

        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=device)
        torch.manual_seed(5)
        base = torch.nn.Sequential(torch.nn.Linear(64, 160), torch.nn.ReLU(), torch.nn.Linear(160, 48),
                                   torch.nn.ReLU(), torch.nn.Linear(48, 8)).to(device)
        runs = []
        for hooked in (True, False):
            model = copy.deepcopy(base)
            ddp = DistributedDataParallel(model, device_ids=[rank], bucket_cap_mb=0.02)
            matrices = [p for p in model.parameters() if p.ndim == 2]
            vectors = [p for p in model.parameters() if p.ndim == 1]
            opt = Muon([{"params": matrices}, {"params": vectors, "algorithm": "adamw"}],
                       lr=0.02, momentum=0.9, nesterov=True, weight_decay=0.01)
            if hooked:
                ddp.register_comm_hook(None, opt.momentum_comm_hook())
            gen = torch.Generator(device=device).manual_seed(100 + rank)
            for _ in range(4):
                x = torch.randn(32, 64, generator=gen, device=device)
                opt.zero_grad(set_to_none=True)
                ddp(x).square().mean().backward()
                if hooked:
                    assert len(opt.__dict__.get("_hooked_updates", {})) == len(matrices), "hook did not run"
                opt.step()
                if hooked:
                    assert not opt.__dict__.get("_hooked_updates"), "step left hooked updates behind"
            runs.append([p.detach().clone() for p in model.parameters()])
        for a, b in zip(*runs, strict=True):
            assert torch.equal(a, b), "hooked momentum differs from momentum in step()"
        torch.cuda.synchronize(device)
        assert _native.device_status(clear=True) == 0
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        status = traceback.format_exc()
    Path(result_dir, f"rank{rank}.txt").write_text(status)


@pytest.mark.parametrize("world", [1, 2])
def test_momentum_hook_equals_momentum_in_step(tmp_path, world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPU(s)")
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("an NCCL rank did not finish")
    for r in range(world):
        result = (tmp_path / f"rank{r}.txt").read_text()
        assert result == "ok", f"rank {r}: {result}"
