"""Two NCCL ranks on two GPUs (skipped with fewer): the distributed layer over
the native kernels.

* long-axis shards (a wide matrix split by columns, a tall one by rows) go
  through the partial-Gram chain; the assembled result matches the single-GPU
  fused chain and the oracle's restatement of the sharded chain (2e-2 relative
  Frobenius error, the whole-chain parity bar);
* short-axis shards use the owner all-to-all scheme and equal the single-GPU
  result bit for bit;
* replicated buckets (round-robin + all-gather) equal the single-rank result on
  every rank bit for bit.
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


def _worker(rank: int, port: int, result_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    status = "ok"
    try:
        import numpy as np
        import torch.distributed as dist

        from gram_newton_schulz_ampere_b200 import GramNewtonSchulz, _native
        from gram_newton_schulz_ampere_b200 import distributed_orthogonalization as D
        from oracle import gns_oracle as O

        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
        dist.init_process_group(
            "nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=120), device_id=device
        )
        group = dist.group.WORLD
        ns = GramNewtonSchulz()
        gen = torch.Generator().manual_seed(99)

        # --- long-axis shards: partial-Gram chain
        for shape, resets in (((2, 256, 1024), (2,)), ((1, 768, 192), (2,)), ((1, 128, 392), (1, 3))):
            ns_r = GramNewtonSchulz(gram_newton_schulz_reset_iterations=resets)
            full = torch.randn(shape, generator=gen).to(torch.bfloat16)
            tall = shape[-2] > shape[-1]
            axis = -2 if tall else -1
            chunks = torch.chunk(full, WORLD, dim=axis)
            local = chunks[rank].to(device)
            got = D.orthogonalize_long_axis_sharded(list(local.unbind(0)), shape[-2:], ns_r, group)
            got = torch.stack(got).float().cpu().numpy()
            whole = ns_r(full.to(device)).float().cpu().numpy()
            mine = np.array_split(whole, WORLD, axis=axis)[rank]
            err = O.relative_error(got, mine)
            assert err < 2e-2, f"long-axis {shape} vs fused chain: {err:.3e}"
            expected = O.long_axis_sharded_gram_newton_schulz(
                [c.float().numpy() for c in chunks], tall, O.polar_express_coefficients(), resets
            )[rank]
            err = O.relative_error(got, expected)
            assert err < 2e-2, f"long-axis {shape} vs oracle: {err:.3e}"

        # --- short-axis shard: owner all-to-all, bit-identical to one GPU
        full = torch.randn(1, 384, 160, generator=gen).to(torch.bfloat16).to(device)
        local = torch.chunk(full, WORLD, dim=-1)[rank].contiguous()
        got = D.orthogonalize_sharded_matrices([local[0]], (384, 160), 1, ns, group)[0]
        want = torch.chunk(ns(full)[0], WORLD, dim=-1)[rank]
        assert torch.equal(got, want), "owner scheme differs from one GPU"

        # --- replicated buckets: every rank ends with the single-rank result
        params = [torch.nn.Parameter(torch.randn(256, 128, generator=gen).to(device)) for _ in range(5)]
        updates = [torch.randn(256, 128, generator=gen).to(torch.bfloat16).to(device) for _ in params]
        shapes = [tuple(p.shape) for p in params]
        out = D.orthogonalize_parameter_updates(params, updates, shapes, ns, group, False)
        single = D.orthogonalize_parameter_updates(params, updates, shapes, ns, None, False)
        for a, b in zip(out, single, strict=True):
            assert torch.equal(a, b), "replicated result differs from single rank"

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
def test_two_nccl_ranks(tmp_path):
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
