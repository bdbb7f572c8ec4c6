"""Multi-rank orchestration on the CPU: two gloo ranks (spawned processes).

Covers the distributed layer with a CPU orthogonaliser (the numpy oracle), as the
reference's torchrun tests do with NCCL (tests/test_distributed.py:40-160):
replicated round-robin + all-gather gives every rank the single-rank result,
Shard(0) / Shard(1) DTensor updates (uneven shapes included) equal the
single-rank result on each shard, batch-sharded buckets stay local, and a
gradient-participation mismatch raises on every rank. Updates sharded along the
long axis of a non-square matrix go through the partial-Gram chain when the
orthogonaliser offers its pieces; with the pieces on the oracle, every rank's
shard equals the oracle's restatement of that chain bit for bit.

Row-sharded Dion3 (``Shard(0)`` parameters, reference dion3.py:213-229 and
tests/test_distributed.py:192-243): the real ``Dion3.step`` runs on two gloo
ranks with its native calls swapped for the oracle's (selection, normalise +
apply) and the oracle as orthogonaliser. Each rank selects
``ceil(fraction * ceil(rows / W))`` rows of its own shard, the selected
matrices are orthogonalised as one Shard(0) matrix on an owner rank, and each
rank applies its rows: checked bit for bit against that sequence restated with
oracle calls, and against the single-rank step with the reference's own bars
(relative difference < 0.2, cosine > 0.99) when every row is selected.
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


class _OracleShardedGram:
    """Gram Newton-Schulz orthogonaliser on the numpy oracle that also offers the
    pieces of the long-axis sharded chain under the B200 backend's names."""

    gram = True

    def __init__(self, reset_iterations=(2,)):
        from oracle import gns_oracle

        self.G = gns_oracle
        self.coefficients = gns_oracle.polar_express_coefficients()
        self.reset_iterations = tuple(reset_iterations)
        self.epsilon = 1e-7
        self.backend = self
        self.whole_matrix_calls = 0

    def __call__(self, matrix):
        self.whole_matrix_calls += 1
        out = self.G.orthogonalize(matrix.detach().float().numpy(), self.coefficients, self.reset_iterations)
        return torch.from_numpy(out).to(matrix.dtype)

    def frobenius_sumsq(self, matrix):
        import numpy as np

        return torch.from_numpy(np.sum(np.square(matrix.double().numpy()), axis=(-2, -1)))

    def frobenius_scale(self, matrix, sumsq, epsilon):
        import numpy as np

        denom = np.sqrt(sumsq.numpy()).astype(np.float32)[:, None, None] + np.float32(epsilon)
        return torch.from_numpy(self.G.to_f16(matrix.float().numpy() / denom))

    def gram_partial(self, normalized, tall):
        x = normalized.numpy()
        xt = x.swapaxes(-1, -2)
        return torch.from_numpy((xt @ x) if tall else (x @ xt))

    def gram_iterations(self, gram, coefficients, it_begin, it_end):
        return torch.from_numpy(self.G.gram_iterations(gram.numpy(), coefficients, it_begin, it_end))

    def apply_polynomial(self, polynomial, normalized, tall, out_dtype):
        q, x = polynomial.numpy(), normalized.numpy()
        out = self.G.baddbmm(None, x, q) if tall else self.G.baddbmm(None, q, x)
        return torch.from_numpy(out).to(out_dtype)


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

        # --- long-axis shards: partial Grams summed over ranks, no whole-matrix assembly
        from oracle import gns_oracle

        for dim, shape, resets in (
            (1, (4, 10), (2,)),
            (0, (10, 4), (2,)),
            (1, (3, 7), (1, 3)),
            (0, (9, 2), ()),
            (1, (2, 3, 8), (2,)),
        ):
            sharded = _OracleShardedGram(resets)
            full_update = torch.randn(shape, generator=gen)
            param = torch.nn.Parameter(distribute_tensor(torch.randn(shape, generator=gen), mesh, [Shard(dim + len(shape) - 2)]))
            local_update = distribute_tensor(full_update, mesh, [Shard(dim + len(shape) - 2)]).to_local()
            got = D.orthogonalize_parameter_updates([param], [local_update], [shape], sharded, mesh, False)[0]
            assert sharded.whole_matrix_calls == 0, "long-axis shard was assembled"
            tall = shape[-2] > shape[-1]
            parts = [c.reshape(-1, *c.shape[-2:]).numpy() for c in torch.chunk(full_update, world, dim=dim + len(shape) - 2)]
            expected = gns_oracle.long_axis_sharded_gram_newton_schulz(parts, tall, sharded.coefficients, resets)[rank]
            assert got.shape == local_update.shape
            assert torch.equal(got.reshape(expected.shape), torch.from_numpy(expected)), f"long-axis {shape} dim {dim}"
            whole = gns_oracle.orthogonalize(full_update.reshape(-1, *shape[-2:]).numpy(), sharded.coefficients, resets)
            mine = torch.chunk(torch.from_numpy(whole), world, dim=-1 if not tall else -2)[rank]
            assert gns_oracle.relative_error(got.reshape(mine.shape).numpy(), mine.numpy()) < 2e-2

        # --- short-axis shard of a Gram orthogonaliser: assembled on owner ranks
        sharded = _OracleShardedGram()
        full_update = torch.randn(6, 5, generator=gen)
        param = torch.nn.Parameter(distribute_tensor(torch.randn(6, 5, generator=gen), mesh, [Shard(1)]))
        local_update = distribute_tensor(full_update, mesh, [Shard(1)]).to_local()
        D.orthogonalize_parameter_updates([param], [local_update], [(6, 5)], sharded, mesh, False)
        assert sharded.whole_matrix_calls == 1

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


def _cpu_dion3_ops():
    """(select_rows, normalize_apply) with the native entry points' signatures and
    in-place semantics, computed by the oracle on CPU tensors."""
    import numpy as np

    from oracle import optim_oracle as O

    def select_rows(momentum, gradient, parameter, selected_count, decay, parameter_decay):
        res = O.dion3_select(
            momentum.numpy(), gradient.float().numpy(), int(selected_count), decay,
            None if parameter is None else parameter.numpy(), parameter_decay,
        )
        momentum.copy_(torch.from_numpy(np.ascontiguousarray(res["momentum"])))
        if parameter is not None:
            parameter.copy_(torch.from_numpy(np.ascontiguousarray(res["parameter"])))
        return torch.from_numpy(res["selected"]).to(torch.bfloat16), torch.from_numpy(res["indices"])

    def normalize_apply(parameter, update, variance, indices, beta2, epsilon, lr, wd, lr_adj):
        res = O.dion3_normalize_apply(
            parameter.numpy(), update.float().numpy(), variance.numpy(), indices.numpy(),
            beta2, epsilon, lr, wd, lr_adj,
        )
        parameter.copy_(torch.from_numpy(np.ascontiguousarray(res["parameter"])))
        variance.copy_(torch.from_numpy(np.ascontiguousarray(res["variance"])))

    def select_rows_multi(momenta, gradients, parameters, selected_count, decay, parameter_decay):
        picks = [select_rows(m, g, None if parameters is None else parameters[i], selected_count, decay,
                             parameter_decay) for i, (m, g) in enumerate(zip(momenta, gradients, strict=True))]
        return torch.stack([p[0] for p in picks]), torch.stack([p[1] for p in picks])

    def normalize_apply_multi(parameters, updates, variances, indices, beta2, epsilon, lr, wd, lr_adj):
        for i, (p, v) in enumerate(zip(parameters, variances, strict=True)):
            normalize_apply(p, updates[i], v, indices[i], beta2, epsilon, lr, wd, lr_adj)

    return select_rows, normalize_apply, select_rows_multi, normalize_apply_multi


def _dion3_row_shard_worker(rank: int, world: int, port: int, result_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import math

    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import DTensor, Shard, distribute_tensor

    from gram_newton_schulz_ampere_b200 import Dion3, ops
    from gram_newton_schulz_ampere_b200.muon import Muon

    status = "ok"
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        mesh = init_device_mesh("cpu", (world,))
        (ops.dion3_select_rows, ops.dion3_normalize_apply, ops.dion3_select_rows_multi,
         ops.dion3_normalize_apply_multi) = _cpu_dion3_ops()
        Muon.validate_cuda_configuration = lambda self: None  # CPU parameters, gloo group
        orth = _oracle_orthogonalizer([])
        gen = torch.Generator().manual_seed(99)

        def make(params, **kw):
            opt = Dion3(params, weight_decay=0.0, adjust_lr=None, **kw)
            opt.newton_schulz = orth
            return opt

        # --- every row selected (the reference's own check, tests/test_distributed.py:192-243)
        full_parameter = torch.randn(6, 4, generator=gen)
        full_gradient = torch.randn(6, 4, generator=gen)
        single = torch.nn.Parameter(full_parameter.clone())
        single.grad = full_gradient.clone()
        make([single], lr=0.03, fraction=1.0, momentum=0.5, muon_beta2=0.9).step()
        param = torch.nn.Parameter(distribute_tensor(full_parameter, mesh, [Shard(0)]))
        param.grad = distribute_tensor(full_gradient, mesh, [Shard(0)])
        opt = make([param], lr=0.03, fraction=1.0, momentum=0.5, muon_beta2=0.9, distributed_mesh=mesh)
        opt.step()
        want = full_parameter - single.detach()
        got = full_parameter - param.full_tensor()
        rel = float((got - want).norm() / want.norm().clamp(min=1e-8))
        cos = float(torch.nn.functional.cosine_similarity(got.flatten(), want.flatten(), dim=0))
        assert rel < 0.2 and cos > 0.99, (rel, cos)
        momentum = opt.state[param]["momentum_buffer"]
        variance = opt.state[param]["variance_neuron"]
        assert isinstance(momentum, DTensor) and isinstance(variance, DTensor)
        assert variance.to_local().shape == (*momentum.to_local().shape[:-1], 1)

        # torch.distributed.checkpoint round trip of the sharded state
        # (reference tests/test_distributed.py:245-314): exact on every shard.
        import torch.distributed.checkpoint as dcp
        from torch.distributed.checkpoint.state_dict import get_optimizer_state_dict, set_optimizer_state_dict

        model = torch.nn.Module()
        model.register_parameter("matrix", param)
        saved = get_optimizer_state_dict(model, opt)
        checkpoint = str(Path(result_dir, "dcp"))
        dcp.save({"optimizer": saved}, checkpoint_id=checkpoint)
        resumed_param = torch.nn.Parameter(distribute_tensor(param.full_tensor().detach(), mesh, [Shard(0)]))
        resumed_model = torch.nn.Module()
        resumed_model.register_parameter("matrix", resumed_param)
        resumed = make([resumed_param], lr=0.03, fraction=1.0, momentum=0.5, muon_beta2=0.9, distributed_mesh=mesh)
        loaded = get_optimizer_state_dict(resumed_model, resumed)
        dcp.load({"optimizer": loaded}, checkpoint_id=checkpoint)
        set_optimizer_state_dict(resumed_model, resumed, loaded)
        resumed.newton_schulz = orth  # load_state_dict rebuilds the (CUDA) orthogonaliser
        for name in ("momentum_buffer", "variance_neuron"):
            got = resumed.state[resumed_param][name]
            assert isinstance(got, DTensor), name
            assert torch.equal(got.to_local(), opt.state[param][name].to_local()), name
        # the resumed optimizer takes the same next step as the original
        grad = torch.randn(6, 4, generator=torch.Generator().manual_seed(5))
        param.grad = distribute_tensor(grad, mesh, [Shard(0)])
        resumed_param.grad = distribute_tensor(grad.clone(), mesh, [Shard(0)])
        opt.step()
        resumed.step()
        assert torch.equal(param.to_local(), resumed_param.to_local())
        dist.barrier()

        # --- local selection of ceil(fraction * ceil(rows / W)) rows per rank
        import numpy as np

        from oracle import gns_oracle, optim_oracle as O

        rows, cols, fraction, mu, beta2, lr = 16, 8, 0.25, 0.9, 0.95, 0.02
        full_parameter = torch.randn(rows, cols, generator=gen)
        full_gradient = torch.randn(rows, cols, generator=gen) * torch.exp(torch.randn(rows, 1, generator=gen))
        param = torch.nn.Parameter(distribute_tensor(full_parameter, mesh, [Shard(0)]))
        param.grad = distribute_tensor(full_gradient, mesh, [Shard(0)])
        opt = make([param], lr=lr, fraction=fraction, momentum=mu, muon_beta2=beta2, distributed_mesh=mesh)
        opt.step()
        local_k = max(1, math.ceil(fraction * math.ceil(rows / world)))
        shards_p = torch.chunk(full_parameter, world)
        shards_g = torch.chunk(full_gradient, world)
        picks = [O.dion3_select(np.zeros(s.shape, np.float32), g.numpy(), local_k, mu)
                 for s, g in zip(shards_p, shards_g, strict=True)]
        assembled = np.concatenate([p["selected"] for p in picks], axis=0)
        orthogonal = gns_oracle.orthogonalize(assembled[None])[0]
        mine = orthogonal[rank * local_k:(rank + 1) * local_k]
        mine = torch.from_numpy(np.ascontiguousarray(mine)).to(torch.bfloat16).float().numpy()
        expected = O.dion3_normalize_apply(
            shards_p[rank].numpy(), mine, np.zeros((shards_p[rank].shape[0], 1), np.float32),
            picks[rank]["indices"], beta2, 1e-8, lr, 0.0, lr,
        )
        assert torch.equal(param.to_local(), torch.from_numpy(expected["parameter"])), "row-sharded Dion3 parameter"
        assert torch.equal(
            opt.state[param]["momentum_buffer"].to_local(), torch.from_numpy(picks[rank]["momentum"])
        ), "row-sharded Dion3 momentum"
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # report to the parent test
        status = traceback.format_exc()
    Path(result_dir, f"rank{rank}.txt").write_text(status)


def _run_ranks(target, tmp_path, world: int = 2) -> None:
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=target, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a gloo rank did not finish")
    for r in range(world):
        result = (tmp_path / f"rank{r}.txt").read_text()
        assert result == "ok", f"rank {r}: {result}"


def _cpu_muon_ops():
    """(muon_momentum, muon_apply) with the native entry points' signatures and
    in-place semantics, in plain torch on CPU tensors."""

    def momentum(gradients, momenta, mu, nesterov, wanted=None):
        updates = []
        for index, (g, m) in enumerate(zip(gradients, momenta, strict=True)):
            m.mul_(mu).add_(g.to(m.dtype))
            want = nesterov and mu != 0.0 and (wanted is None or wanted[index])
            updates.append(g + mu * m if want else None)
        return updates if nesterov and mu != 0.0 else None

    def apply(parameters, updates, decay, rates):
        for p, o, rate in zip(parameters, updates, rates, strict=True):
            if decay is not None:
                p.mul_(decay)
            p.sub_(o.to(p.dtype) * rate)

    return momentum, apply


def _muon_owner_apply_worker(rank: int, world: int, port: int, result_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    from gram_newton_schulz_ampere_b200 import Muon, ops

    status = "ok"
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        ops.muon_momentum, ops.muon_apply = _cpu_muon_ops()
        Muon.validate_cuda_configuration = lambda self: None  # CPU parameters, gloo group
        gen = torch.Generator().manual_seed(31)
        # Three buckets: 5 x (8, 4), 3 x (6, 10) and one (5, 5) (fewer matrices than
        # ranks x 2, uneven split, one rank owning nothing in the last bucket).
        shapes = [(8, 4)] * 5 + [(6, 10)] * 3 + [(5, 5)]
        start = [torch.randn(s, generator=gen) for s in shapes]
        grads = [[torch.randn(s, generator=gen) for s in shapes] for _ in range(2)]

        def run(mesh, exchange="all_gather", contiguous=False):
            calls: list = []
            params = [torch.nn.Parameter(t.clone()) for t in start]
            opt = Muon(params, lr=0.05, momentum=0.9, nesterov=True, weight_decay=0.1, distributed_mesh=mesh)
            opt.replicated_exchange = exchange
            opt.contiguous_buckets = contiguous
            opt.newton_schulz = _oracle_orthogonalizer(calls)
            for step_grads in grads:
                for p, g in zip(params, step_grads, strict=True):
                    p.grad = g.clone()
                opt.step()
            return params, opt, calls

        single, single_opt, _ = run(None)
        params, opt, calls = run(dist.group.WORLD)
        for a, b in zip(params, single, strict=True):
            assert torch.equal(a.detach(), b.detach()), "owner-apply result differs from single rank"
        for a, b in zip(params, single, strict=True):
            assert torch.equal(opt.state[a]["momentum_buffer"], single_opt.state[b]["momentum_buffer"])
        # every matrix was orthogonalised by exactly one rank in each step
        done = torch.zeros(3, dtype=torch.int64)
        for shape in calls[: len(calls) // 2]:
            done[[(8, 4), (6, 10), (5, 5)].index(shape[1:])] += shape[0]
        dist.all_reduce(done)
        assert done.tolist() == [5, 3, 1], done
        gathered = [torch.empty_like(params[0]) for _ in range(world)]
        dist.all_gather(gathered, params[0].detach())
        assert all(torch.equal(g, gathered[0]) for g in gathered)
        # the point-to-point exchange gives the same bits
        sent, _, _ = run(dist.group.WORLD, "p2p")
        for a, b in zip(sent, single, strict=True):
            assert torch.equal(a.detach(), b.detach()), "p2p exchange differs from single rank"
        # contiguous buckets: parameters moved into one buffer per bucket, gathered in place
        flat, flat_opt, _ = run(dist.group.WORLD, contiguous=True)
        for a, b in zip(flat, single, strict=True):
            assert torch.equal(a.detach(), b.detach()), "contiguous-bucket exchange differs from single rank"
        buffers = flat_opt.__dict__["_flat_buckets"]
        assert len(buffers) == 3
        slots = {slot.data_ptr() for _, buffer in buffers.values() for slot in buffer}
        assert all(p.data_ptr() in slots for p in flat)  # every parameter lives in its bucket buffer
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # report to the parent test
        status = traceback.format_exc()
    Path(result_dir, f"rank{rank}.txt").write_text(status)


def test_muon_owner_apply_two_gloo_ranks(tmp_path):
    _run_ranks(_muon_owner_apply_worker, tmp_path)


def test_dion3_row_sharded_two_gloo_ranks(tmp_path):
    _run_ranks(_dion3_row_shard_worker, tmp_path)


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
