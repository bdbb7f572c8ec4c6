"""Muon / Dion3 on the GPU: the reference's known-answer tests, the fused
optimizer-state kernels against the CPU oracle, and checkpoint round trips.

Mirrors tests/test_muon.py and tests/test_dion3.py of the reference.
"""

from __future__ import annotations

import copy
from pathlib import Path

import numpy as np
import pytest
import torch

from gram_newton_schulz_ampere_b200 import Dion3, GramNewtonSchulz, Muon, StandardNewtonSchulz, ops
from gram_newton_schulz_ampere_b200.kernels.dion3_cuda import (
    apply_rows_cuda,
    normalize_apply_rows_cuda,
    normalize_rows_cuda,
    normalize_apply_rows_cuda_batch,
    select_dion3_rows_cuda,
    select_dion3_rows_cuda_batch,
)
from oracle import optim_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
NP_DT = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}


class IdentityOrthogonalizer:
    def __init__(self) -> None:
        self.input_shapes: list[tuple[int, ...]] = []

    def __call__(self, matrix: torch.Tensor) -> torch.Tensor:
        self.input_shapes.append(tuple(matrix.shape))
        return matrix


# ------------------------------------------------------------------- Muon
def test_muon_momentum_nesterov_known_answer(cuda_device):
    golden = np.load(GOLDEN / "muon_reference.npz")
    g1 = torch.tensor(golden["kat__g1"], device=cuda_device)
    g2 = torch.tensor(golden["kat__g2"], device=cuda_device)
    for nesterov, tag in ((False, "plain"), (True, "nesterov")):
        p = torch.nn.Parameter(torch.zeros(2, 2, device=cuda_device))
        opt = Muon([p], lr=0.1, momentum=0.5, nesterov=nesterov, adjust_lr=None)
        opt.newton_schulz = IdentityOrthogonalizer()
        for g in (g1, g2):
            p.grad = g.clone()
            opt.step()
        torch.testing.assert_close(p.detach().cpu().numpy(), golden[f"kat_{tag}__parameter"])
        torch.testing.assert_close(opt.state[p]["momentum_buffer"].cpu().numpy(), golden[f"kat_{tag}__momentum"])
    # Reference expectation written out (tests/test_muon.py:48-53).
    expected_momentum = 0.5 * g1 + g2
    p = torch.nn.Parameter(torch.zeros(2, 2, device=cuda_device))
    opt = Muon([p], lr=0.1, momentum=0.5, nesterov=False, adjust_lr=None)
    opt.newton_schulz = IdentityOrthogonalizer()
    for g in (g1, g2):
        p.grad = g.clone()
        opt.step()
    torch.testing.assert_close(p.detach(), -0.1 * g1 - 0.1 * expected_momentum)


def test_momentum_without_some_update_outputs(cuda_device):
    """A tensor whose update output is not wanted advances its momentum exactly
    as with the output, and no update tensor is made for it."""
    gen = torch.Generator(device=cuda_device).manual_seed(17)
    shapes = [(64, 96), (64, 96), (33, 7), (64, 96)]
    grads = [torch.randn(s, generator=gen, device=cuda_device).bfloat16() for s in shapes]
    moms = [torch.randn(s, generator=gen, device=cuda_device).bfloat16() for s in shapes]
    full_m = [m.clone() for m in moms]
    full = ops.muon_momentum(grads, full_m, 0.95, True)
    part_m = [m.clone() for m in moms]
    wanted = [True, False, False, True]
    part = ops.muon_momentum(grads, part_m, 0.95, True, wanted=wanted)
    for i, want in enumerate(wanted):
        assert torch.equal(part_m[i], full_m[i])
        if want:
            assert torch.equal(part[i], full[i])
        else:
            assert part[i] is None
    # the wanted updates of one shape are consecutive slices of one buffer
    assert part[3].data_ptr() == part[0].data_ptr() + part[0].numel() * part[0].element_size()


def test_closure_runs_once_with_grad_and_returns_loss(cuda_device):
    # tests/test_muon.py:72-89 of the reference.
    p = torch.nn.Parameter(torch.zeros(2, 2, device=cuda_device))
    p.grad = torch.ones_like(p)
    opt = Muon([p], momentum=0.0, nesterov=False)
    opt.newton_schulz = IdentityOrthogonalizer()
    modes: list[bool] = []

    def closure() -> float:
        modes.append(torch.is_grad_enabled())
        return float(p.square().sum().detach())

    with torch.no_grad():
        loss = opt.step(closure)
    assert loss is not None and modes == [True]


def test_rejected_param_groups_leave_optimizer_unchanged(cuda_device):
    # tests/test_muon.py:304-313 and tests/test_dion3.py:227-242 of the reference.
    for make, bad_group, match in (
        (Muon, {"params": [torch.nn.Parameter(torch.zeros(3, device=cuda_device))], "algorithm": "muon"}, "matrix"),
        (Dion3, {"params": [torch.nn.Parameter(torch.zeros(2, 2, device=cuda_device))], "algorithm": "dion3",
                 "fraction": 0.0}, "fraction"),
    ):
        opt = make([torch.nn.Parameter(torch.zeros(3, 2, device=cuda_device))])
        groups, known = len(opt.param_groups), set(opt.state)
        with torch.no_grad(), pytest.raises(ValueError, match=match):
            opt.add_param_group(bad_group)
        assert len(opt.param_groups) == groups and set(opt.state) == known


def test_flatten_orthogonalizes_conv_weights_as_matrices(cuda_device):
    # muon.py:478-498 of the reference: with flatten=True a [out, in, kh, kw]
    # weight is orthogonalised as an [out, in*kh*kw] matrix and its learning
    # rate is adjusted for that matrix shape; without it the trailing two axes
    # form a batch of kh x kw matrices.
    gen = torch.Generator(device=cuda_device).manual_seed(5)
    init = torch.randn(6, 2, 3, 3, generator=gen, device=cuda_device)
    grad = torch.randn(6, 2, 3, 3, generator=gen, device=cuda_device)
    for flatten, matrix in ((True, (6, 18)), (False, (3, 3))):
        p = torch.nn.Parameter(init.clone())
        p.grad = grad.clone()
        opt = Muon([{"params": [p], "flatten": flatten}], lr=0.1, momentum=0.0, nesterov=False, weight_decay=0.0)
        rec = IdentityOrthogonalizer()
        opt.newton_schulz = rec
        opt.step()
        assert rec.input_shapes and all(s[-2:] == matrix for s in rec.input_shapes)
        rate = Muon.adjusted_learning_rate(None, 0.1, (6, 18) if flatten else (6, 2, 3, 3), "spectral_norm")
        torch.testing.assert_close(p.detach(), init - rate * grad)
    p = torch.nn.Parameter(init.clone())
    p.grad = grad.clone()
    Muon([{"params": [p], "flatten": True}], lr=0.1, momentum=0.0, nesterov=False, weight_decay=0.0,
         adjust_lr=None).step()
    want = init - 0.1 * GramNewtonSchulz()(grad.reshape(6, 18)).float().reshape(6, 2, 3, 3)
    torch.testing.assert_close(p.detach(), want, rtol=0, atol=1e-6)


def test_nesterov_updates_of_one_shape_form_one_batch(cuda_device):
    # The momentum kernel's Nesterov updates of equal shape are consecutive
    # slices of one buffer, so the orthogonaliser's bucket needs no stacking copy.
    from gram_newton_schulz_ampere_b200.distributed_orthogonalization import stack_matrices

    shapes = [(8, 4), (6, 4), (8, 4), (8, 4)]
    grads = [torch.randn(s, device=cuda_device) for s in shapes]
    moms = [torch.randn(s, device=cuda_device) for s in shapes]
    updates = ops.muon_momentum(grads, moms, 0.9, True)
    same = [updates[i] for i in (0, 2, 3)]
    batch = stack_matrices(same)
    assert batch.untyped_storage().data_ptr() == same[0].untyped_storage().data_ptr()
    assert torch.equal(batch, torch.stack(same))
    for g, m, u in zip(grads, moms, updates, strict=True):
        torch.testing.assert_close(u, g + 0.9 * m, rtol=1e-6, atol=1e-6)  # m: the updated buffer


def test_decay_uses_base_lr_and_update_uses_adjusted_lr(cuda_device):
    p = torch.nn.Parameter(torch.ones(8, 2, device=cuda_device))
    p.grad = torch.ones_like(p)
    opt = Muon([p], lr=0.1, momentum=0.0, nesterov=False, weight_decay=0.2, adjust_lr="spectral_norm")
    opt.newton_schulz = IdentityOrthogonalizer()
    opt.step()
    expected = torch.ones_like(p) * (1 - 0.1 * 0.2) - torch.ones_like(p) * 0.1 * 2.0
    torch.testing.assert_close(p.detach(), expected)


def test_actual_gram_update_matches_direct_call(cuda_device):
    gen = torch.Generator(device=cuda_device).manual_seed(67)
    gradient = torch.randn(8, 4, generator=gen, device=cuda_device)
    p = torch.nn.Parameter(torch.zeros_like(gradient))
    p.grad = gradient.clone()
    opt = Muon([p], lr=0.05, momentum=0.0, nesterov=False, adjust_lr=None)
    assert isinstance(opt.newton_schulz, GramNewtonSchulz)
    opt.step()
    torch.testing.assert_close(p.detach(), -0.05 * GramNewtonSchulz()(gradient))


# Every instantiation of the momentum and update kernels: the fixed-dtype ones
# (the first five momentum pairs; same-dtype updates) and the runtime-dtype
# fallback (fp32 gradients with bf16 momentum; fp16 parameters with fp32 updates).
@pytest.mark.parametrize("g_dtype,m_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                             (torch.bfloat16, torch.float32), (torch.float16, torch.float16),
                                             (torch.float16, torch.float32), (torch.float32, torch.bfloat16)])
def test_fused_momentum_and_apply_match_oracle(cuda_device, g_dtype, m_dtype):
    gen = torch.Generator().manual_seed(5)
    shapes = [(16, 24), (3, 40, 8), (1, 7), (1000, 33)] + [(5, 8)] * 60  # > 48 tensors: two launches
    grads = [(torch.randn(s, generator=gen) * 1e-3).to(g_dtype) for s in shapes]
    moms = [(torch.randn(s, generator=gen) * 1e-3).to(m_dtype) for s in shapes]
    params = [(torch.randn(s, generator=gen) * 0.02).to(g_dtype) for s in shapes]
    dg = [g.to(cuda_device) for g in grads]
    dm = [m.to(cuda_device) for m in moms]
    dp = [p.to(cuda_device) for p in params]
    updates = ops.muon_momentum(dg, dm, 0.95, True)
    rates = [3e-3 * (1 + i % 3) for i in range(len(shapes))]
    ops.muon_apply(dp, updates, 1 - 3e-3 * 0.1, rates)
    for i in range(len(shapes)):
        m_ref, u_ref = O.muon_momentum(grads[i].float().numpy(), moms[i].float().numpy(), 0.95, True,
                                       NP_DT[g_dtype], NP_DT[m_dtype])
        p_ref = O.muon_apply(params[i].float().numpy(), u_ref, 3e-3, 0.1, rates[i], NP_DT[g_dtype])
        # The kernel fuses a*x+y (one rounding); numpy rounds the product too: <= 1 ulp apart.
        # Relative: one ulp of a normal number. Absolute: one ulp of the operands
        # (~1e-3 here) for cancelling sums, or of fp16's smallest subnormals.
        tol = {"f32": (1e-6, 1e-9), "bf16": (8e-3, 1e-9), "f16": (1e-3, 6e-8)}
        for got, want, dt in ((dm[i], m_ref, m_dtype), (updates[i], u_ref, updates[i].dtype), (dp[i], p_ref, g_dtype)):
            rtol, atol = tol[NP_DT[dt]]
            np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=rtol, atol=atol)


def test_state_dict_resume_scheduler_and_add_param_group(cuda_device):
    gen = torch.Generator(device=cuda_device).manual_seed(71)
    initial = torch.randn(4, 3, generator=gen, device=cuda_device)
    grads = [torch.randn(4, 3, generator=gen, device=cuda_device) for _ in range(3)]
    a = torch.nn.Parameter(initial.clone())
    b = torch.nn.Parameter(initial.clone())
    opt_a = Muon([a], lr=0.1, momentum=0.5, nesterov=True, adjust_lr=None)
    opt_b = Muon([b], lr=0.1, momentum=0.5, nesterov=True, adjust_lr=None)
    for o in (opt_a, opt_b):
        o.newton_schulz = IdentityOrthogonalizer()
    a.grad, b.grad = grads[0].clone(), grads[0].clone()
    opt_a.step()
    opt_b.step()
    resumed = torch.nn.Parameter(b.detach().clone())
    opt_r = Muon([resumed], lr=0.1, momentum=0.5, nesterov=True, adjust_lr=None)
    opt_r.load_state_dict(copy.deepcopy(opt_b.state_dict()))
    opt_r.newton_schulz = IdentityOrthogonalizer()
    sched = torch.optim.lr_scheduler.StepLR(opt_r, step_size=1, gamma=0.5)
    a.grad, resumed.grad = grads[1].clone(), grads[1].clone()
    opt_a.step()
    opt_r.step()
    sched.step()
    opt_a.param_groups[0]["lr"] = 0.05
    a.grad, resumed.grad = grads[2].clone(), grads[2].clone()
    opt_a.step()
    opt_r.step()
    torch.testing.assert_close(resumed, a)
    vector = torch.nn.Parameter(torch.ones(3, device=cuda_device))
    opt_r.add_param_group({"params": [vector], "algorithm": "adamw"})
    assert set(opt_r.state[vector]) == {"step", "exp_avg", "exp_avg_sq"}


def test_adamw_group_matches_torch(cuda_device):
    initial = torch.tensor([1.0, -2.0, 3.0], device=cuda_device)
    ours = torch.nn.Parameter(initial.clone())
    ref = torch.nn.Parameter(initial.clone())
    opt = Muon([{"params": [ours], "algorithm": "adamw"}], lr=0.03, weight_decay=0.1, betas=(0.8, 0.9), epsilon=1e-6)
    ref_opt = torch.optim.AdamW([ref], lr=0.03, weight_decay=0.1, betas=(0.8, 0.9), eps=1e-6)
    for g in (torch.tensor([0.5, -0.25, 1.0]), torch.tensor([-0.5, 0.75, 0.25])):
        ours.grad = g.to(cuda_device)
        ref.grad = g.to(cuda_device)
        opt.step()
        ref_opt.step()
    torch.testing.assert_close(ours, ref, rtol=1e-6, atol=1e-7)


def test_newton_schulz_configuration_resume(cuda_device):
    p = torch.nn.Parameter(torch.randn(4, 3, device=cuda_device))
    opt = Muon([p], ns_algorithm="standard_newton_schulz")
    p.grad = torch.randn_like(p)
    opt.step()
    ckpt = copy.deepcopy(opt.state_dict())
    q = torch.nn.Parameter(p.detach().clone())
    resumed = Muon([q], ns_algorithm="gram_newton_schulz")
    resumed.load_state_dict(ckpt)
    assert resumed.ns_algorithm == "standard_newton_schulz"
    assert isinstance(resumed.newton_schulz, StandardNewtonSchulz)
    missing = copy.deepcopy(ckpt)
    missing["state"] = {}
    resumed.load_state_dict(missing)
    assert "momentum_buffer" in resumed.state[q]


def test_muon_rejects_sparse_and_complex_gradients(cuda_device):
    sparse = torch.nn.Parameter(torch.zeros(3, 3, device=cuda_device))
    sparse.grad = torch.eye(3, device=cuda_device).to_sparse()
    with pytest.raises(RuntimeError, match="sparse"):
        Muon([sparse]).step()
    cplx = torch.nn.Parameter(torch.zeros(3, 3, dtype=torch.complex64, device=cuda_device))
    cplx.grad = torch.ones_like(cplx)
    with pytest.raises(RuntimeError, match="complex"):
        Muon([cplx]).step()


# ------------------------------------------------------------------ Dion3
def test_dion3_known_answer_optimizer(cuda_device):
    matrix = torch.nn.Parameter(torch.zeros(4, 2, device=cuda_device))
    vector = torch.nn.Parameter(torch.tensor([1.0, -2.0], device=cuda_device))
    opt = Dion3(
        [{"params": [matrix], "algorithm": "dion3"}, {"params": [vector], "algorithm": "adamw"}],
        lr=0.1, fraction=0.5, momentum=0.5, muon_beta2=0.9, weight_decay=0.0, adjust_lr=None,
    )
    opt.newton_schulz = IdentityOrthogonalizer()
    calls = 0

    def closure() -> float:
        nonlocal calls
        calls += 1
        matrix.grad = torch.tensor([[1.0, 0.0], [4.0, 4.0], [2.0, 0.0], [0.5, 0.0]], device=cuda_device)
        vector.grad = torch.tensor([0.25, -0.5], device=cuda_device)
        return float((matrix.square().sum() + vector.square().sum()).detach())

    assert opt.step(closure) is not None and calls == 1
    # Reference tests/test_dion3.py:140-141.
    torch.testing.assert_close(matrix[1].detach(), torch.tensor([-0.3, -0.3], device=cuda_device), atol=2e-3, rtol=0)
    torch.testing.assert_close(matrix[2].detach(), torch.tensor([-0.425, 0.0], device=cuda_device), atol=2e-3, rtol=0)
    assert set(opt.state[matrix]) == {"momentum_buffer", "variance_neuron"}
    assert set(opt.state[vector]) == {"step", "exp_avg", "exp_avg_sq"}
    saved = copy.deepcopy(opt.state_dict())
    m2 = torch.nn.Parameter(matrix.detach().clone())
    v2 = torch.nn.Parameter(vector.detach().clone())
    resumed = Dion3(
        [{"params": [m2], "algorithm": "dion3"}, {"params": [v2], "algorithm": "adamw"}],
        lr=0.1, fraction=0.5, momentum=0.5, muon_beta2=0.9, weight_decay=0.0, adjust_lr=None,
    )
    resumed.load_state_dict(saved)
    resumed.newton_schulz = IdentityOrthogonalizer()
    for mat, vec, o in ((matrix, vector, opt), (m2, v2, resumed)):
        mat.grad = torch.ones_like(mat)
        vec.grad = torch.tensor([0.1, -0.1], device=cuda_device)
        o.step()
    assert torch.equal(matrix, m2) and torch.equal(vector, v2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape,fraction", [((2, 512, 256), 0.25), ((1, 300, 72), 0.1), ((3, 64, 40), 1.0),
                                            ((1, 4096, 128), 0.25)])
def test_dion3_selection_matches_oracle(cuda_device, dtype, shape, fraction):
    gen = torch.Generator().manual_seed(sum(shape))
    scale = torch.exp(torch.randn(*shape[:-1], 1, generator=gen))
    grad = (torch.randn(shape, generator=gen) * 1e-3 * scale).to(dtype)
    mom = (torch.randn(shape, generator=gen) * 1e-3).to(dtype)
    par = (torch.randn(shape, generator=gen) * 0.02).to(dtype)
    k = O.selected_count(shape[-2], fraction)
    want = O.dion3_select(mom.float().numpy(), grad.float().numpy(), k, 0.95, par.float().numpy(), 0.999,
                          NP_DT[dtype])
    dm, dp = mom.to(cuda_device), par.to(cuda_device)
    sel, idx = select_dion3_rows_cuda(dm, grad.to(cuda_device), fraction, 0.95, None, dp, 0.999)
    # Row-selection indices: bit-exact (north-star requirement).
    np.testing.assert_array_equal(idx.cpu().numpy(), want["indices"])
    np.testing.assert_array_equal(sel.float().cpu().numpy(), want["selected"])
    np.testing.assert_array_equal(dm.float().cpu().numpy(), want["momentum"])
    np.testing.assert_array_equal(dp.float().cpu().numpy(), want["parameter"])


@pytest.mark.parametrize("p_dtype", [torch.float32, torch.bfloat16])
def test_dion3_normalize_apply_matches_oracle(cuda_device, p_dtype):
    gen = torch.Generator().manual_seed(11)
    b, rows, cols, k = 2, 256, 192, 64
    par = (torch.randn(b, rows, cols, generator=gen) * 0.02).to(p_dtype)
    upd = torch.randn(b, k, cols, generator=gen).bfloat16() * 0.05
    var = torch.rand(b, rows, 1, generator=gen) * 1e-4
    idx = torch.stack([torch.randperm(rows, generator=gen)[:k].sort().values for _ in range(b)])
    want = O.dion3_normalize_apply(par.float().numpy(), upd.float().numpy(), var.numpy(), idx.numpy(),
                                   0.95, 1e-8, 0.01, 0.0, 0.02, NP_DT[p_dtype])
    dp, dv = par.to(cuda_device), var.to(cuda_device)
    normalize_apply_rows_cuda(dp, upd.to(cuda_device), dv, idx.to(cuda_device), 0.95, 1e-8, 0.01, 0.0, 0.02)
    np.testing.assert_allclose(dv.cpu().numpy(), want["variance"], rtol=1e-5, atol=1e-12)
    rtol = 1e-5 if p_dtype == torch.float32 else 8e-3
    np.testing.assert_allclose(dp.float().cpu().numpy(), want["parameter"], rtol=rtol, atol=1e-7)


def test_dion3_normalize_rows_matches_oracle(cuda_device):
    # Reference kernels/dion3_cuda.py:151-170: variance updated in place, fp32 normalised rows,
    # per-matrix (sum u^2, sum n^2).
    gen = torch.Generator().manual_seed(12)
    b, rows, cols, k = 3, 200, 136, 50
    upd = torch.randn(b, k, cols, generator=gen).bfloat16() * 0.05
    var = torch.rand(b, rows, 1, generator=gen) * 1e-4
    idx = torch.stack([torch.randperm(rows, generator=gen)[:k].sort().values for _ in range(b)])
    want = O.dion3_normalize_rows(upd.float().numpy(), var.numpy(), idx.numpy(), 0.95, 1e-8)
    dv = var.to(cuda_device)
    normalized, squared = normalize_rows_cuda(upd.to(cuda_device), dv, idx.to(cuda_device), 0.95, 1e-8)
    assert normalized.dtype == torch.float32 and normalized.shape == upd.shape and squared.shape == (b, 2)
    np.testing.assert_allclose(dv.cpu().numpy(), want["variance"], rtol=1e-5, atol=1e-12)
    np.testing.assert_allclose(normalized.cpu().numpy(), want["normalized"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(squared.cpu().numpy(), want["squared_norms"], rtol=1e-4)


@pytest.mark.parametrize("p_dtype", [torch.float32, torch.bfloat16])
def test_dion3_split_rows_equal_fused_call(cuda_device, p_dtype):
    # normalize_apply_rows = normalize_rows + apply_rows (reference dion3_cuda.cu:472-490), bit for bit.
    gen = torch.Generator(device=cuda_device).manual_seed(13)
    b, rows, cols, k = 2, 256, 192, 64
    par = (torch.randn(b, rows, cols, generator=gen, device=cuda_device) * 0.02).to(p_dtype)
    upd = (torch.randn(b, k, cols, generator=gen, device=cuda_device) * 0.05).bfloat16()
    var = torch.rand(b, rows, 1, generator=gen, device=cuda_device) * 1e-4
    idx = torch.stack([torch.randperm(rows, generator=gen, device=cuda_device)[:k].sort().values for _ in range(b)])
    p_fused, v_fused = par.clone(), var.clone()
    normalize_apply_rows_cuda(p_fused, upd, v_fused, idx, 0.95, 1e-8, 0.01, 0.1, 0.02)
    p_split, v_split = par.clone(), var.clone()
    normalized, squared = normalize_rows_cuda(upd, v_split, idx, 0.95, 1e-8)
    apply_rows_cuda(p_split, normalized, idx, squared, 0.01, 0.1, 0.02, 1e-8)
    assert torch.equal(v_split, v_fused)
    assert torch.equal(p_split, p_fused)


def test_dion3_batched_entry_points_match_individual_calls(cuda_device):
    gen = torch.Generator(device=cuda_device).manual_seed(317)
    shapes = ((64, 32), (96, 48))
    grads = [torch.randn(s, generator=gen, device=cuda_device) for s in shapes]
    mom_a = [torch.randn(s, generator=gen, device=cuda_device) for s in shapes]
    mom_b = [m.clone() for m in mom_a]
    par_a = [torch.randn(s, generator=gen, device=cuda_device) for s in shapes]
    par_b = [p.clone() for p in par_a]
    counts = [16, 24]
    ref_sel, ref_idx = [], []
    for i in range(2):
        s, ix = select_dion3_rows_cuda(mom_a[i], grads[i], 0.25, 0.95, counts[i], par_a[i], 0.999)
        ref_sel.append(s)
        ref_idx.append(ix)
    sel, idx = select_dion3_rows_cuda_batch(mom_b, grads, par_b, counts, 0.95, 0.999)
    for i in range(2):
        assert torch.equal(mom_a[i], mom_b[i]) and torch.equal(par_a[i], par_b[i])
        assert torch.equal(sel[i], ref_sel[i]) and torch.equal(idx[i], ref_idx[i])
    va = [torch.zeros((s[0], 1), device=cuda_device) for s in shapes]
    vb = [v.clone() for v in va]
    pa = [p.clone() for p in par_a]
    pb = [p.clone() for p in par_a]
    for i in range(2):
        normalize_apply_rows_cuda(pa[i], ref_sel[i], va[i], ref_idx[i], 0.95, 1e-8, 0.01, 0.0, [0.01, 0.02][i])
    normalize_apply_rows_cuda_batch(pb, ref_sel, vb, ref_idx, 0.95, 1e-8, 0.01, 0.0, [0.01, 0.02])
    for i in range(2):
        assert torch.equal(pa[i], pb[i]) and torch.equal(va[i], vb[i])


@pytest.mark.parametrize("count,shape,k", [(5, (96, 40), 24), (70, (16, 8), 4)])
def test_dion3_multi_tensor_calls_equal_per_tensor_calls(cuda_device, count, shape, k):
    """One multi-tensor call over separate same-shape matrices (70 crosses the
    64-matrix launch chunk) gives the per-tensor calls' bits: momentum, decayed
    parameters, selected rows, indices, variances and updated parameters."""
    gen = torch.Generator(device=cuda_device).manual_seed(4040 + count)
    scale = [torch.exp(torch.randn((shape[0], 1), generator=gen, device=cuda_device)) for _ in range(count)]
    grads = [torch.randn(shape, generator=gen, device=cuda_device) * s for s in scale]
    mom_a = [torch.randn(shape, generator=gen, device=cuda_device) for _ in range(count)]
    par_a = [torch.randn(shape, generator=gen, device=cuda_device) for _ in range(count)]
    mom_b, par_b = [m.clone() for m in mom_a], [p.clone() for p in par_a]
    ref = [ops.dion3_select_rows(mom_a[i], grads[i], par_a[i], k, 0.9, 0.995) for i in range(count)]
    sel, idx = ops.dion3_select_rows_multi(mom_b, grads, par_b, k, 0.9, 0.995)
    for i in range(count):
        assert torch.equal(mom_a[i], mom_b[i]) and torch.equal(par_a[i], par_b[i])
        assert torch.equal(sel[i], ref[i][0]) and torch.equal(idx[i], ref[i][1])
    upd = (torch.randn((count, k, shape[1]), generator=gen, device=cuda_device) * 0.1).bfloat16()
    var_a = [torch.rand((shape[0], 1), generator=gen, device=cuda_device) for _ in range(count)]
    var_b = [v.clone() for v in var_a]
    for i in range(count):
        ops.dion3_normalize_apply(par_a[i], upd[i], var_a[i], idx[i], 0.95, 1e-8, 0.01, 0.1, 0.02)
    ops.dion3_normalize_apply_multi(par_b, upd, var_b, idx, 0.95, 1e-8, 0.01, 0.1, 0.02)
    for i in range(count):
        assert torch.equal(par_a[i], par_b[i]) and torch.equal(var_a[i], var_b[i])


def test_dion3_full_step_matches_oracle_composition(cuda_device):
    gen = torch.Generator().manual_seed(21)
    shape = (256, 128)
    p0 = torch.randn(shape, generator=gen) * 0.02
    g = torch.randn(shape, generator=gen) * 1e-3 * torch.exp(torch.randn(shape[0], 1, generator=gen))
    p = torch.nn.Parameter(p0.clone().to(cuda_device))
    p.grad = g.to(cuda_device)
    opt = Dion3([p], lr=0.01, fraction=0.25, momentum=0.95, muon_beta2=0.95, weight_decay=0.01)
    opt.step()
    # Oracle composition: select -> Gram NS (oracle) -> normalise + apply.
    from oracle import gns_oracle

    k = O.selected_count(shape[0], 0.25)
    sel = O.dion3_select(np.zeros(shape, np.float32), g.numpy(), k, 0.95, p0.numpy(), 1 - 0.01 * 0.01)
    ortho = O.to_bf16(gns_oracle.orthogonalize(sel["selected"]))
    lr_adj = O.adjusted_learning_rate(0.01, shape, "spectral_norm")
    want = O.dion3_normalize_apply(sel["parameter"], ortho, np.zeros((shape[0], 1), np.float32), sel["indices"],
                                   0.95, 1e-8, 0.01, 0.0, lr_adj)
    got = p.detach().cpu().numpy()
    delta_got = got - p0.numpy()
    delta_want = want["parameter"] - p0.numpy()
    rel = np.linalg.norm(delta_got - delta_want) / np.linalg.norm(delta_want)
    assert rel < 2e-2, rel
    np.testing.assert_allclose(opt.state[p]["variance_neuron"].cpu().numpy(), want["variance"], rtol=3e-2, atol=1e-12)


def test_dion3_validation_messages(cuda_device):
    with pytest.raises(ValueError, match="fraction"):
        Dion3([torch.nn.Parameter(torch.zeros(2, 2, device=cuda_device))], fraction=0.0)
    with pytest.raises(ValueError, match="matrix"):
        Dion3([torch.nn.Parameter(torch.zeros(2, device=cuda_device))])
    with pytest.raises(ValueError, match="Muon parameter groups"):
        Dion3([{"params": [torch.nn.Parameter(torch.zeros(2, 2, device=cuda_device))], "algorithm": "muon"}])
    opt = Dion3([torch.nn.Parameter(torch.zeros(3, 2, device=cuda_device))])
    added = torch.nn.Parameter(torch.zeros(2, 2, device=cuda_device))
    opt.add_param_group({"params": [added]})
    assert opt.param_groups[-1]["algorithm"] == "dion3" and "variance_neuron" in opt.state[added]
    groups = len(opt.param_groups)
    with pytest.raises(ValueError, match="fraction"):
        opt.add_param_group({"params": [torch.nn.Parameter(torch.zeros(2, 2, device=cuda_device))], "fraction": 0.0})
    assert len(opt.param_groups) == groups
    bf = torch.nn.Parameter(torch.zeros(3, 4, dtype=torch.bfloat16, device=cuda_device))
    assert Dion3([bf]).state[bf]["variance_neuron"].dtype == torch.float32
    batched = torch.nn.Parameter(torch.zeros(2, 3, 4, 5, device=cuda_device))
    bo = Dion3([batched], fraction=0.5, adjust_lr=None)
    bo.newton_schulz = IdentityOrthogonalizer()
    batched.grad = torch.randn_like(batched)
    bo.step()
    assert bo.state[batched]["variance_neuron"].shape == (2, 3, 4, 1)
    assert torch.isfinite(batched).all()


def _reference_adamw_step(params, grads, avgs, avg_sqs, steps, lr, wd, betas, eps):
    # The reference's per-parameter torch sequence (muon.py:516-553), on the GPU.
    from math import sqrt

    for p, g, m, v, t in zip(params, grads, avgs, avg_sqs, steps, strict=True):
        t.add_(1)
        step = float(t.item())
        g = g.to(dtype=m.dtype)
        m.mul_(betas[0]).add_(g, alpha=1 - betas[0])
        v.mul_(betas[1]).addcmul_(g, g, value=1 - betas[1])
        if wd != 0.0:
            p.mul_(1 - lr * wd)
        c1 = 1 - betas[0] ** step
        c2 = 1 - betas[1] ** step
        d = v.sqrt().div_(sqrt(c2)).add_(eps)
        p.sub_(m.div(d).mul(lr / c1).to(dtype=p.dtype))


def _reference_lion_step(params, grads, buffers, lr, wd, betas):
    # The reference's per-parameter torch sequence (muon.py:555-583), on the GPU.
    for p, g, b in zip(params, grads, buffers, strict=True):
        g = g.to(dtype=b.dtype)
        d = b.mul(betas[0]).add(g, alpha=1 - betas[0])
        if wd != 0.0:
            p.mul_(1 - lr * wd)
        p.sub_(d.sign().mul(lr).to(dtype=p.dtype))
        b.mul_(betas[1]).add_(g, alpha=1 - betas[1])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("algorithm", ["adamw", "lion"])
def test_fused_adamw_and_lion_groups_match_reference_sequence(cuda_device, dtype, algorithm):
    gen = torch.Generator(device=cuda_device).manual_seed(21)
    shapes = [(4096,), (33,), (7, 5), (129, 64)]
    ours = [torch.nn.Parameter((torch.randn(s, generator=gen, device=cuda_device) * 0.1).to(dtype)) for s in shapes]
    ref = [p.detach().clone() for p in ours]
    kw = {"lr": 0.01, "weight_decay": 0.1, "betas": (0.9, 0.95)}
    if algorithm == "adamw":
        kw["epsilon"] = 1e-8
    opt = Muon([{"params": ours, "algorithm": algorithm}], **kw)
    ref_avgs = [torch.zeros_like(p) for p in ref]
    ref_sqs = [torch.zeros_like(p) for p in ref]
    ref_steps = [torch.zeros((), device=cuda_device) for _ in ref]
    for _ in range(3):
        grads = [(torch.randn(s, generator=gen, device=cuda_device) * 0.01).to(dtype) for s in shapes]
        for p, g in zip(ours, grads, strict=True):
            p.grad = g
        opt.step()
        if algorithm == "adamw":
            _reference_adamw_step(ref, grads, ref_avgs, ref_sqs, ref_steps, 0.01, 0.1, (0.9, 0.95), 1e-8)
        else:
            _reference_lion_step(ref, grads, ref_avgs, 0.01, 0.1, (0.9, 0.95))
    # Same roundings as torch's CUDA kernels for the reference's sequence: identical bits.
    for p, r in zip(ours, ref, strict=True):
        assert torch.equal(p.detach(), r)
    key = "exp_avg" if algorithm == "adamw" else "momentum_buffer"
    for p, r in zip(ours, ref_avgs, strict=True):
        assert torch.equal(opt.state[p][key], r)
    if algorithm == "adamw":
        for p, r in zip(ours, ref_sqs, strict=True):
            assert torch.equal(opt.state[p]["exp_avg_sq"], r)
    if algorithm == "adamw":
        assert all(float(opt.state[p]["step"]) == 3.0 for p in ours)
