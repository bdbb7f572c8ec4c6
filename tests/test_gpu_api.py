"""Public API parity on the GPU: GramNewtonSchulz / StandardNewtonSchulz against the
reference's own outputs (tests/golden/gns_reference.npz, produced by the reference's
torch code), plus call semantics mirrored from the reference's tests."""

from __future__ import annotations

import warnings
from pathlib import Path

import numpy as np
import pytest
import torch

from gram_newton_schulz_ampere_b200 import GramNewtonSchulz, Muon, StandardNewtonSchulz
from gram_newton_schulz_ampere_b200.kernels.b200_ns import B200Backend
from gram_newton_schulz_ampere_b200.kernels.interface import select_matrix_backend
from gram_newton_schulz_ampere_b200.newton_schulz import build_gram_newton_schulz_operation
from oracle import gns_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "gns_reference.npz")
TORCH_DTYPES = {2: torch.float32, 1: torch.bfloat16, 0: torch.float16}
REL_TOL = 2e-2  # north-star parity bar: relative Frobenius error vs the reference


@pytest.mark.parametrize("name", [str(n) for n in GOLDEN["case_names"]])
def test_matches_reference_outputs(cuda_device, name):
    meta = GOLDEN[f"{name}__meta"]
    dtype = TORCH_DTYPES[int(meta[0])]
    gram = bool(meta[1])
    resets = tuple(int(v) for v in meta[3:])
    x = torch.from_numpy(GOLDEN[f"{name}__x"]).to(dtype).to(cuda_device)
    y = GOLDEN[f"{name}__y"]
    ns = GramNewtonSchulz(gram_newton_schulz_reset_iterations=resets) if gram else StandardNewtonSchulz()
    out = ns(x)
    assert out.dtype == dtype and out.shape == x.shape
    got = out.float().cpu().numpy()
    err = O.relative_error(got, y)
    assert err < REL_TOL, f"{name}: relative error vs reference {err:.3e}"
    lo, hi = O.singular_value_band(y)
    glo, ghi = O.singular_value_band(got)
    assert glo > lo - 0.02 and ghi < hi + 0.02


def test_square_gram_equals_standard_exactly(cuda_device):
    # Reference tests/test_muon.py:298-301: square inputs use the standard iteration.
    square = torch.randn(4, 4, device=cuda_device)
    torch.testing.assert_close(GramNewtonSchulz()(square), StandardNewtonSchulz()(square), rtol=0, atol=0)


def test_shapes_batches_and_dtypes(cuda_device):
    ns = GramNewtonSchulz()
    for shape in [(8, 4), (3, 5, 7), (2, 3, 16, 40)]:
        x = torch.randn(shape, device=cuda_device)
        out = ns(x)
        assert out.shape == x.shape and out.dtype == x.dtype and torch.isfinite(out).all()
    with pytest.raises(ValueError, match="matrix"):
        ns(torch.randn(5, device=cuda_device))
    with pytest.raises(ValueError, match="CUDA"):
        ns(torch.randn(4, 8))


def test_deterministic_and_batch_invariant(cuda_device):
    gen = torch.Generator(device=cuda_device).manual_seed(6767)
    x = torch.randn((3, 256, 64), device=cuda_device, dtype=torch.bfloat16, generator=gen)
    ns = GramNewtonSchulz()
    a, b = ns(x), ns(x)
    assert torch.equal(a, b)
    single = torch.stack([ns(x[i]) for i in range(3)])
    assert torch.equal(a, single)


def test_composed_backend_matches_fused_chain(cuda_device):
    """The reference's product sequence over B200Backend's four primitives equals the
    fused native chain to fp16 rounding."""
    x = torch.randn(2, 96, 320, device=cuda_device).bfloat16()
    backend = select_matrix_backend("b200")
    assert isinstance(backend, B200Backend)

    class PrimitivesOnly:
        symmetric_matmul = backend.symmetric_matmul
        symmetric_batch_matrix_matrix_product = backend.symmetric_batch_matrix_matrix_product
        matmul = backend.matmul
        matmul_add = backend.matmul_add

    composed = build_gram_newton_schulz_operation(PrimitivesOnly(), O.polar_express_coefficients(), (2,), 1e-7)
    fused = GramNewtonSchulz()(x)
    got = composed(x).to(torch.bfloat16)
    err = O.relative_error(got.float().cpu().numpy(), fused.float().cpu().numpy())
    assert err < 5e-3


def test_backend_primitives_match_torch(cuda_device):
    backend = B200Backend()
    x = torch.randn(2, 64, 136, device=cuda_device, dtype=torch.float16)
    g = backend.symmetric_matmul(x, x.mT)
    assert torch.equal(g, g.mT)
    torch.testing.assert_close(g.float(), x.float() @ x.float().mT, rtol=5e-3, atol=2e-2)
    p = backend.symmetric_batch_matrix_matrix_product(g, g, g, alpha=0.01, beta=0.5)
    torch.testing.assert_close(p.float(), 0.01 * (g.float() @ g.float()) + 0.5 * g.float(), rtol=5e-3, atol=5e-2)
    y = backend.matmul_add(g, x, x, beta=2.0)
    torch.testing.assert_close(y.float(), g.float() @ x.float() + 2.0 * x.float(), rtol=5e-3, atol=5e-2)
    z = backend.matmul(g, x)
    assert z.shape == (2, 64, 136)
    torch.testing.assert_close(z.float(), g.float() @ x.float(), rtol=5e-3, atol=5e-2)


def test_optimizer_state_with_a_reference_backend_name_loads(cuda_device):
    # The reference stores ns_backend (default "torch") in its parameter groups,
    # so its checkpoints carry it; loading one keeps the name and runs the same
    # kernels as ns_backend="b200".
    gen = torch.Generator(device=cuda_device).manual_seed(8)
    init = torch.randn(64, 96, generator=gen, device=cuda_device)
    grads = [torch.randn(64, 96, generator=gen, device=cuda_device) for _ in range(2)]
    a = torch.nn.Parameter(init.clone())
    b = torch.nn.Parameter(init.clone())
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        saved = Muon([a], lr=0.02, ns_backend="torch")
    plain = Muon([b], lr=0.02)
    for opt, p in ((saved, a), (plain, b)):
        p.grad = grads[0].clone()
        opt.step()
    resumed_param = torch.nn.Parameter(a.detach().clone())
    resumed = Muon([resumed_param], lr=0.02)
    resumed.load_state_dict(saved.state_dict())
    assert resumed.ns_backend == "torch" and resumed.param_groups[0]["ns_backend"] == "torch"
    for opt, p in ((resumed, resumed_param), (plain, b)):
        p.grad = grads[1].clone()
        opt.step()
    assert torch.equal(resumed_param, b)


def test_reference_backend_names_run_the_b200_kernels(cuda_device):
    # Code written for the reference (default ns_backend="torch") keeps working
    # and gets the same bits as ns_backend="b200".
    x = torch.randn(3, 96, 200, generator=torch.Generator(device=cuda_device).manual_seed(4), device=cuda_device)
    want = GramNewtonSchulz(ns_backend="b200")(x)
    for name in ("torch", "cutlass", "triton"):
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            got = GramNewtonSchulz(ns_backend=name)(x)
        assert torch.equal(got, want)
