"""Whole-chain Newton-Schulz parity: native sm_100a chain vs the CPU oracle.

The oracle (oracle/gns_oracle.py) restates the reference's torch backend
(newton_schulz.py:66-223). Tolerance: relative Frobenius error below 2e-2 and
singular values inside the oracle's band widened by 0.02, as the reference
defines the accuracy of a backend (benchmark.py:140-165).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from gram_newton_schulz_ampere_b200 import ops
from oracle import gns_oracle as O

pytestmark = pytest.mark.gpu

REL_TOL = 2e-2
COEFFS = O.polar_express_coefficients()


def _check(out: torch.Tensor, expected: np.ndarray, tol: float = REL_TOL) -> float:
    got = out.float().cpu().numpy()
    err = O.relative_error(got, expected)
    assert err < tol, f"relative Frobenius error {err:.3e} >= {tol}"
    lo, hi = O.singular_value_band(expected)
    glo, ghi = O.singular_value_band(got)
    assert glo > lo - 0.02 and ghi < hi + 0.02, f"singular values [{glo:.3f}, {ghi:.3f}] vs oracle [{lo:.3f}, {hi:.3f}]"
    return err


@pytest.mark.parametrize(
    "shape,dtype",
    [
        ((1, 128, 256), torch.float32),
        ((2, 256, 128), torch.bfloat16),
        ((3, 64, 160), torch.bfloat16),
        ((2, 200, 72), torch.float16),
        ((2, 136, 264), torch.bfloat16),
        ((1, 5, 4), torch.float32),
        ((2, 384, 1024), torch.bfloat16),
        # several 256-blocks with a partial last block: upper block storage reads
        # tiles below the band transposed (wide and tall orientation)
        ((1, 600, 904), torch.bfloat16),
        ((1, 904, 600), torch.float16),
    ],
)
def test_gram_chain_matches_oracle(cuda_device, shape, dtype):
    gen = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(shape, generator=gen).to(dtype)
    expected = O.gram_newton_schulz(x.float().numpy(), COEFFS, (2,), 1e-7)
    out = ops.newton_schulz_chain(x.to(cuda_device), COEFFS, 1e-7, gram=True, reset_iterations=(2,))
    assert out.dtype == dtype and out.shape == x.shape
    _check(out, O.to_f16(expected))


@pytest.mark.parametrize(
    "shape,dtype",
    [
        ((2, 96, 96), torch.float32),
        ((1, 256, 256), torch.bfloat16),
        ((2, 128, 200), torch.bfloat16),
        ((2, 200, 128), torch.float16),
        ((1, 520, 520), torch.bfloat16),  # square: standard iteration over three 256-blocks
    ],
)
def test_standard_chain_matches_oracle(cuda_device, shape, dtype):
    gen = torch.Generator().manual_seed(7 + sum(shape))
    x = torch.randn(shape, generator=gen).to(dtype)
    expected = O.standard_newton_schulz(x.float().numpy(), COEFFS, 1e-7)
    out = ops.newton_schulz_chain(x.to(cuda_device), COEFFS, 1e-7, gram=False)
    _check(out, expected)


@pytest.mark.parametrize("resets", [(), (2,), (1, 3), (2, 4)])
def test_gram_reset_schedules(cuda_device, resets):
    gen = torch.Generator().manual_seed(99)
    x = torch.randn(2, 96, 256, generator=gen).bfloat16()
    expected = O.gram_newton_schulz(x.float().numpy(), COEFFS, resets, 1e-7)
    out = ops.newton_schulz_chain(x.to(cuda_device), COEFFS, 1e-7, gram=True, reset_iterations=resets)
    _check(out, expected)


def test_cfg2_like_batch(cuda_device):
    # The batched workload's statistics (N(0,1) * 1e-2, 1024 x 4096), 2 matrices for speed.
    gen = torch.Generator().manual_seed(1234)
    x = (torch.randn(2, 1024, 4096, generator=gen) * 1e-2).bfloat16()
    expected = O.gram_newton_schulz(x.float().numpy(), COEFFS, (2,), 1e-7)
    out = ops.newton_schulz_chain(x.to(cuda_device), COEFFS, 1e-7, gram=True, reset_iterations=(2,))
    _check(out, expected)


def test_empty_batch_and_missing_coefficients(cuda_device):
    x = torch.zeros(0, 8, 16, device=cuda_device, dtype=torch.bfloat16)
    assert ops.newton_schulz_chain(x, COEFFS, 1e-7, gram=True).shape == (0, 8, 16)
    with pytest.raises(RuntimeError, match="requires coefficients"):
        ops.newton_schulz_chain(torch.ones(1, 4, 8, device=cuda_device), (), 1e-7, gram=True)


@pytest.mark.parametrize("shape", [(3, 64, 160), (3, 200, 72), (3, 256, 512), (3, 96, 96), (3, 256, 256)])
@pytest.mark.parametrize("fused", [True, False])
def test_zero_matrices_give_zero_and_leave_the_batch_alone(cuda_device, shape, fused):
    # A zero update (say a parameter whose gradient is all zeros) normalises to
    # X / (0 + eps) = 0, so every product and the result are exactly zero, as in
    # the reference; the other matrices of the batch are unaffected (up to the
    # Frobenius norm's summation order, which follows the batch-dependent row
    # slicing of the normalisation: a last-bit difference at most).
    gen = torch.Generator(device=cuda_device).manual_seed(sum(shape))
    x = torch.randn(shape, generator=gen, device=cuda_device).bfloat16()
    x[1] = 0
    square = shape[-1] == shape[-2]
    with ops.small_chain_tactic(fused):
        out = ops.newton_schulz_chain(x, COEFFS, 1e-7, gram=not square, reset_iterations=(2,))
        solo = ops.newton_schulz_chain(x[2:3], COEFFS, 1e-7, gram=not square, reset_iterations=(2,))
    assert torch.count_nonzero(out[1]) == 0 and torch.isfinite(out).all()
    assert O.relative_error(out[2:3].float().cpu().numpy(), solo.float().cpu().numpy()) < 1e-3
    expected = O.gram_newton_schulz(x[:1].float().cpu().numpy(), COEFFS, (2,), 1e-7) if not square else None
    if expected is not None:
        _check(out[:1], expected)


@pytest.mark.parametrize("shape", [(3, 64, 160), (3, 256, 512), (3, 96, 96)])
@pytest.mark.parametrize("fused", [True, False])
def test_non_finite_matrix_stays_contained(cuda_device, shape, fused):
    # A matrix holding a NaN gives a NaN result, as torch's normalisation and
    # products would; the other matrices of the batch stay finite, with the fused
    # small-matrix chain and with one launch per product.
    gen = torch.Generator(device=cuda_device).manual_seed(11 + sum(shape))
    x = torch.randn(shape, generator=gen, device=cuda_device).bfloat16()
    x[1, 3, 5] = float("nan")
    square = shape[-1] == shape[-2]
    with ops.small_chain_tactic(fused):
        out = ops.newton_schulz_chain(x, COEFFS, 1e-7, gram=not square, reset_iterations=(2,))
    assert torch.isnan(out[1]).any()
    assert torch.isfinite(out[0]).all() and torch.isfinite(out[2]).all()
