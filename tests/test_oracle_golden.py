"""Pins the CPU oracle against outputs of the reference itself (tests/golden/*.npz).

The fixtures were produced by tests/golden/make_golden.py, which runs the
reference's own torch code. These tests run on the CPU.

Gram/standard Newton-Schulz: the oracle is run with ``identity_alpha_f16=True``
(torch's CPU add rounds ``alpha`` to fp16; its CUDA add does not). The one
remaining difference is the summation order of the fp32 Frobenius norm (1 ulp in
the normalised input), which the Newton-Schulz iteration amplifies to ~1e-3
relative; the pin tolerance is 4e-3, five times tighter than the 2e-2 parity
bar used for the GPU kernels.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import gns_oracle as G
from oracle import optim_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
PIN_TOL = 4e-3
DTYPES = {2: "f32", 1: "bf16", 0: "f16"}


@pytest.fixture(scope="module")
def gns():
    return np.load(GOLDEN / "gns_reference.npz")


@pytest.fixture(scope="module")
def dion3():
    return np.load(GOLDEN / "dion3_reference.npz")


@pytest.fixture(scope="module")
def muon():
    return np.load(GOLDEN / "muon_reference.npz")


def test_coefficients_match_reference(gns):
    np.testing.assert_array_equal(np.array(G.polar_express_coefficients()), gns["coefficients"])
    from gram_newton_schulz_ampere_b200.coefficients import polar_express_coefficients

    np.testing.assert_array_equal(np.array(polar_express_coefficients()), gns["coefficients"])


def _case(gns, name):
    meta = gns[f"{name}__meta"]
    dtype = DTYPES[int(meta[0])]
    gram = bool(meta[1])
    resets = tuple(int(v) for v in meta[3:])
    return gns[f"{name}__x"], gns[f"{name}__y"], dtype, gram, resets


@pytest.mark.parametrize(
    "name",
    ["cfg1", "wide_bf16", "tall_f16", "tall_bf16", "square_f32", "noreset_bf16", "resets13_bf16",
     "standard_wide_bf16", "cfg2_like_bf16"],
)
def test_newton_schulz_oracle_matches_reference(gns, name):
    x, y, dtype, gram, resets = _case(gns, name)
    out = G.orthogonalize(x, G.polar_express_coefficients(), resets, 1e-7, gram=gram, identity_alpha_f16=True)
    out = O.round_to(out, dtype)
    err = G.relative_error(out, y)
    assert err < PIN_TOL, f"{name}: oracle vs reference relative error {err:.2e}"
    assert out.shape == y.shape


def test_square_input_uses_standard_iteration(gns):
    # Reference: Gram NS on square input == standard NS exactly (tests/test_muon.py:298-301).
    x, y, dtype, _, _ = _case(gns, "square_f32")
    a = G.orthogonalize(x, gram=True)
    b = G.orthogonalize(x, gram=False)
    np.testing.assert_array_equal(a, b)


def test_singular_value_band_cfg1(gns):
    _, y, _, _, _ = _case(gns, "cfg1")
    lo, hi = G.singular_value_band(y)
    assert 0.80 < lo < 0.90 and 1.08 < hi < 1.16


def test_dion3_known_answer(dion3):
    grad = dion3["kat__grad"]
    got = O.dion3_select(np.zeros_like(grad), grad, O.selected_count(4, 0.5), 0.5)
    np.testing.assert_array_equal(got["indices"], dion3["kat__indices"])
    np.testing.assert_array_equal(got["indices"], [1, 2])
    np.testing.assert_array_equal(got["momentum"], dion3["kat__momentum"])
    np.testing.assert_array_equal(got["selected"], dion3["kat__selected"])
    res = O.dion3_normalize_apply(
        np.ones((4, 2), np.float32), got["selected"], np.zeros((4, 1), np.float32), got["indices"],
        0.9, 1e-8, 0.1, 0.2, 0.1,
    )
    np.testing.assert_allclose(res["normalized"], dion3["kat__normalized"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(res["normalized"], [[3.0, 3.0], [4.2426405, 0.0]], atol=2e-2)
    np.testing.assert_allclose(res["variance"], dion3["kat__variance"], rtol=1e-6)
    np.testing.assert_allclose(res["parameter"], dion3["kat__parameter"], rtol=1e-6, atol=1e-6)


def test_dion3_random_selection_is_bit_exact(dion3):
    got = O.dion3_select(dion3["rnd__momentum_in"], dion3["rnd__grad"], O.selected_count(64, 0.25), 0.95)
    np.testing.assert_array_equal(got["indices"], dion3["rnd__indices"])
    np.testing.assert_array_equal(got["selected"], dion3["rnd__selected"])
    np.testing.assert_array_equal(got["momentum"], dion3["rnd__momentum"])
    res = O.dion3_normalize_apply(
        dion3["rnd__parameter_in"], got["selected"], dion3["rnd__variance_in"], got["indices"],
        0.95, 1e-8, 0.01, 0.0, 0.01,
    )
    # CUDA-path rounding vs the torch twin's lerp / ratio form: equal to float32 ulps.
    np.testing.assert_allclose(res["variance"], dion3["rnd__variance"], rtol=1e-5, atol=1e-12)
    np.testing.assert_allclose(res["normalized"], dion3["rnd__normalized"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(res["parameter"], dion3["rnd__parameter"], rtol=1e-5, atol=1e-7)


def test_muon_known_answers(muon):
    g1, g2 = muon["kat__g1"], muon["kat__g2"]
    for nesterov, tag in ((False, "plain"), (True, "nesterov")):
        p = np.zeros((2, 2), np.float32)
        m = np.zeros((2, 2), np.float32)
        for g in (g1, g2):
            m, u = O.muon_momentum(g, m, 0.5, nesterov, "f32", "f32")
            p = O.muon_apply(p, u, 0.1, 0.0, 0.1, "f32")
        np.testing.assert_allclose(p, muon[f"kat_{tag}__parameter"], rtol=1e-6)
        np.testing.assert_allclose(m, muon[f"kat_{tag}__momentum"], rtol=1e-6)
    p = np.ones((8, 2), np.float32)
    _, u = O.muon_momentum(np.ones((8, 2), np.float32), np.zeros((8, 2), np.float32), 0.0, False, "f32", "f32")
    p = O.muon_apply(p, u, 0.1, 0.2, O.adjusted_learning_rate(0.1, (8, 2), "spectral_norm"), "f32")
    np.testing.assert_allclose(p, muon["decay__parameter"], rtol=1e-6)


def test_muon_bf16_steps(muon):
    p = muon["bf16__p0"].copy()
    m = np.zeros_like(p)
    lr_adj = O.adjusted_learning_rate(3e-3, p.shape, "spectral_norm")
    for g in muon["bf16__grads"]:
        m, u = O.muon_momentum(g, m, 0.95, True, "bf16", "bf16", cpu_rounding=True)
        p = O.muon_apply(p, u, 3e-3, 0.1, lr_adj, "bf16", cpu_rounding=True)
    # Bit-exact with torch's CPU bf16 rounding (alpha * y rounded before the add).
    np.testing.assert_array_equal(m, muon["bf16__momentum"])
    np.testing.assert_array_equal(p, muon["bf16__parameter"])


# ------------------------------------------------ full workload sizes
# tests/golden/baseline_shapes.npz holds the reference's outputs at full size;
# the inputs are regenerated from their seeds (tests/golden/baseline_inputs.py).


@pytest.fixture(scope="module")
def full_size():
    import sys

    sys.path.insert(0, str(GOLDEN))
    import baseline_inputs

    return baseline_inputs, np.load(GOLDEN / "baseline_shapes.npz")


def test_oracle_matches_reference_gram_1024x4096(full_size):
    import torch

    B, golden = full_size
    x = B.gram_input()
    np.testing.assert_allclose(B.input_checksum(x), golden["gram_1024x4096__input_checksum"], rtol=1e-12)
    y = G.orthogonalize(x.float().numpy(), G.polar_express_coefficients(), (2,), 1e-7, gram=True)
    y = torch.from_numpy(np.ascontiguousarray(y)).to(torch.bfloat16)[0].double()
    rows = B.from_bf16_bits(golden["gram_1024x4096__rows"]).double().numpy()
    assert G.relative_error(y[:: B.GRAM_ROW_STEP].numpy(), rows) < PIN_TOL
    sketch = (y @ B.sketch_matrix(y.shape[-1])).numpy()
    assert G.relative_error(sketch, golden["gram_1024x4096__sketch"]) < PIN_TOL


def test_oracle_dion3_selection_bit_exact_4096x4096(full_size):
    """The two matrices whose k-th and (k+1)-th row norms lie closest (relative gap
    1.5e-5 and 8.1e-5): the oracle's index sets equal the reference's."""
    import torch

    B, golden = full_size
    momentum, gradient = B.dion3_inputs()
    pick = np.argsort(golden["dion3_16x4096__boundary_gap"])[:2]
    want = golden["dion3_16x4096__indices"].astype(np.int64)[pick]
    k = want.shape[-1]
    res = O.dion3_select(momentum[pick].numpy(), gradient[pick].numpy(), k, B.DION3_DECAY)
    np.testing.assert_array_equal(res["indices"], want)
    np.testing.assert_array_equal(
        B.per_matrix_sums(torch.from_numpy(res["selected"])), golden["dion3_16x4096__selected_sums"][pick]
    )
    np.testing.assert_array_equal(
        B.per_matrix_sums(torch.from_numpy(res["momentum"])), golden["dion3_16x4096__momentum_sums"][pick]
    )


@pytest.mark.parametrize(
    "name",
    ["cfg1", "wide_bf16", "tall_f16", "tall_bf16", "square_f32", "noreset_bf16", "resets13_bf16",
     "standard_wide_bf16", "cfg2_like_bf16"],
)
def test_torch_cpu_port_reproduces_reference(gns, name):
    """The CPU baseline's torch restatement runs the reference's own operations in
    its order, so on the CPU its outputs equal the reference's bit for bit."""
    import torch

    from oracle import gns_torch_port as T

    x, y, dtype, gram, resets = _case(gns, name)
    tdtype = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    xt = torch.from_numpy(x).to(tdtype)
    coeffs = G.polar_express_coefficients()
    if gram:
        out = T.orthogonalize(xt, coeffs, resets, 1e-7)
    else:
        out = T.standard_newton_schulz(xt, coeffs, 1e-7)
    np.testing.assert_array_equal(out.float().numpy(), y)
