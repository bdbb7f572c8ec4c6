"""Parity with the reference at full workload sizes (tests/golden/baseline_shapes.npz).

The fixture holds outputs of the reference's own torch code, run on the CPU by
tests/golden/make_golden.py --baseline-shapes; the inputs are regenerated here
from the same seeds (tests/golden/baseline_inputs.py) and their checksums are
compared with the ones the reference consumed before anything else is checked.

* One 1024 x 4096 bf16 matrix through ``GramNewtonSchulz(ns_backend="b200")``
  (the Gram chain), and one 4096 x 4096 bf16 matrix (the Muon q/o shape; the
  standard chain): relative Frobenius error < 2e-2 on the stored rows (every
  16th / 64th row) and on a 16-column Gaussian sketch of the whole output, and
  singular values inside the reference's band +- 0.02.
* Dion3 row selection of 16 x 4096 x 4096 fp32 with k = 1024 through the C ABI
  in one call: the selected index sets equal the reference's bit for bit, and
  per-matrix float64 checksums of the selected bf16 rows and of the updated
  momentum equal the reference's.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from gram_newton_schulz_ampere_b200 import GramNewtonSchulz, ops

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN_DIR))
import baseline_inputs as B  # noqa: E402

pytestmark = pytest.mark.gpu

REL_TOL = 2e-2  # relative Frobenius error against the reference
BAND_SLACK = 0.02  # singular values inside the reference's band +- 0.02


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN_DIR / "baseline_shapes.npz")


def _relative(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize(
    "name,make", [("gram_1024x4096", B.gram_input), ("standard_4096", B.standard_input)]
)
def test_newton_schulz_matches_reference_at_full_size(cuda_device, golden, name, make):
    x = make()
    np.testing.assert_allclose(B.input_checksum(x), golden[f"{name}__input_checksum"], rtol=1e-12)
    out = GramNewtonSchulz(ns_backend="b200")(x.to(cuda_device))
    assert out.dtype == torch.bfloat16 and out.shape == x.shape
    y = out[0].double().cpu()
    step = int(golden[f"{name}__row_step"])
    want_rows = B.from_bf16_bits(golden[f"{name}__rows"]).double().numpy()
    row_err = _relative(y[::step].numpy(), want_rows)
    sketch = (y @ B.sketch_matrix(y.shape[-1])).numpy()
    sketch_err = _relative(sketch, golden[f"{name}__sketch"])
    assert row_err < REL_TOL, f"{name}: relative error on sampled rows {row_err:.3e}"
    assert sketch_err < REL_TOL, f"{name}: relative error of the sketch {sketch_err:.3e}"
    sv = torch.linalg.svdvals(out[0].float()).double().cpu().numpy()
    ref_sv = golden[f"{name}__singular_values"]
    assert sv.min() > ref_sv.min() - BAND_SLACK and sv.max() < ref_sv.max() + BAND_SLACK, (
        f"{name}: singular values [{sv.min():.4f}, {sv.max():.4f}] vs reference "
        f"[{ref_sv.min():.4f}, {ref_sv.max():.4f}]"
    )


def test_dion3_selection_bit_exact_at_full_size(cuda_device, golden):
    momentum, gradient = B.dion3_inputs()
    np.testing.assert_allclose(
        np.stack((B.input_checksum(momentum), B.input_checksum(gradient))),
        golden["dion3_16x4096__input_checksum"], rtol=1e-12,
    )
    want = golden["dion3_16x4096__indices"].astype(np.int64)
    k = want.shape[-1]
    m = momentum.to(cuda_device)
    g = gradient.to(cuda_device)
    del momentum, gradient
    selected, indices = ops.dion3_select_rows(m, g, None, k, B.DION3_DECAY, 1.0)
    got = indices.cpu().numpy()
    assert np.array_equal(np.sort(got, axis=-1), got), "indices are emitted in ascending order"
    for b in range(want.shape[0]):
        if not np.array_equal(got[b], want[b]):
            diff = np.setxor1d(got[b], want[b])
            gap = float(golden["dion3_16x4096__boundary_gap"][b])
            raise AssertionError(f"matrix {b}: index sets differ in {diff.size} rows (boundary gap {gap:.2e})")
    np.testing.assert_allclose(
        B.per_matrix_sums(selected.cpu()), golden["dion3_16x4096__selected_sums"], rtol=1e-12, atol=0
    )
    np.testing.assert_allclose(
        B.per_matrix_sums(m.cpu()), golden["dion3_16x4096__momentum_sums"], rtol=1e-12, atol=0
    )
