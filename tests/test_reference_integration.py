"""The drop-in into the reference package itself (CPU; skipped where the
reference is not importable, e.g. on a GPU box).

INTEGRATION.md registers ``"b200"`` in the reference with three edits and
points its Dion3 imports at this package. These tests make the same edits by
patching the imported reference modules and check that:

* the reference's own ``GramNewtonSchulz(ns_backend="b200")`` builds on
  ``B200Backend`` and routes its products to it (a CPU tensor reaches the
  native boundary and is refused loudly: there is no CPU fallback);
* the fused-chain preference snippet wires ``gram_operation`` /
  ``standard_operation`` to the backend's whole-chain entry points;
* ``B200Backend`` has the reference ``MatrixBackend`` methods with the same
  parameter names, and ``kernels/dion3_cuda`` offers every name the reference's
  ``dion3.py`` imports with the same parameters.
"""

from __future__ import annotations

import importlib
import inspect
import os
import sys
from pathlib import Path

import pytest
import torch

REFERENCE = Path(os.environ.get("GNS_REFERENCE_ROOT", "/root/reference"))
pytestmark = pytest.mark.skipif(
    not (REFERENCE / "gram_newton_schulz_ampere" / "newton_schulz.py").exists(),
    reason="the reference package is not available here",
)


@pytest.fixture(scope="module")
def reference():
    os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
    sys.path.insert(0, str(REFERENCE))
    try:
        ns = importlib.import_module("gram_newton_schulz_ampere.newton_schulz")
        protocols = importlib.import_module("gram_newton_schulz_ampere.kernels.protocols")
        yield ns, protocols
    finally:
        sys.path.remove(str(REFERENCE))


@pytest.fixture
def registered(reference, monkeypatch):
    """The reference's backend selection with INTEGRATION.md's "b200" branch."""
    ns, _ = reference
    original = ns.select_matrix_backend

    def select(name):
        if name == "b200":
            from gram_newton_schulz_ampere_b200.kernels.b200_ns import B200Backend

            return B200Backend()
        return original(name)

    monkeypatch.setattr(ns, "select_matrix_backend", select)
    return ns


def test_reference_gram_newton_schulz_runs_on_b200_backend(registered):
    from gram_newton_schulz_ampere_b200.kernels.b200_ns import B200Backend

    orthogonalizer = registered.GramNewtonSchulz(ns_backend="b200")
    assert isinstance(orthogonalizer.backend, B200Backend)
    assert not orthogonalizer.compile_operation  # the reference compiles only the torch backend
    x = torch.randn(1, 16, 48)
    with pytest.raises(ValueError, match="CUDA"):
        orthogonalizer.gram_operation(x)  # the reference's product sequence reaches the native boundary


def test_fused_chain_preference_snippet(registered):
    orthogonalizer = registered.GramNewtonSchulz(ns_backend="b200")
    backend = orthogonalizer.backend
    assert hasattr(backend, "gram_newton_schulz") and hasattr(backend, "standard_newton_schulz")
    calls = []
    backend_gram = backend.gram_newton_schulz
    try:
        backend.gram_newton_schulz = lambda m, c, r, e: calls.append(("gram", tuple(r), e)) or m
        # newton_schulz.py, after self.backend = select_matrix_backend(backend)
        coeffs, resets, eps = orthogonalizer.coefficients, orthogonalizer.reset_iterations, orthogonalizer.epsilon
        orthogonalizer.gram_operation = lambda m: orthogonalizer.backend.gram_newton_schulz(m, coeffs, resets, eps)
        orthogonalizer.gram_operation(torch.zeros(1, 2, 3))
    finally:
        backend.gram_newton_schulz = backend_gram
    assert calls == [("gram", (2,), 1e-7)]


def test_backend_methods_match_reference_protocol(reference):
    _, protocols = reference
    from gram_newton_schulz_ampere_b200.kernels.b200_ns import B200Backend

    for name in ("symmetric_matmul", "symmetric_batch_matrix_matrix_product", "matmul", "matmul_add"):
        want = list(inspect.signature(getattr(protocols.MatrixBackend, name)).parameters)
        got = list(inspect.signature(getattr(B200Backend, name)).parameters)
        assert got == want, name


def test_dion3_kernel_names_match_reference_imports(reference):
    text = (REFERENCE / "gram_newton_schulz_ampere" / "dion3.py").read_text()
    block = text.split("from gram_newton_schulz_ampere.kernels.dion3_cuda import (", 1)[1].split(")", 1)[0]
    names = [n.strip().rstrip(",") for n in block.split() if n.strip().rstrip(",")]
    assert names, "the reference's dion3.py imports no kernel names"
    ours = importlib.import_module("gram_newton_schulz_ampere_b200.kernels.dion3_cuda")
    sys.path.insert(0, str(REFERENCE))
    try:
        theirs = importlib.import_module("gram_newton_schulz_ampere.kernels.dion3_cuda")
    finally:
        sys.path.remove(str(REFERENCE))
    for name in names:
        assert hasattr(ours, name), name
        want = list(inspect.signature(getattr(theirs, name)).parameters)
        got = list(inspect.signature(getattr(ours, name)).parameters)
        assert got == want, f"{name}: {got} != {want}"
