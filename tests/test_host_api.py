"""Host-side API behaviour that needs no GPU: validation, backend selection,
learning-rate adjustment and parameter-group bookkeeping (messages and error
types as in the reference's muon.py / dion3.py / newton_schulz.py)."""

from __future__ import annotations

import warnings

import pytest
import torch

from gram_newton_schulz_ampere_b200 import Dion3, GramNewtonSchulz, Muon
from gram_newton_schulz_ampere_b200.kernels.interface import select_matrix_backend
from gram_newton_schulz_ampere_b200.kernels.protocols import FusedNewtonSchulzBackend, MatrixBackend


def cpu_param(*shape):
    return torch.nn.Parameter(torch.zeros(*shape))


def test_backend_selection():
    backend = select_matrix_backend("b200")
    assert isinstance(backend, MatrixBackend) and isinstance(backend, FusedNewtonSchulzBackend)
    assert select_matrix_backend("b200") is backend  # cached singleton
    # The reference's backend names select the same B200 backend, with a warning
    # once per name (the selection is cached).
    select_matrix_backend.cache_clear()
    for name in ("torch", "cutlass", "triton"):
        with pytest.warns(UserWarning, match="B200 kernels"):
            assert select_matrix_backend(name) is select_matrix_backend("b200")
    with pytest.raises(ValueError, match="Unknown"):
        select_matrix_backend("tpu")


def test_reference_backend_names_select_the_b200_backend():
    # The reference's default ns_backend is "torch": code that passes it keeps working.
    for name in ("torch", "cutlass", "triton"):
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            ns = GramNewtonSchulz(ns_backend=name)
        assert ns.backend is select_matrix_backend("b200")


def test_newton_schulz_rejects_cpu_and_vectors():
    ns = GramNewtonSchulz()
    with pytest.raises(ValueError, match="CUDA"):
        ns(torch.randn(4, 8))
    with pytest.raises(TypeError):
        ns(torch.ones(4, 8, dtype=torch.int32))
    assert ns.reset_iterations == (2,) and len(ns.coefficients) == 5 and ns.gram


@pytest.mark.parametrize(
    "kwargs,exc,match",
    [
        ({"lr": -1.0}, ValueError, "Learning rate"),
        ({"momentum": 1.0}, ValueError, "Momentum"),
        ({"weight_decay": -0.1}, ValueError, "Weight decay"),
        ({"betas": (0.9, 1.0)}, ValueError, "Betas"),
        ({"epsilon": 0.0}, ValueError, "epsilon"),
        ({"ns_epsilon": 0.0}, ValueError, "Newton--Schulz epsilon"),
        ({"ns_algorithm": "svd"}, ValueError, "Newton--Schulz algorithm"),
        ({"ns_backend": "xla"}, ValueError, "Unknown Newton--Schulz kernel backend"),
        ({"adjust_lr": "sqrt"}, TypeError, "adjust_lr"),
    ],
)
def test_muon_constructor_validation(kwargs, exc, match):
    with pytest.raises(exc, match=match):
        Muon([cpu_param(2, 2)], **kwargs)


def test_callable_adjustment_rejected():
    with pytest.raises(TypeError, match="adjust_lr"):
        Muon([cpu_param(2, 2)], adjust_lr=lambda lr, shape: lr)


def test_group_validation_before_placement():
    with pytest.raises(ValueError, match="matrix parameters"):
        Muon([cpu_param(3)])
    with pytest.raises(ValueError, match="Dion3 parameter groups require the Dion3 optimizer"):
        Muon([{"params": [cpu_param(2, 2)], "algorithm": "dion3"}])
    with pytest.raises(ValueError, match="optimizer-wide"):
        Muon([{"params": [cpu_param(2, 2)], "ns_epsilon": 1e-3}])
    with pytest.raises(TypeError, match="flatten"):
        Muon([{"params": [cpu_param(2, 2)], "flatten": 1}])


def test_cpu_parameters_rejected():
    with pytest.raises(ValueError, match="CUDA parameters"):
        Muon([cpu_param(2, 2)])
    with pytest.raises(ValueError, match="CUDA parameters"):
        Dion3([cpu_param(2, 2)])


def test_dion3_group_preparation_and_validation():
    with pytest.raises(ValueError, match="at least one"):
        Dion3([])
    with pytest.raises(TypeError, match="mix"):
        Dion3([{"params": [cpu_param(2, 2)]}, cpu_param(2, 2)])
    with pytest.raises(ValueError, match="different values"):
        Dion3([cpu_param(2, 2)], momentum=0.5, mu=0.9)


def test_adjusted_learning_rate_formulas():
    adjust = Muon.adjusted_learning_rate
    assert adjust(None, 0.1, (8, 2), "spectral_norm") == pytest.approx(0.2)
    assert adjust(None, 0.1, (8, 2), "rms_norm") == pytest.approx(0.1 * 0.2 * 8**0.5)
    assert adjust(None, 0.1, (8, 2), None) == 0.1
    assert Muon.matrix_shape(None, (6, 2, 3, 3), True) == (6, 18)
    assert Muon.matrix_shape(None, (6, 2, 3, 3), False) == (6, 2, 3, 3)


def test_stack_matrices_views_consecutive_slices_without_copy():
    from gram_newton_schulz_ampere_b200.distributed_orthogonalization import stack_matrices

    block = torch.arange(3 * 4 * 5, dtype=torch.float32).reshape(3, 4, 5)
    stacked = stack_matrices(list(block.unbind(0)))
    assert stacked.data_ptr() == block.data_ptr() and torch.equal(stacked, block)
    tail = stack_matrices([block[1], block[2]])
    assert tail.data_ptr() == block[1].data_ptr() and torch.equal(tail, block[1:])
    # Anything else is copied, in the given order.
    for matrices in ([block[2], block[0]], [block[0], block[2]], [block[0], torch.zeros(4, 5)], [block[0].t(), block[1].t()]):
        got = stack_matrices(matrices)
        assert torch.equal(got, torch.stack(matrices))
        assert got.untyped_storage().data_ptr() != block.untyped_storage().data_ptr()


def test_custom_ops_registered_with_shape_only_implementations():
    # torch.compile traces the native calls as these ops; their fake versions give
    # the output's shape, dtype and layout without running anything.
    from gram_newton_schulz_ampere_b200 import ops  # noqa: F401  (registers the ops)

    x = torch.empty(2, 8, 16, device="meta", dtype=torch.bfloat16)
    y = torch.ops.gns_b200.newton_schulz_chain(x, [1.0] * 15, 1e-7, True, [2], torch.float32)
    assert y.shape == x.shape and y.dtype == torch.float32 and y.is_contiguous()
    a = torch.empty(3, 8, 16, device="meta", dtype=torch.float16)
    b = torch.empty(3, 16, 32, device="meta", dtype=torch.float16)
    assert torch.ops.gns_b200.gemm(a, b, None, 1.0, 0.0, False, None).shape == (3, 8, 32)
    assert torch.ops.gns_b200.gemm(a[0], b[0], None, 1.0, 0.0, False, torch.float32).shape == (8, 32)
