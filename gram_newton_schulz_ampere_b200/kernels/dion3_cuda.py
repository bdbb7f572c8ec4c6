"""Dion3 row kernels (mirrors the entry points of kernels/dion3_cuda.py of the reference).

The reference builds an ATen extension for sm_80/86 (dion3_cuda.py:17-36) that
cannot launch on sm_100. These wrappers keep its Python names and argument
meaning and run the sm_100a kernels of ``libgns_b200.so`` instead. One
difference is by design: selected indices come back in ascending row order
(the reference's ``at::topk(..., sorted=False)`` order is unspecified), and the
selected index SET is identical.
"""

from __future__ import annotations

from collections.abc import Sequence
from math import ceil

from torch import Tensor

from gram_newton_schulz_ampere_b200 import ops
from gram_newton_schulz_ampere_b200.distributed_orthogonalization import stack_matrices


def select_dion3_rows_cuda(
    momentum: Tensor,
    gradient: Tensor,
    fraction: float,
    decay: float,
    selected_count: int | None = None,
    parameter: Tensor | None = None,
    parameter_decay: float = 1.0,
) -> tuple[Tensor, Tensor]:
    """m += g; p *= parameter_decay; top-k rows by L1 norm; bf16 gather; m[idx] *= decay
    (reference dion3_cuda.py:56-108). k defaults to max(1, ceil(fraction * rows))."""
    rows = momentum.shape[-2]
    requested = selected_count if selected_count is not None else max(1, ceil(fraction * rows))
    return ops.dion3_select_rows(momentum, gradient, parameter, min(requested, max(rows, 1)), decay, parameter_decay)


def select_dion3_rows_cuda_batch(
    momenta: Sequence[Tensor],
    gradients: Sequence[Tensor],
    parameters: Sequence[Tensor],
    selected_counts: Sequence[int],
    decay: float,
    parameter_decay: float,
) -> tuple[list[Tensor], list[Tensor]]:
    """Selection for a list of parameters (reference dion3_cuda.py:111-148). Contiguous
    2-D tensors of one shape, dtype and count run as one multi-tensor call; the
    results are views of its stacks, returned in input order."""
    count = len(momenta)
    if not (len(gradients) == count and len(parameters) == count and len(selected_counts) == count):
        raise ValueError("batched selection inputs must have equal lengths")
    for momentum, k in zip(momenta, selected_counts, strict=True):
        if not 0 < k < momentum.shape[-2]:
            raise ValueError("batched selection requires partial row selection")
    selected: list[Tensor | None] = [None] * count
    indices: list[Tensor | None] = [None] * count
    groups: dict[tuple, list[int]] = {}
    for i, (m, p) in enumerate(zip(momenta, parameters, strict=True)):
        if m.ndim == 2 and m.is_contiguous() and p.is_contiguous() and p.dtype == m.dtype:
            groups.setdefault((tuple(m.shape), m.dtype, int(selected_counts[i]), m.device), []).append(i)
        else:
            selected[i], indices[i] = ops.dion3_select_rows(
                m, gradients[i], p, selected_counts[i], decay, parameter_decay
            )
    for (_, _, k, _), members in groups.items():
        stack, idx = ops.dion3_select_rows_multi(
            [momenta[i] for i in members], [gradients[i] for i in members], [parameters[i] for i in members],
            k, decay, parameter_decay,
        )
        for slot, i in enumerate(members):
            selected[i], indices[i] = stack[slot], idx[slot]
    return selected, indices  # type: ignore[return-value]


def normalize_rows_cuda(
    selected_update: Tensor,
    variance: Tensor,
    indices: Tensor,
    beta_two: float,
    epsilon: float,
) -> tuple[Tensor, Tensor]:
    """v <- beta2 v + (1 - beta2) mean(u^2) for the selected rows; returns
    (u / (sqrt(v) + eps) in fp32, per-matrix (sum u^2, sum n^2)) (reference dion3_cuda.py:151-170)."""
    return ops.dion3_normalize_rows(selected_update, variance, indices, beta_two, epsilon)


def apply_rows_cuda(
    parameter: Tensor,
    normalized_update: Tensor,
    indices: Tensor,
    squared_norms: Tensor,
    learning_rate: float,
    weight_decay: float,
    adjusted_learning_rate: float,
    epsilon: float,
) -> None:
    """p *= 1 - lr wd; p[idx] += -lr_adj * n * |u| / max(|n|, eps) (reference dion3_cuda.py:173-192)."""
    ops.dion3_apply_rows(
        parameter, normalized_update, indices, squared_norms, learning_rate, weight_decay, adjusted_learning_rate,
        epsilon,
    )


def normalize_apply_rows_cuda(
    parameter: Tensor,
    selected_update: Tensor,
    variance: Tensor,
    indices: Tensor,
    beta_two: float,
    epsilon: float,
    learning_rate: float,
    weight_decay: float,
    adjusted_learning_rate: float,
) -> None:
    """NorMuon normalisation + norm-preserving rescale + row update (reference dion3_cuda.py:195-217)."""
    ops.dion3_normalize_apply(
        parameter, selected_update, variance, indices, beta_two, epsilon, learning_rate, weight_decay,
        adjusted_learning_rate,
    )


def normalize_apply_rows_cuda_batch(
    parameters: Sequence[Tensor],
    selected_updates: Sequence[Tensor],
    variances: Sequence[Tensor],
    indices: Sequence[Tensor],
    beta_two: float,
    epsilon: float,
    learning_rate: float,
    weight_decay: float,
    adjusted_learning_rates: Sequence[float],
) -> None:
    """Normalise + apply for a list of parameters (reference dion3_cuda.py:220-253).
    Contiguous 2-D parameters of one shape and dtype, with updates of one dtype and
    count and one adjusted learning rate, run as one multi-tensor call."""
    count = len(parameters)
    if not (
        len(selected_updates) == count
        and len(variances) == count
        and len(indices) == count
        and len(adjusted_learning_rates) == count
    ):
        raise ValueError("batched normalization inputs must have equal lengths")
    groups: dict[tuple, list[int]] = {}
    for i, p in enumerate(parameters):
        u = selected_updates[i]
        if p.ndim == 2 and p.is_contiguous() and u.ndim == 2 and variances[i].is_contiguous():
            key = (tuple(p.shape), p.dtype, u.dtype, u.shape[0], float(adjusted_learning_rates[i]), p.device)
            groups.setdefault(key, []).append(i)
        else:
            ops.dion3_normalize_apply(
                p, u, variances[i], indices[i], beta_two, epsilon, learning_rate, weight_decay,
                adjusted_learning_rates[i],
            )
    for key, members in groups.items():
        ops.dion3_normalize_apply_multi(
            [parameters[i] for i in members],
            stack_matrices([selected_updates[i] for i in members]),
            [variances[i] for i in members],
            stack_matrices([indices[i].reshape(-1) for i in members]),
            beta_two, epsilon, learning_rate, weight_decay, key[4],
        )
