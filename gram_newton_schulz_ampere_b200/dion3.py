"""Dion3 optimizer on the B200 kernels (mirrors dion3.py of the reference).

Behaviour follows the reference (dion3.py:41-354): parameter-group preparation
(groups default to ``algorithm='dion3'``), validation messages, the selected
row count ``k = max(1, ceil(fraction * rows))`` (per rank, of the padded local
row count, for row-sharded DTensors), parameter decay folded into the selection
pass, orthogonalisation of the bf16 selected rows through the distributed
layer, and the fp32 NorMuon normalisation with ``epsilon = 1e-8`` applied to
the selected rows. Only ``selection_scope='local'`` exists, as in the reference.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from math import ceil
from typing import cast

import torch
from torch import Tensor

from gram_newton_schulz_ampere_b200 import ops
from gram_newton_schulz_ampere_b200.distributed_orthogonalization import (
    local_tensor,
    orthogonalize_parameter_updates,
    parameter_layout,
    resolve_gradient,
    stack_matrices,
    validate_gradient_participation,
)
from gram_newton_schulz_ampere_b200.muon import Muon
from gram_newton_schulz_ampere_b200.optimizer_types import (
    Coefficients,
    DistributedMesh,
    LearningRate,
    LearningRateAdjustment,
    LossClosure,
    NewtonSchulzAlgorithm,
    NewtonSchulzBackend,
    OptimizerAlgorithm,
    OptimizerParameters,
    ParameterGroup,
    ParameterGroupInput,
)

NORMUON_EPSILON = 1e-8


def _as_float(value: LearningRate) -> float:
    return float(value.item()) if isinstance(value, Tensor) else float(value)


class Dion3(Muon):
    def __init__(
        self,
        params: OptimizerParameters,
        lr: float = 0.01,
        fraction: float = 0.25,
        momentum: float = 0.95,
        muon_beta2: float = 0.95,
        mu: float | None = None,
        weight_decay: float = 0.01,
        *,
        distributed_mesh: DistributedMesh = None,
        betas: tuple[float, float] = (0.9, 0.95),
        epsilon: float = 1e-8,
        adjust_lr: LearningRateAdjustment = "spectral_norm",
        selection_scope: str = "local",
        ns_algorithm: NewtonSchulzAlgorithm = "gram_newton_schulz",
        ns_epsilon: float = 1e-7,
        ns_backend: NewtonSchulzBackend = "b200",
        ns_coefficients: Coefficients | None = None,
        gram_newton_schulz_reset_iterations: Sequence[int] = (2,),
        ns_compile: bool = True,
    ) -> None:
        if mu is not None:
            if momentum != 0.95 and momentum != mu:
                raise ValueError("momentum and mu specify different values")
            momentum = mu
        groups = self.prepare_dion3_parameter_groups(params)
        super().__init__(
            groups,
            lr=lr,
            momentum=momentum,
            nesterov=False,
            weight_decay=weight_decay,
            distributed_mesh=distributed_mesh,
            betas=betas,
            epsilon=epsilon,
            adjust_lr=adjust_lr,
            flatten=False,
            ns_algorithm=ns_algorithm,
            ns_epsilon=ns_epsilon,
            ns_backend=ns_backend,
            ns_coefficients=ns_coefficients,
            gram_newton_schulz_reset_iterations=gram_newton_schulz_reset_iterations,
            ns_compile=ns_compile,
        )
        extra = {"fraction": fraction, "muon_beta2": muon_beta2, "selection_scope": selection_scope}
        self.defaults["algorithm"] = "dion3"
        self.defaults.update(extra)
        for group in self.param_groups:
            for name, value in extra.items():
                group.setdefault(name, value)
            self.validate_dion3_parameter_group(group)

    def accepts_dion3_parameter_groups(self) -> bool:
        return True

    def add_param_group(self, param_group: ParameterGroupInput) -> None:
        group = dict(param_group)
        group.setdefault("algorithm", "dion3")
        group_count = len(self.param_groups)
        known_state = set(self.state)
        try:
            super().add_param_group(group)
            if self.state_prepopulation_enabled:
                self.validate_dion3_parameter_group(self.param_groups[-1])
        except (TypeError, ValueError, RuntimeError):
            del self.param_groups[group_count:]
            for parameter in set(self.state) - known_state:
                del self.state[parameter]
            raise

    @torch.no_grad()
    def step(self, closure: LossClosure | None = None) -> float | None:  # type: ignore[override]
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        with ops.status_checked():
            for group in self.param_groups:
                algorithm = cast(OptimizerAlgorithm, group["algorithm"])
                if algorithm == "dion3":
                    self.step_dion3_group(group)
                elif algorithm == "adamw":
                    self.step_adamw_group(group)
                elif algorithm == "lion":
                    self.step_lion_group(group)
                else:
                    raise ValueError(f"Unknown Dion3 parameter algorithm: {algorithm}")
        return loss

    def prepare_dion3_parameter_groups(self, params: OptimizerParameters) -> tuple[ParameterGroup, ...]:
        inputs = list(params)
        if not inputs:
            raise ValueError("Dion3 requires at least one parameter or parameter group")
        if not isinstance(inputs[0], Mapping):
            return ({"params": inputs, "algorithm": "dion3"},)
        groups: list[ParameterGroup] = []
        for item in inputs:
            if not isinstance(item, Mapping):
                raise TypeError("Parameter inputs cannot mix groups and tensors")
            group = dict(item)
            group.setdefault("algorithm", "dion3")
            groups.append(group)
        return tuple(groups)

    def validate_dion3_parameter_group(self, group: ParameterGroup) -> None:
        algorithm = group["algorithm"]
        if algorithm == "muon":
            raise ValueError("Muon parameter groups require the Muon optimizer")
        if algorithm != "dion3":
            return
        bad = [tuple(p.shape) for p in cast(list[Tensor], group["params"]) if p.ndim < 2]
        if bad:
            raise ValueError(f"Dion3 requires matrix parameters, got {bad}")
        fraction = group["fraction"]
        if not isinstance(fraction, float) or not 0.0 < fraction <= 1.0:
            raise ValueError(f"fraction must be a float in (0, 1], got {fraction}")
        beta2 = group["muon_beta2"]
        if not isinstance(beta2, float) or not 0.0 <= beta2 < 1.0:
            raise ValueError(f"muon_beta2 must be a float in [0, 1), got {beta2}")
        if group["selection_scope"] != "local":
            raise NotImplementedError("Dion3 supports selection_scope='local' only")

    def selected_row_count(self, parameter: Tensor, fraction: float) -> tuple[int, int]:
        """(rows selected on this rank, rows of the assembled selected matrix) (dion3.py:213-229)."""
        layout = parameter_layout(parameter, self.distributed_mesh, False)
        row_dim = parameter.ndim - 2
        if layout.sharded_tensor_dimension not in (None, row_dim):
            raise NotImplementedError("Dion3 supports replicated matrices and row-sharded DTensors")
        rows = parameter.shape[-2]
        if layout.sharded_tensor_dimension == row_dim:
            if layout.process_group is None:
                raise ValueError("A row-sharded parameter requires a process group")
            world = torch.distributed.get_world_size(layout.process_group)
            local_k = max(1, ceil(fraction * ceil(rows / world)))
            return local_k, local_k * world
        k = max(1, ceil(fraction * rows))
        return k, k

    def step_dion3_group(self, group: ParameterGroup) -> None:
        all_parameters = cast(list[Tensor], group["params"])
        validate_gradient_participation(all_parameters, self.distributed_mesh, False)
        parameters = [p for p in all_parameters if p.grad is not None]
        if not parameters:
            return
        fraction = cast(float, group["fraction"])
        feedback_decay = cast(float, group["momentum"])
        lr = cast(LearningRate, group["lr"])
        wd = cast(LearningRate, group["weight_decay"])
        # Weight decay is folded into the selection pass (dion3.py:202-207).
        parameter_decay = 1.0 - _as_float(lr) * _as_float(wd)

        count = len(parameters)
        selected_updates: list[Tensor | None] = [None] * count
        selected_indices: list[Tensor | None] = [None] * count
        global_shapes: list[tuple[int, ...]] = []
        gradients, buffers, locals_, counts = [], [], [], []
        for parameter in parameters:
            local_k, global_rows = self.selected_row_count(parameter, fraction)
            gradient = resolve_gradient(parameter)
            self.reject_sparse_or_complex_gradient(gradient)
            gradients.append(gradient)
            buffers.append(local_tensor(cast(Tensor, self.state[parameter]["momentum_buffer"])))
            locals_.append(local_tensor(parameter))
            counts.append(local_k)
            global_shapes.append((*parameter.shape[:-2], global_rows, parameter.shape[-1]))
        # Matrices of one local shape, dtype and row count are selected in one
        # multi-tensor call; the selected rows come back as one stack, which is
        # the batch the orthogonaliser takes.
        buckets: dict[tuple, list[int]] = {}
        for i, (buffer, local) in enumerate(zip(buffers, locals_, strict=True)):
            if buffer.ndim == 2 and buffer.is_contiguous() and local.is_contiguous() and local.dtype == buffer.dtype \
                    and 0 < counts[i] <= buffer.shape[0]:
                buckets.setdefault((tuple(buffer.shape), buffer.dtype, counts[i]), []).append(i)
            else:
                selected_updates[i], selected_indices[i] = ops.dion3_select_rows(
                    buffers[i], gradients[i], locals_[i], counts[i], feedback_decay, parameter_decay
                )
        for (_, _, k), members in buckets.items():
            stack, idx = ops.dion3_select_rows_multi(
                [buffers[i] for i in members], [gradients[i] for i in members], [locals_[i] for i in members],
                k, feedback_decay, parameter_decay,
            )
            for slot, i in enumerate(members):
                selected_updates[i], selected_indices[i] = stack[slot], idx[slot]

        orthogonalized = orthogonalize_parameter_updates(
            parameters, cast(list[Tensor], selected_updates), global_shapes, self.newton_schulz,
            self.distributed_mesh, False,
        )
        adjust = cast(LearningRateAdjustment, group["adjust_lr"])
        beta2 = cast(float, group["muon_beta2"])
        variances = [local_tensor(cast(Tensor, self.state[p]["variance_neuron"])) for p in parameters]
        rates = [_as_float(self.adjusted_learning_rate(lr, tuple(p.shape), adjust)) for p in parameters]
        applies: dict[tuple, list[int]] = {}
        for i, (local, update) in enumerate(zip(locals_, orthogonalized, strict=True)):
            if local.ndim == 2 and local.is_contiguous() and update.ndim == 2 and variances[i].is_contiguous():
                key = (tuple(local.shape), local.dtype, update.dtype, update.shape[0], rates[i])
                applies.setdefault(key, []).append(i)
            else:
                ops.dion3_normalize_apply(
                    local, update, variances[i], cast(Tensor, selected_indices[i]), beta2, NORMUON_EPSILON,
                    _as_float(lr), 0.0, rates[i],
                )
        for key, members in applies.items():
            ops.dion3_normalize_apply_multi(
                [locals_[i] for i in members],
                stack_matrices([orthogonalized[i] for i in members]),
                [variances[i] for i in members],
                stack_matrices([cast(Tensor, selected_indices[i]) for i in members]),
                beta2, NORMUON_EPSILON, _as_float(lr), 0.0, key[4],
            )
