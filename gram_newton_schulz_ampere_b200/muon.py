"""Muon optimizer on the B200 kernels (mirrors muon.py of the reference).

Public behaviour follows the reference (muon.py:37-594): constructor arguments
and validation messages, per-group algorithms (muon / adamw / lion), state
names and dtypes (``momentum_buffer``; ``step``/``exp_avg``/``exp_avg_sq``),
``state_dict`` round trips that restore the Newton-Schulz configuration, and
atomic ``add_param_group``.

The Muon group step is three native stages per group:
  1. one fused multi-tensor momentum kernel (m <- g + mu m, Nesterov u = g + mu m),
  2. the orthogonalisation (bucketed, round-robin / sharded over ranks),
  3. one fused multi-tensor update kernel (p <- p (1 - lr wd) - lr_adj O).
With replicated (non-DTensor) parameters on more than one rank, stages 2 and 3
run per bucket on the owner rank only: the owner of a matrix (the reference's
round-robin, distributed_orthogonalization.py:241-252) orthogonalises it and
applies the update to its copy of the parameter, and the bucket's updated
parameters are all-gathered into every rank's copies while the next bucket is
being orthogonalised. The reference instead all-gathers the orthogonalised updates
and every rank applies every update (muon.py:399-476); both leave every rank
with the same bits, but here the update pass and the update writes of the
momentum kernel shrink to the owned 1/W share.
AdamW and Lion groups (vectors and scalars) are one fused multi-tensor kernel
per dtype combination. Under DistributedDataParallel, ``momentum_comm_hook()``
moves stage 1 into the backward pass: each gradient bucket's momentum runs as
soon as its all-reduce has landed.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from math import sqrt
from typing import cast

import torch
import torch.distributed as dist
from torch import Tensor
from torch.distributed.tensor import DTensor
from torch.optim.optimizer import Optimizer, StateDict

from gram_newton_schulz_ampere_b200 import ops
from gram_newton_schulz_ampere_b200.coefficients import polar_express_coefficients
from gram_newton_schulz_ampere_b200.distributed_orthogonalization import (
    configured_process_group,
    local_tensor,
    orthogonalize_parameter_updates,
    resolve_gradient,
    round_robin_owners,
    gather_owned_tensors,
    send_owned_tensors,
    stack_matrices,
    validate_gradient_participation,
)
from gram_newton_schulz_ampere_b200.newton_schulz import GramNewtonSchulz, StandardNewtonSchulz
from gram_newton_schulz_ampere_b200.optimizer_types import (
    REFERENCE_BACKEND_NAMES,
    SUPPORTED_BACKENDS,
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

NS_SETTINGS = ("ns_algorithm", "ns_epsilon", "ns_backend", "ns_coefficients", "gram_newton_schulz_reset_iterations")
ALGORITHMS = frozenset({"muon", "dion3", "adamw", "lion"})
ADJUSTMENTS = frozenset({"spectral_norm", "rms_norm"})


def orthogonalization_flops(shape: tuple[int, ...]) -> float:
    """Algorithmic flops of one orthogonalisation: 20 n^3 for a square matrix
    (standard iteration), 6 m^2 n + 14 m^3 otherwise (m, n = short, long side)."""
    rows, cols = shape[-2], shape[-1]
    m, n = min(rows, cols), max(rows, cols)
    return 20.0 * n**3 if m == n else 6.0 * m * m * n + 14.0 * m**3


def exchange_order(buckets: list[list[int]], shapes: list[tuple[int, ...]], parameters: list[Tensor]) -> list[list[int]]:
    """Processing order of replicated buckets: each bucket's exchange overlaps the
    orthogonalisation of the buckets after it, so only the last bucket's exchange
    is exposed. The last is the bucket with the most work per exchanged byte
    (its orthogonalisation best hides the one before it, its own exchange is
    small); the others run in decreasing order of work. Numerics do not depend
    on the order."""
    def work(indices: list[int]) -> float:
        return len(indices) * orthogonalization_flops(shapes[indices[0]])

    def nbytes(indices: list[int]) -> float:
        p = parameters[indices[0]]
        return float(len(indices) * p.numel() * p.element_size()) or 1.0

    ordered = sorted(buckets, key=work, reverse=True)
    if len(ordered) > 2:
        last = max(ordered[1:], key=lambda b: work(b) / nbytes(b))
        ordered.remove(last)
        ordered.append(last)
    return ordered


def _freeze_coefficients(values: Coefficients) -> tuple[tuple[float, ...], ...]:
    return tuple(tuple(float(v) for v in triple) for triple in values)


class Muon(Optimizer):
    def __init__(
        self,
        params: OptimizerParameters,
        lr: float = 0.02,
        momentum: float = 0.95,
        nesterov: bool = True,
        weight_decay: float = 0.0,
        *,
        distributed_mesh: DistributedMesh = None,
        betas: tuple[float, float] = (0.9, 0.95),
        epsilon: float = 1e-8,
        adjust_lr: LearningRateAdjustment = "spectral_norm",
        flatten: bool = False,
        ns_algorithm: NewtonSchulzAlgorithm = "gram_newton_schulz",
        ns_epsilon: float = 1e-7,
        ns_backend: NewtonSchulzBackend = "b200",
        ns_coefficients: Coefficients | None = None,
        gram_newton_schulz_reset_iterations: Sequence[int] = (2,),
        ns_compile: bool = True,
    ) -> None:
        self.validate_constructor_values(
            lr=lr,
            momentum=momentum,
            weight_decay=weight_decay,
            betas=betas,
            epsilon=epsilon,
            ns_epsilon=ns_epsilon,
            ns_algorithm=ns_algorithm,
            ns_backend=ns_backend,
            adjust_lr=adjust_lr,
        )
        self.distributed_mesh = distributed_mesh
        self.ns_algorithm = ns_algorithm
        self.ns_epsilon = ns_epsilon
        self.ns_backend = ns_backend
        self.ns_coefficients = _freeze_coefficients(
            polar_express_coefficients() if ns_coefficients is None else ns_coefficients
        )
        self.gram_newton_schulz_reset_iterations = tuple(gram_newton_schulz_reset_iterations)
        self.ns_compile = ns_compile
        self.state_prepopulation_enabled = False
        defaults: ParameterGroup = {
            "lr": lr,
            "momentum": momentum,
            "nesterov": nesterov,
            "weight_decay": weight_decay,
            "algorithm": "muon",
            "betas": betas,
            "epsilon": epsilon,
            "adjust_lr": adjust_lr,
            "flatten": flatten,
            **self.newton_schulz_settings(),
        }
        super().__init__(params, defaults)
        for group in self.param_groups:
            self.validate_parameter_group(group)
        self.validate_cuda_configuration()
        self.configure_newton_schulz()
        for group in self.param_groups:
            self.initialize_parameter_group_state(group)
        self.state_prepopulation_enabled = True

    # ---------------------------------------------------------- configuration
    def newton_schulz_settings(self) -> ParameterGroup:
        return {
            "ns_algorithm": self.ns_algorithm,
            "ns_epsilon": self.ns_epsilon,
            "ns_backend": self.ns_backend,
            "ns_coefficients": self.ns_coefficients,
            "gram_newton_schulz_reset_iterations": self.gram_newton_schulz_reset_iterations,
        }

    def configure_newton_schulz(self) -> None:
        if self.ns_algorithm == "gram_newton_schulz":
            self.newton_schulz = GramNewtonSchulz(
                ns_epsilon=self.ns_epsilon,
                ns_backend=self.ns_backend,
                ns_coefficients=self.ns_coefficients,
                gram_newton_schulz_reset_iterations=self.gram_newton_schulz_reset_iterations,
                ns_compile=self.ns_compile,
            )
        elif self.ns_algorithm == "standard_newton_schulz":
            self.newton_schulz = StandardNewtonSchulz(
                ns_epsilon=self.ns_epsilon,
                ns_backend=self.ns_backend,
                ns_coefficients=self.ns_coefficients,
                ns_compile=self.ns_compile,
            )
        else:
            raise ValueError(f"Unknown Newton--Schulz algorithm: {self.ns_algorithm}")

    def load_state_dict(self, state_dict: StateDict) -> None:
        super().load_state_dict(state_dict)
        first = self.param_groups[0]
        self.ns_algorithm = cast(NewtonSchulzAlgorithm, first.get("ns_algorithm", self.ns_algorithm))
        self.ns_epsilon = cast(float, first.get("ns_epsilon", self.ns_epsilon))
        self.ns_backend = cast(NewtonSchulzBackend, first.get("ns_backend", self.ns_backend))
        self.ns_coefficients = _freeze_coefficients(
            cast(Coefficients, first.get("ns_coefficients", self.ns_coefficients))
        )
        self.gram_newton_schulz_reset_iterations = tuple(
            cast(Sequence[int], first.get("gram_newton_schulz_reset_iterations", self.gram_newton_schulz_reset_iterations))
        )
        settings = self.newton_schulz_settings()
        self.defaults.update(settings)
        for group in self.param_groups:
            for name, value in settings.items():
                if group.get(name, value) != value:
                    raise ValueError(f"Checkpoint has inconsistent Newton--Schulz setting {name}")
                group[name] = value
            self.initialize_parameter_group_state(group)
        self.validate_cuda_configuration()
        self.configure_newton_schulz()

    def add_param_group(self, param_group: ParameterGroupInput) -> None:
        group_count = len(self.param_groups)
        known_state = set(self.state)
        try:
            super().add_param_group(dict(param_group))
            if self.state_prepopulation_enabled:
                added = self.param_groups[-1]
                self.validate_parameter_group(added)
                self.validate_cuda_configuration()
                self.initialize_parameter_group_state(added)
        except (TypeError, ValueError, RuntimeError):
            del self.param_groups[group_count:]
            for parameter in set(self.state) - known_state:
                del self.state[parameter]
            raise

    # ---------------------------------------------------------------- step
    def step(self, closure: LossClosure | None = None) -> float | None:  # type: ignore[override]
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        with torch.no_grad(), ops.status_checked():
            for group in self.param_groups:
                algorithm = cast(OptimizerAlgorithm, group["algorithm"])
                if algorithm == "muon":
                    self.step_muon_group(group)
                elif algorithm == "adamw":
                    self.step_adamw_group(group)
                elif algorithm == "lion":
                    self.step_lion_group(group)
                else:
                    raise ValueError(f"Unknown optimizer algorithm: {algorithm}")
        return loss

    # ----------------------------------------------------------- validation
    def validate_constructor_values(
        self,
        lr: float,
        momentum: float,
        weight_decay: float,
        betas: tuple[float, float],
        epsilon: float,
        ns_epsilon: float,
        ns_algorithm: NewtonSchulzAlgorithm,
        ns_backend: NewtonSchulzBackend,
        adjust_lr: LearningRateAdjustment,
    ) -> None:
        if lr < 0.0:
            raise ValueError(f"Learning rate must be non-negative, got {lr}")
        if not 0.0 <= momentum < 1.0:
            raise ValueError(f"Momentum must be in [0, 1), got {momentum}")
        if weight_decay < 0.0:
            raise ValueError(f"Weight decay must be non-negative, got {weight_decay}")
        if not (0.0 <= betas[0] < 1.0 and 0.0 <= betas[1] < 1.0):
            raise ValueError(f"Betas must be in [0, 1), got {betas}")
        if epsilon <= 0.0:
            raise ValueError(f"AdamW epsilon must be positive, got {epsilon}")
        if ns_epsilon <= 0.0:
            raise ValueError(f"Newton--Schulz epsilon must be positive, got {ns_epsilon}")
        if ns_algorithm not in ("gram_newton_schulz", "standard_newton_schulz"):
            raise ValueError(f"Unknown Newton--Schulz algorithm: {ns_algorithm}")
        if ns_backend not in SUPPORTED_BACKENDS and ns_backend not in REFERENCE_BACKEND_NAMES:
            raise ValueError(f"Unknown Newton--Schulz kernel backend: {ns_backend}")
        if adjust_lr is not None and adjust_lr not in ADJUSTMENTS:
            raise TypeError("adjust_lr must be spectral_norm, rms_norm, or None")

    def accepts_dion3_parameter_groups(self) -> bool:
        return False

    def validate_parameter_group(self, group: ParameterGroup) -> None:
        algorithm = group["algorithm"]
        if algorithm not in ALGORITHMS:
            raise ValueError(f"Unknown optimizer algorithm: {algorithm}")
        if algorithm == "dion3" and not self.accepts_dion3_parameter_groups():
            raise ValueError("Dion3 parameter groups require the Dion3 optimizer")
        for name, expected in self.newton_schulz_settings().items():
            if group[name] != expected:
                raise ValueError(f"Newton--Schulz setting {name} must be optimizer-wide")
        if algorithm in ("muon", "dion3"):
            bad = [tuple(p.shape) for p in cast(list[Tensor], group["params"]) if p.ndim < 2]
            if bad:
                raise ValueError(
                    "Orthogonal optimizer groups require matrix parameters. Put scalar "
                    f"and vector parameters in an adamw or lion group. Invalid shapes: {bad}"
                )
        self.validate_nonnegative_group_scalar(group, "lr")
        self.validate_nonnegative_group_scalar(group, "weight_decay")
        momentum = group["momentum"]
        if not isinstance(momentum, float) or not 0.0 <= momentum < 1.0:
            raise ValueError(f"Momentum must be a float in [0, 1), got {momentum}")
        betas = group["betas"]
        if not isinstance(betas, tuple) or len(betas) != 2:
            raise ValueError(f"Betas must be a pair, got {betas}")
        if not all(isinstance(b, float) and 0.0 <= b < 1.0 for b in betas):
            raise ValueError(f"Betas must be floats in [0, 1), got {betas}")
        epsilon = group["epsilon"]
        if not isinstance(epsilon, float) or epsilon <= 0.0:
            raise ValueError(f"Epsilon must be a positive float, got {epsilon}")
        if not isinstance(group["flatten"], bool):
            raise TypeError(f"flatten must be bool, got {type(group['flatten']).__name__}")
        adjust = group["adjust_lr"]
        if adjust is not None and adjust not in ADJUSTMENTS:
            raise TypeError("adjust_lr must be spectral_norm, rms_norm, or None")

    def validate_nonnegative_group_scalar(self, group: ParameterGroup, name: str) -> None:
        value = group[name]
        if isinstance(value, Tensor):
            if value.numel() != 1 or bool((value < 0).item()):
                raise ValueError(f"{name} must be a non-negative scalar, got {value}")
            return
        if not isinstance(value, float) or value < 0.0:
            raise ValueError(f"{name} must be a non-negative float, got {value}")

    def validate_cuda_configuration(self) -> None:
        devices = {local_tensor(p).device for g in self.param_groups for p in cast(list[Tensor], g["params"])}
        if any(d.type != "cuda" for d in devices):
            raise ValueError("Muon and Dion3 require CUDA parameters")
        if len(devices) > 1:
            raise ValueError("One optimizer cannot span multiple CUDA devices")
        group = configured_process_group(self.distributed_mesh)
        if group is not None and torch.distributed.get_backend(group) != torch.distributed.Backend.NCCL:
            raise ValueError("Distributed Muon and Dion3 require an NCCL process group")

    def initialize_parameter_group_state(self, group: ParameterGroup) -> None:
        algorithm = group["algorithm"]
        for parameter in cast(list[Tensor], group["params"]):
            state = self.state[parameter]
            if algorithm in ("muon", "dion3", "lion") and "momentum_buffer" not in state:
                state["momentum_buffer"] = torch.zeros_like(parameter)
            if algorithm == "dion3":
                variance = state.get("variance_neuron")
                if variance is None:
                    state["variance_neuron"] = torch.zeros_like(parameter[..., :1], dtype=torch.float32)
                elif cast(Tensor, variance).dtype != torch.float32:
                    state["variance_neuron"] = cast(Tensor, variance).float()
            elif algorithm == "adamw":
                if "step" not in state:
                    state["step"] = torch.zeros((), dtype=torch.float32, device=local_tensor(parameter).device)
                if "exp_avg" not in state:
                    state["exp_avg"] = torch.zeros_like(parameter)
                if "exp_avg_sq" not in state:
                    state["exp_avg_sq"] = torch.zeros_like(parameter)

    def reject_sparse_or_complex_gradient(self, gradient: Tensor) -> None:
        if gradient.is_sparse:
            raise RuntimeError("Muon does not support sparse gradients")
        if gradient.is_complex():
            raise RuntimeError("Muon does not support complex gradients")

    # -------------------------------------------------------------- shapes
    def reshape_for_orthogonalization(self, update: Tensor, global_shape: tuple[int, ...], flatten: bool) -> Tensor:
        if not flatten or len(global_shape) == 2:
            return update
        return update.reshape(update.shape[0], -1)

    def matrix_shape(self, global_shape: tuple[int, ...], flatten: bool) -> tuple[int, ...]:
        if not flatten or len(global_shape) == 2:
            return global_shape
        columns = 1
        for size in global_shape[1:]:
            columns *= size
        return (global_shape[0], columns)

    def adjusted_learning_rate(
        self,
        learning_rate: LearningRate,
        matrix_shape: tuple[int, ...],
        adjustment: LearningRateAdjustment,
    ) -> LearningRate:
        """lr * sqrt(rows / cols) ("spectral_norm") or lr * 0.2 * sqrt(max(rows, cols)) ("rms_norm")."""
        if adjustment is None:
            return learning_rate
        rows, columns = matrix_shape[-2], matrix_shape[-1]
        if adjustment == "spectral_norm":
            return learning_rate * sqrt(rows / columns)
        if adjustment == "rms_norm":
            return learning_rate * 0.2 * sqrt(max(rows, columns))
        raise ValueError(f"Unknown learning-rate adjustment: {adjustment}")

    # ------------------------------------------------------------ Muon group
    def _momentum_updates(
        self, parameters: list[Tensor], momentum: float, nesterov: bool, gradients: list[Tensor] | None = None
    ) -> list[Tensor]:
        """Runs the fused momentum kernel per (grad dtype, momentum dtype) class; returns the
        tensors to orthogonalise, in parameter order. Updates already formed by
        ``momentum_comm_hook`` during backward are taken as they are."""
        pending = self.__dict__.get("_hooked_updates", {})
        if gradients is None and pending:
            ready = [pending.pop(id(p), None) for p in parameters]
            for u in ready:
                if u is not None:
                    # Formed on the hook's callback stream, consumed on this one.
                    u.record_stream(torch.cuda.current_stream(u.device))
            rest = [p for p, u in zip(parameters, ready, strict=True) if u is None]
            computed = iter(self._momentum_updates(rest, momentum, nesterov) if rest else [])
            return [u if u is not None else next(computed) for u in ready]
        given = gradients
        gradients = []
        buffers: list[Tensor] = []
        for index, parameter in enumerate(parameters):
            gradient = resolve_gradient(parameter) if given is None else given[index]
            self.reject_sparse_or_complex_gradient(gradient)
            gradients.append(gradient.contiguous())
            buffers.append(local_tensor(cast(Tensor, self.state[parameter]["momentum_buffer"])))
        classes: dict[tuple[torch.dtype, torch.dtype], list[int]] = {}
        for index, (g, m) in enumerate(zip(gradients, buffers, strict=True)):
            classes.setdefault((g.dtype, m.dtype), []).append(index)
        updates: list[Tensor | None] = [None] * len(parameters)
        for indices in classes.values():
            produced = ops.muon_momentum([gradients[i] for i in indices], [buffers[i] for i in indices], momentum, nesterov)
            for slot, index in enumerate(indices):
                if produced is not None:
                    updates[index] = produced[slot]
                elif momentum == 0.0:
                    updates[index] = gradients[index]
                else:
                    updates[index] = buffers[index]
        return cast(list[Tensor], updates)

    # ------------------------------------------ DDP gradient-bucket overlap
    def momentum_comm_hook(
        self, process_group: dist.ProcessGroup | None = None
    ) -> Callable[[object, dist.GradBucket], torch.futures.Future[Tensor]]:
        """A DistributedDataParallel communication hook for ``register_comm_hook``.

        Each gradient bucket is averaged and all-reduced as by DDP's default hook;
        once the all-reduce has landed, the fused momentum kernel runs on the
        bucket's parameters of Muon groups (m <- g + mu m and, for Nesterov,
        u = g + mu m), on the stream of the future's callback, so the momentum
        pass overlaps the rest of the backward pass instead of running in
        ``step()``. ``step()`` then orthogonalises the stored updates; parameters
        whose bucket did not run this way take the usual path.

        Contract (the momentum buffers are updated during backward): the
        gradients must reach ``step()`` unchanged (no clipping or unscaling in
        between), and every backward pass with the hook must be followed by
        ``step()``. Groups with momentum 0 are left to ``step()``.
        """

        # Unannotated: DistributedDataParallel.register_comm_hook compares the
        # annotations with the classes themselves, not with postponed strings.
        def hook(state, bucket):  # type: ignore[no-untyped-def]
            group = process_group if process_group is not None else dist.group.WORLD
            buffer = bucket.buffer()
            buffer.div_(dist.get_world_size(group))
            future = dist.all_reduce(buffer, group=group, async_op=True).get_future()

            def momentum(done: torch.futures.Future[list[Tensor]]) -> Tensor:
                reduced = done.value()[0]
                with torch.no_grad():
                    self._bucket_momentum(list(bucket.parameters()), list(bucket.gradients()))
                return reduced

            return future.then(momentum)

        return hook

    def _bucket_momentum(self, parameters: list[Tensor], gradients: list[Tensor]) -> None:
        """Momentum of the Muon-group parameters among `parameters` (gradients: the
        all-reduced bucket views); the updates wait in ``_hooked_updates`` for step()."""
        owner: dict[int, ParameterGroup] = {}
        for group in self.param_groups:
            if group["algorithm"] == "muon" and cast(float, group["momentum"]) != 0.0:
                for p in cast(list[Tensor], group["params"]):
                    owner[id(p)] = group
        chosen: dict[int, tuple[ParameterGroup, list[Tensor], list[Tensor]]] = {}
        for p, g in zip(parameters, gradients, strict=True):
            group = owner.get(id(p))
            if group is None:
                continue
            entry = chosen.setdefault(id(group), (group, [], []))
            entry[1].append(p)
            entry[2].append(g.view(p.shape))
        pending = self.__dict__.setdefault("_hooked_updates", {})
        for group, params, grads in chosen.values():
            updates = self._momentum_updates(
                params, cast(float, group["momentum"]), cast(bool, group["nesterov"]), gradients=grads
            )
            for p, u in zip(params, updates, strict=True):
                pending[id(p)] = u

    def step_muon_group(self, group: ParameterGroup) -> None:
        all_parameters = cast(list[Tensor], group["params"])
        flatten = cast(bool, group["flatten"])
        validate_gradient_participation(all_parameters, self.distributed_mesh, flatten)
        parameters = [p for p in all_parameters if p.grad is not None]
        if not parameters:
            return
        if self._owner_apply_eligible(group, parameters):
            self._step_replicated_owner_apply(group, parameters)
            return
        self._mark("start")
        updates = self._momentum_updates(parameters, cast(float, group["momentum"]), cast(bool, group["nesterov"]))
        self._mark("momentum")
        shapes = [self.matrix_shape(tuple(p.shape), flatten) for p in parameters]
        matrices = [
            self.reshape_for_orthogonalization(u, tuple(p.shape), flatten)
            for u, p in zip(updates, parameters, strict=True)
        ]
        orthogonalized = orthogonalize_parameter_updates(
            parameters, matrices, shapes, self.newton_schulz, self.distributed_mesh, flatten
        )
        self._mark("orthogonalized")
        self.apply_orthogonal_updates(group, parameters, orthogonalized, shapes)
        self._mark("applied")

    # ------------------------------------- replicated parameters, W > 1
    # Records (label, CUDA event) pairs at the stage boundaries of the next steps
    # when set to a list (bench.py's breakdown); None records nothing.
    phase_events: list[tuple[str, torch.cuda.Event]] | None = None
    # How owners hand updated parameters to the other ranks: "all_gather" (NCCL
    # all-gather of each bucket's owned parameters into a staging buffer, then a
    # copy into place) or "p2p" (point-to-point sends straight into place).
    replicated_exchange: str = "all_gather"
    # True (the default): each replicated bucket's parameters are moved, on the
    # first step, into one contiguous buffer in bucket order (``p.data`` becomes
    # a view of it; values unchanged). Every rank's owned parameters are then one
    # slice of that buffer, and the exchange is a single in-place all-gather into
    # the parameters themselves: no staging buffer and no copy into place. Set it
    # to False where something else relies on the parameters' storage staying
    # where it was allocated; the exchange then gathers through a staging buffer.
    contiguous_buckets: bool = True
    # SMs left to the collectives while a bucket is orthogonalised beside the
    # previous bucket's all-gather (every bucket but the first): the GEMMs then
    # use the others (gns_set_gemm_sm_limit). 0 disables the cap.
    collective_sm_reserve: int = 32
    # Momentum of the matrices a rank does not own is needed only by the next
    # step: it runs after the last bucket's orthogonalisation, while that
    # bucket's exchange is in flight (True), or up front with the owned ones.
    defer_momentum: bool = True

    def _mark(self, label: str) -> None:
        if self.phase_events is not None:
            event = torch.cuda.Event(enable_timing=True)
            event.record()
            self.phase_events.append((label, event))

    def _owner_apply_eligible(self, group: ParameterGroup, parameters: list[Tensor]) -> bool:
        process_group = configured_process_group(self.distributed_mesh)
        if process_group is None or dist.get_world_size(process_group) == 1:
            return False
        hooked = self.__dict__.get("_hooked_updates")
        if hooked and not all(id(p) in hooked for p in parameters):
            return False  # some but not all updates formed during backward: the generic path
        if not (isinstance(group["lr"], float) and isinstance(group["weight_decay"], float)):
            return False
        return all(not isinstance(p, DTensor) and p.is_contiguous() for p in parameters)

    def _step_replicated_owner_apply(self, group: ParameterGroup, parameters: list[Tensor]) -> None:
        """Momentum on every rank; orthogonalisation and update on the owner, then an
        exchange that gives every rank the owner's parameter.

        Buckets and owners are the reference's (same keys, first-seen order,
        contiguous ceil(n/W) slices). The momentum kernel writes Nesterov updates
        only for this rank's matrices. Buckets run in decreasing order of work so
        that the exchange of each overlaps the orthogonalisation of the next and
        the last (cheapest) exchange is the only one left exposed.
        """
        process_group = cast(dist.ProcessGroup, configured_process_group(self.distributed_mesh))
        world = dist.get_world_size(process_group)
        rank = dist.get_rank(process_group)
        flatten = cast(bool, group["flatten"])
        mu = cast(float, group["momentum"])
        nesterov = cast(bool, group["nesterov"])
        gradients = []
        for parameter in parameters:
            gradient = resolve_gradient(parameter)
            self.reject_sparse_or_complex_gradient(gradient)
            gradients.append(gradient.contiguous())
        buffers = [local_tensor(cast(Tensor, self.state[p]["momentum_buffer"])) for p in parameters]
        shapes = [self.matrix_shape(tuple(p.shape), flatten) for p in parameters]

        def update_dtype(g: Tensor, m: Tensor) -> torch.dtype:
            if mu == 0.0:
                return g.dtype
            return torch.promote_types(g.dtype, m.dtype) if nesterov else m.dtype

        buckets: dict[tuple, list[int]] = {}
        for index, parameter in enumerate(parameters):
            key = (tuple(parameter.shape), shapes[index], update_dtype(gradients[index], buffers[index]),
                   parameter.device)
            buckets.setdefault(key, []).append(index)
        rounds = exchange_order(list(buckets.values()), shapes, parameters)
        owner = [0] * len(parameters)
        for indices in rounds:
            for index, rank_of in zip(indices, round_robin_owners(len(indices), world), strict=True):
                owner[index] = rank_of
        mine = [o == rank for o in owner]

        # The side stream copies each bucket's gathered parameters into place as
        # soon as its all-gather lands, while later buckets are orthogonalised.
        device = parameters[0].device
        compute = torch.cuda.current_stream(device) if parameters[0].is_cuda else None
        side = self._side_stream(device) if compute is not None else None
        if side is not None:
            side.wait_stream(compute)

        self._mark("start")
        updates: list[Tensor | None] = [None] * len(parameters)
        deferred: dict[tuple[torch.dtype, torch.dtype], list[int]] = {}
        classes: dict[tuple[torch.dtype, torch.dtype], list[int]] = {}
        hooked = self.__dict__.get("_hooked_updates", {})
        if hooked:
            # momentum_comm_hook already advanced every momentum buffer and formed
            # the updates during backward, on its callback stream.
            for index, p in enumerate(parameters):
                u = hooked.pop(id(p))
                if u.is_cuda:
                    u.record_stream(torch.cuda.current_stream(u.device))
                updates[index] = u
        else:
            for index, (g, m) in enumerate(zip(gradients, buffers, strict=True)):
                later = self.defer_momentum and not mine[index]
                (deferred if later else classes).setdefault((g.dtype, m.dtype), []).append(index)

        def momentum_pass(chosen: dict[tuple[torch.dtype, torch.dtype], list[int]]) -> None:
            for indices in chosen.values():
                produced = ops.muon_momentum(
                    [gradients[i] for i in indices], [buffers[i] for i in indices], mu, nesterov,
                    wanted=[mine[i] for i in indices],
                )
                for slot, index in enumerate(indices):
                    if produced is not None:
                        updates[index] = produced[slot]
                    else:
                        updates[index] = gradients[index] if mu == 0.0 else buffers[index]

        momentum_pass(classes)
        self._mark("momentum")

        pending: list[dist.Work] = []
        sm_count = torch.cuda.get_device_properties(device).multi_processor_count if compute is not None else 0
        reserve = self.collective_sm_reserve if 0 < self.collective_sm_reserve < sm_count else 0
        previous_limit = None
        try:
            for position, indices in enumerate(rounds):
                if reserve and position == 1:
                    previous_limit = ops.gemm_sm_limit(sm_count - reserve)
                owned = [i for i in indices if mine[i]]
                if owned:
                    matrices = [
                        self.reshape_for_orthogonalization(cast(Tensor, updates[i]), tuple(parameters[i].shape), flatten)
                        for i in owned
                    ]
                    orthogonalized = list(self.newton_schulz(stack_matrices(matrices)).unbind(0))
                    self._mark("orthogonalized {}x{}".format(*shapes[owned[0]][-2:]))
                    self.apply_orthogonal_updates(group, [parameters[i] for i in owned], orthogonalized,
                                                  [shapes[i] for i in owned])
                    self._mark("applied")
                tensors = [parameters[i].detach() for i in indices]
                flat = self._contiguous_bucket([parameters[i] for i in indices], world) if self.contiguous_buckets else None
                if flat is not None:
                    per_rank = flat.shape[0] // world
                    mine_slice = flat[rank * per_rank:(rank + 1) * per_rank]
                    if dist.get_backend(process_group) == "gloo":
                        pending.append(dist.all_gather(list(flat.chunk(world)), mine_slice.clone(),
                                                       group=process_group, async_op=True))
                    else:
                        pending.append(dist.all_gather_into_tensor(flat, mine_slice, group=process_group, async_op=True))
                elif self.replicated_exchange == "p2p":
                    pending += send_owned_tensors(tensors, [owner[i] for i in indices], process_group)
                else:
                    gathered = gather_owned_tensors(tensors, [owner[i] for i in indices], process_group)
                    if side is None:
                        gathered.finish()
                    else:
                        with torch.cuda.stream(side):
                            gathered.finish()
        finally:
            if previous_limit is not None:
                ops.gemm_sm_limit(previous_limit)
        if deferred:
            momentum_pass(deferred)
            self._mark("deferred_momentum")
        for request in pending:
            request.wait()
        if side is not None:
            compute.wait_stream(side)
        self._mark("exchanged")

    def _contiguous_bucket(self, members: list[Tensor], world: int) -> Tensor | None:
        """The bucket's contiguous parameter buffer ([W * ceil(n / W), *shape], the
        members first, in order), created on first use: the parameters' values
        are copied in and each ``p.data`` becomes its slot. Recreated when a
        member no longer lives in its slot (its data was replaced). None for
        members that cannot share one buffer."""
        first = members[0]
        if any(p.shape != first.shape or p.dtype != first.dtype or p.device != first.device for p in members):
            return None
        # One buffer per bucket shape; a bucket whose members changed (a parameter
        # without a gradient this step, or replaced data) gets a new buffer.
        cache: dict[tuple, tuple[tuple[int, ...], Tensor]] = self.__dict__.setdefault("_flat_buckets", {})
        key = (tuple(first.shape), first.dtype, first.device)
        ids = tuple(id(p) for p in members)
        entry = cache.get(key)
        if entry is not None and entry[0] == ids and all(
            p.data_ptr() == entry[1][i].data_ptr() for i, p in enumerate(members)
        ):
            return entry[1]
        per_rank = -(-len(members) // world)
        flat = torch.zeros((world * per_rank, *first.shape), dtype=first.dtype, device=first.device)
        for slot, p in zip(flat, members):
            slot.copy_(p.detach())
            p.data = slot
        cache[key] = (ids, flat)
        return flat

    def _side_stream(self, device: torch.device) -> torch.cuda.Stream:
        streams: dict[torch.device, torch.cuda.Stream] = self.__dict__.setdefault("_side_streams", {})
        if device not in streams:
            streams[device] = torch.cuda.Stream(device)
        return streams[device]

    def apply_orthogonal_updates(
        self,
        group: ParameterGroup,
        parameters: list[Tensor],
        orthogonalized: list[Tensor],
        shapes: list[tuple[int, ...]],
    ) -> None:
        """p <- p * (1 - lr * wd) (when wd != 0) then p <- p - lr_adj * O (muon.py:458-476)."""
        lr = cast(LearningRate, group["lr"])
        wd = cast(LearningRate, group["weight_decay"])
        adjust = cast(LearningRateAdjustment, group["adjust_lr"])
        lr_adj = [self.adjusted_learning_rate(lr, shape, adjust) for shape in shapes]
        locals_ = [local_tensor(p) for p in parameters]
        outs = [o.reshape(p.shape) for o, p in zip(orthogonalized, locals_, strict=True)]
        if isinstance(lr, float) and isinstance(wd, float) and all(isinstance(v, float) for v in lr_adj):
            decay = None if wd == 0.0 else 1.0 - lr * wd
            classes: dict[tuple[torch.dtype, torch.dtype], list[int]] = {}
            for index, (p, o) in enumerate(zip(locals_, outs, strict=True)):
                classes.setdefault((p.dtype, o.dtype), []).append(index)
            for indices in classes.values():
                ops.muon_apply(
                    [locals_[i] for i in indices],
                    [outs[i].contiguous() for i in indices],
                    decay,
                    [cast(float, lr_adj[i]) for i in indices],
                )
            return
        # Tensor-valued learning rates stay on the device as torch scalars.
        for p, o, rate in zip(locals_, outs, lr_adj, strict=True):
            if not isinstance(wd, float) or wd != 0.0:
                p.mul_(1 - lr * wd)
            p.sub_(o * rate)

    # ------------------------------------------------------- AdamW / Lion
    def _host_step_values(self, steps: list[Tensor]) -> list[float]:
        """The post-increment values of the ``step`` tensors, known on the host.

        After the first step each value is the previous one plus one, kept in a
        host-side shadow keyed by the step tensor itself, so the group needs no
        device read-back; a step tensor the shadow has not seen (first step,
        ``load_state_dict``, a replaced state) is read back once, with one
        synchronisation for all of them. Changing ``state["step"]`` in place from
        outside the optimizer is not tracked.
        """
        shadow: dict[int, tuple[Tensor, float]] = self.__dict__.setdefault("_adamw_host_steps", {})
        values: list[float | None] = []
        unknown: list[int] = []
        for i, t in enumerate(steps):
            record = shadow.get(id(t))
            if record is not None and record[0] is t:
                values.append(record[1] + 1.0)
            else:
                values.append(None)
                unknown.append(i)
        if unknown:
            read = torch.stack([steps[i].reshape(()) for i in unknown]).cpu().tolist()
            for i, v in zip(unknown, read, strict=True):
                values[i] = float(v) + 1.0
        for t, v in zip(steps, values, strict=True):
            shadow[id(t)] = (t, cast(float, v))
        return cast(list[float], values)

    def step_adamw_group(self, group: ParameterGroup) -> None:
        """AdamW over the group's parameters (reference muon.py:516-553) as one
        multi-tensor kernel per dtype combination. Every ``step`` tensor is
        incremented on the device; its new value is known on the host without a
        read-back after the first step (``_host_step_values``; the reference reads
        each one back), and the bias corrections are formed on the host in double
        precision exactly as the reference forms them."""
        lr = float(cast(LearningRate, group["lr"]))
        wd = float(cast(LearningRate, group["weight_decay"]))
        beta1, beta2 = cast(tuple[float, float], group["betas"])
        epsilon = cast(float, group["epsilon"])
        entries = []
        for parameter in cast(list[Tensor], group["params"]):
            if parameter.grad is None:
                continue
            gradient = resolve_gradient(parameter)
            self.reject_sparse_or_complex_gradient(gradient)
            state = self.state[parameter]
            entries.append((
                local_tensor(parameter), gradient, local_tensor(cast(Tensor, state["exp_avg"])),
                local_tensor(cast(Tensor, state["exp_avg_sq"])), cast(Tensor, state["step"]),
            ))
        if not entries:
            return
        steps = [e[4] for e in entries]
        step_values = self._host_step_values(steps)
        torch._foreach_add_(steps, 1)
        decay = (1 - lr * wd) if wd != 0.0 else None
        groups: dict[tuple, list[int]] = {}
        for i, (p, g, m, v, _) in enumerate(entries):
            if m.dtype != v.dtype:
                raise TypeError("exp_avg and exp_avg_sq must share a dtype")
            groups.setdefault((p.dtype, g.dtype, m.dtype, p.device), []).append(i)
        for indices in groups.values():
            params, grads, avgs, avg_sqs, lr_bc1, inv_bc2 = [], [], [], [], [], []
            writeback: list[tuple[Tensor, Tensor]] = []
            for i in indices:
                p, g, m, v, _ = entries[i]
                step = float(step_values[i])
                lr_bc1.append(lr / (1 - beta1**step))
                # torch divides by a host scalar as a multiplication by its reciprocal,
                # formed in double precision and rounded to float
                inv_bc2.append(1.0 / sqrt(1 - beta2**step))
                params.append(_contiguous_in_place(p, writeback))
                avgs.append(_contiguous_in_place(m, writeback))
                avg_sqs.append(_contiguous_in_place(v, writeback))
                grads.append(g.contiguous())
            ops.adamw_step(params, grads, avgs, avg_sqs, lr_bc1, inv_bc2, beta1, beta2, epsilon, decay)
            for original, copy in writeback:
                original.copy_(copy)

    def step_lion_group(self, group: ParameterGroup) -> None:
        """Lion over the group's parameters (reference muon.py:555-583) as one
        multi-tensor kernel per dtype combination."""
        lr = float(cast(LearningRate, group["lr"]))
        wd = float(cast(LearningRate, group["weight_decay"]))
        beta1, beta2 = cast(tuple[float, float], group["betas"])
        decay = (1 - lr * wd) if wd != 0.0 else None
        groups: dict[tuple, list[tuple[Tensor, Tensor, Tensor]]] = {}
        for parameter in cast(list[Tensor], group["params"]):
            if parameter.grad is None:
                continue
            gradient = resolve_gradient(parameter)
            self.reject_sparse_or_complex_gradient(gradient)
            buffer = local_tensor(cast(Tensor, self.state[parameter]["momentum_buffer"]))
            p = local_tensor(parameter)
            groups.setdefault((p.dtype, gradient.dtype, buffer.dtype, p.device), []).append((p, gradient, buffer))
        for members in groups.values():
            params, grads, buffers = [], [], []
            writeback: list[tuple[Tensor, Tensor]] = []
            for p, g, b in members:
                params.append(_contiguous_in_place(p, writeback))
                buffers.append(_contiguous_in_place(b, writeback))
                grads.append(g.contiguous())
            ops.lion_step(params, grads, buffers, lr, beta1, beta2, decay)
            for original, copy in writeback:
                original.copy_(copy)


def _contiguous_in_place(tensor: Tensor, writeback: list[tuple[Tensor, Tensor]]) -> Tensor:
    """The tensor itself when contiguous; otherwise a contiguous copy, recorded so
    that the caller copies the updated values back."""
    if tensor.is_contiguous():
        return tensor
    copy = tensor.contiguous()
    writeback.append((tensor, copy))
    return copy
