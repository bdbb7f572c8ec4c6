"""Distributed orchestration of the orthogonalisation step.

Mirrors distributed_orthogonalization.py of the reference (:15-364) in behaviour:

* parameters are bucketed by (local shape, global matrix shape, update dtype,
  device, shard dimension, batch-sharded) in first-seen order (:160-185);
* replicated parameters: each rank orthogonalises a contiguous ``ceil(n/W)``
  slice of every bucket (zero-padded) and the results are all-gathered (:231-262),
  so every rank ends with bit-identical outputs;
* one active DTensor shard dimension over a matrix axis: matrices are assembled
  on owner ranks with an all-to-all, orthogonalised, and sent back (:278-349);
* a shard dimension over a batch axis: purely local (:198-199).

The functions are device-agnostic (the orthogonaliser decides where the math
runs); the optimizers pass the native B200 orthogonaliser and NCCL groups.
Process groups without all-to-all support (gloo) exchange through an
all-gather instead, which keeps the CPU multi-rank tests meaningful.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
from torch import Tensor, distributed
from torch.distributed import ProcessGroup
from torch.distributed.tensor import DeviceMesh, DTensor, Shard

from gram_newton_schulz_ampere_b200.optimizer_types import (
    DistributedMesh,
    Orthogonalizer,
    ParameterLayout,
)


def local_tensor(tensor: Tensor) -> Tensor:
    """The rank-local shard of a DTensor, or the tensor itself."""
    return tensor.to_local() if isinstance(tensor, DTensor) else tensor


def resolve_gradient(parameter: Tensor) -> Tensor:
    """Local gradient laid out like the parameter (reference :21-38)."""
    gradient = parameter.grad
    if gradient is None:
        raise RuntimeError("Cannot resolve a missing gradient")
    if not isinstance(parameter, DTensor):
        if isinstance(gradient, DTensor):
            raise TypeError("A regular Tensor parameter cannot use a DTensor gradient")
        return gradient
    if not isinstance(gradient, DTensor):
        raise TypeError("A DTensor parameter requires a DTensor gradient")
    if gradient.device_mesh != parameter.device_mesh:
        raise ValueError("Parameter and gradient must use the same DeviceMesh")
    if gradient.placements != parameter.placements:
        gradient = gradient.redistribute(device_mesh=parameter.device_mesh, placements=parameter.placements)
    return gradient.to_local()


def configured_process_group(distributed_mesh: DistributedMesh) -> ProcessGroup | None:
    """The optimizer's process group: a ProcessGroup, a 1-D mesh of size > 1, or None (reference :41-53)."""
    if isinstance(distributed_mesh, ProcessGroup):
        return distributed_mesh
    if isinstance(distributed_mesh, DeviceMesh):
        if distributed_mesh.ndim != 1:
            raise ValueError("Pass a 1D optimizer submesh, not a multidimensional DeviceMesh")
        return distributed_mesh.get_group() if distributed_mesh.size() > 1 else None
    return None


def parameter_layout(parameter: Tensor, distributed_mesh: DistributedMesh, flatten: bool) -> ParameterLayout:
    """Classifies a parameter's placement (reference :56-94)."""
    group = configured_process_group(distributed_mesh)
    if not isinstance(parameter, DTensor):
        return ParameterLayout(group, None, False)
    active: list[tuple[int, Shard]] = []
    for mesh_dim, placement in enumerate(parameter.placements):
        if placement.is_partial():
            raise NotImplementedError("Partial DTensor parameters are not supported")
        if isinstance(placement, Shard) and parameter.device_mesh.size(mesh_dim) > 1:
            active.append((mesh_dim, placement))
    if len(active) > 1:
        raise NotImplementedError(
            "Muon supports one active DTensor shard dimension; combined FSDP2 and TP is not supported"
        )
    if not active:
        return ParameterLayout(group, None, False)
    mesh_dim, shard = active[0]
    shard_group = parameter.device_mesh.get_group(mesh_dim)
    if group is not None and group != shard_group:
        raise ValueError("The optimizer process group must match the parameter shard mesh axis")
    shard_dim = shard.dim if shard.dim >= 0 else shard.dim + parameter.ndim
    if flatten and shard_dim != 0:
        raise NotImplementedError("Flattened tensors can only be sharded on output dimension 0")
    batch_sharded = not flatten and shard_dim not in (parameter.ndim - 2, parameter.ndim - 1)
    return ParameterLayout(shard_group, shard_dim, batch_sharded)


def validate_gradient_participation(
    parameters: Sequence[Tensor],
    distributed_mesh: DistributedMesh,
    flatten: bool,
) -> None:
    """Raises unless every rank has gradients for the same parameters (reference :97-140).

    One MIN all-reduce over [present, -present] per group replaces the
    reference's separate MIN and MAX reductions: equal participation holds
    exactly when min(present) == -min(-present) == max(present).
    """
    groups: dict[tuple[ProcessGroup, torch.device], list[int]] = {}
    for parameter in parameters:
        layout = parameter_layout(parameter, distributed_mesh, flatten)
        if layout.process_group is None:
            continue
        key = (layout.process_group, local_tensor(parameter).device)
        groups.setdefault(key, []).append(1 if parameter.grad is not None else 0)
    for (group, device), present in groups.items():
        if distributed.get_world_size(group) == 1:
            continue
        flags = torch.tensor(present + [-p for p in present], dtype=torch.int32, device=device)
        distributed.all_reduce(flags, op=distributed.ReduceOp.MIN, group=group)
        n = len(present)
        if not torch.equal(flags[:n], -flags[n:]):
            raise RuntimeError(
                "Distributed orthogonal optimizers require the same gradient participation on every rank"
            )


def orthogonalize_parameter_updates(
    parameters: Sequence[Tensor],
    local_updates: Sequence[Tensor],
    global_matrix_shapes: Sequence[tuple[int, ...]],
    orthogonalizer: Orthogonalizer,
    distributed_mesh: DistributedMesh,
    flatten: bool,
) -> list[Tensor]:
    """Orthogonalises every update, choosing per bucket how work is spread over ranks."""
    if not (len(parameters) == len(local_updates) == len(global_matrix_shapes)):
        raise ValueError("Parameters, updates, and global shapes must have equal lengths")
    if not parameters:
        return []
    buckets: dict[tuple, list[int]] = {}
    layouts = []
    for index, parameter in enumerate(parameters):
        layout = parameter_layout(parameter, distributed_mesh, flatten)
        layouts.append(layout)
        update = local_updates[index]
        key = (
            tuple(parameter.shape),
            tuple(global_matrix_shapes[index]),
            update.dtype,
            update.device,
            layout.sharded_tensor_dimension,
            layout.batch_sharded,
        )
        buckets.setdefault(key, []).append(index)

    outputs: list[Tensor | None] = [None] * len(parameters)
    pending: list[tuple[list[int], PendingGather]] = []
    for indices in buckets.values():
        layout = layouts[indices[0]]
        if any(layouts[i] != layout for i in indices):
            raise ValueError("One shape bucket cannot span different optimizer mesh layouts")
        matrices = [local_updates[i] for i in indices]
        if layout.batch_sharded:
            results = orthogonalize_local_matrices(matrices, orthogonalizer)
        elif layout.sharded_tensor_dimension is not None:
            shard_dim = 0 if flatten else layout.sharded_tensor_dimension
            global_shape = global_matrix_shapes[indices[0]]
            if shards_long_axis(global_shape, shard_dim, matrices[0].ndim) and supports_partial_gram(orthogonalizer):
                results = orthogonalize_long_axis_sharded(matrices, global_shape, orthogonalizer, layout.process_group)
            else:
                results = orthogonalize_sharded_matrices(
                    matrices, global_shape, shard_dim, orthogonalizer, layout.process_group
                )
        else:
            gathered = orthogonalize_replicated_matrices(
                matrices, orthogonalizer, layout.process_group, deferred=True
            )
            if isinstance(gathered, PendingGather):
                # The all-gather runs while the next buckets are orthogonalised.
                pending.append((indices, gathered))
                continue
            results = gathered
        for slot, index in enumerate(indices):
            outputs[index] = results[slot]
    for indices, gathered in pending:
        for slot, result in enumerate(gathered.results()):
            outputs[indices[slot]] = result
    return [out for out in outputs if out is not None]


def stack_matrices(matrices: Sequence[Tensor]) -> Tensor:
    """``torch.stack(matrices)``, returned as a view without copying when the
    matrices are already consecutive equal-shape slices of one buffer (as the
    fused momentum kernel's outputs are)."""
    first = matrices[0]
    count, numel, size = len(matrices), first.numel(), first.element_size()
    storage = first.untyped_storage()
    consecutive = first.is_contiguous() and all(
        m.shape == first.shape
        and m.dtype == first.dtype
        and m.is_contiguous()
        and m.untyped_storage().data_ptr() == storage.data_ptr()
        and m.data_ptr() == first.data_ptr() + i * numel * size
        for i, m in enumerate(matrices)
    )
    if consecutive and (first.storage_offset() + count * numel) * size <= storage.nbytes():
        return torch.as_strided(first, (count, *first.shape), (numel, *first.stride()))
    return torch.stack(list(matrices))


def orthogonalize_local_matrices(matrices: Sequence[Tensor], orthogonalizer: Orthogonalizer) -> list[Tensor]:
    """One batched orthogonaliser call over a bucket (reference :223-228)."""
    stacked = orthogonalizer(stack_matrices(matrices))
    return list(stacked.unbind(0))


class PendingGather:
    """An all-gather in flight; ``results()`` waits for it (the caller's stream
    then orders after it) and returns the bucket's matrices in order."""

    def __init__(self, work: distributed.Work, gathered: Tensor, count: int) -> None:
        self.work = work
        self.gathered = gathered
        self.count = count

    def results(self) -> list[Tensor]:
        self.work.wait()
        return list(self.gathered[: self.count].unbind(0))


def orthogonalize_replicated_matrices(
    matrices: Sequence[Tensor],
    orthogonalizer: Orthogonalizer,
    process_group: ProcessGroup | None,
    deferred: bool = False,
) -> list[Tensor] | PendingGather:
    """Round-robin ownership + all-gather (reference :231-262).

    Rank r orthogonalises matrices [r*k, (r+1)*k) of the zero-padded bucket,
    k = ceil(n / W); the all-gather returns every result to every rank in the
    same order, so all ranks hold identical outputs. With ``deferred`` the
    all-gather is issued asynchronously and a PendingGather is returned, so the
    caller can orthogonalise the next bucket while it runs (every rank issues
    the same collectives in the same order either way).
    """
    if process_group is None or distributed.get_world_size(process_group) == 1:
        return orthogonalize_local_matrices(matrices, orthogonalizer)
    world = distributed.get_world_size(process_group)
    rank = distributed.get_rank(process_group)
    count = len(matrices)
    per_rank = -(-count // world)
    start = rank * per_rank
    mine = [matrices[i] if i < count else torch.zeros_like(matrices[0]) for i in range(start, start + per_rank)]
    local = orthogonalizer(stack_matrices(mine)).contiguous()
    gathered = torch.empty((world * per_rank, *local.shape[1:]), dtype=local.dtype, device=local.device)
    if distributed.get_backend(process_group) == "gloo":
        work = distributed.all_gather(list(gathered.chunk(world)), local, group=process_group, async_op=deferred)
    else:
        work = distributed.all_gather_into_tensor(gathered, local, group=process_group, async_op=deferred)
    if deferred:
        return PendingGather(work, gathered, count)
    return list(gathered[:count].unbind(0))


def round_robin_owners(count: int, world: int) -> list[int]:
    """Owner rank of each matrix of a replicated bucket: rank r owns positions
    [r*k, (r+1)*k), k = ceil(count / W) (reference :241-252)."""
    per_rank = -(-count // world)
    return [position // per_rank for position in range(count)]


def send_owned_tensors(
    tensors: Sequence[Tensor], owners: Sequence[int], process_group: ProcessGroup
) -> list[distributed.Work]:
    """Sends each tensor from its owner rank to every other rank, in place.

    Every rank passes the same tensors (its own copies) and owners; the owner's
    values overwrite the others' copies, so all ranks end bit-identical. The
    point-to-point operations of the whole list are issued as one group and
    returned unfinished; they read and write the tensors directly, so nothing is
    staged or copied.
    """
    rank = distributed.get_rank(process_group)
    world = distributed.get_world_size(process_group)
    operations = []
    for tensor, owner in zip(tensors, owners, strict=True):
        if owner == rank:
            for peer in range(world):
                if peer != rank:
                    operations.append(
                        distributed.P2POp(distributed.isend, tensor, group=process_group, group_peer=peer)
                    )
        else:
            operations.append(distributed.P2POp(distributed.irecv, tensor, group=process_group, group_peer=owner))
    return distributed.batch_isend_irecv(operations) if operations else []


class PendingOwnedGather:
    """A bucket's all-gather of owner-updated tensors in flight; ``finish()``
    makes the current stream wait for it and copies every tensor this rank does
    not own out of the gathered buffer into place, on that stream."""

    def __init__(self, work: distributed.Work | None, gathered: Tensor, targets: list[tuple[Tensor, int]]) -> None:
        self.work = work
        self.gathered = gathered
        self.targets = targets

    def finish(self) -> None:
        if self.work is not None:
            self.work.wait()
        if self.targets:
            if self.gathered.is_cuda:
                self.gathered.record_stream(torch.cuda.current_stream(self.gathered.device))
            torch._foreach_copy_([t for t, _ in self.targets], [self.gathered[slot] for _, slot in self.targets])


def gather_owned_tensors(tensors: Sequence[Tensor], owners: Sequence[int], process_group: ProcessGroup) -> PendingOwnedGather:
    """All-gathers equal-shape tensors from their round-robin owners into every
    rank's copies: the owner's values land in every rank's tensor, so all ranks
    end bit-identical.

    The owned tensors are packed into this rank's slot of one buffer of
    ``W * ceil(n / W)`` tensors (zero-padded at the end), which is all-gathered
    in place asynchronously; the returned object copies the other ranks' tensors
    into place when finished.
    """
    rank = distributed.get_rank(process_group)
    world = distributed.get_world_size(process_group)
    count = len(tensors)
    per_rank = -(-count // world)
    first = tensors[0]
    gathered = torch.empty((world * per_rank, *first.shape), dtype=first.dtype, device=first.device)
    mine = gathered[rank * per_rank:(rank + 1) * per_rank]
    own = [(t, i - rank * per_rank) for i, t in enumerate(tensors) if owners[i] == rank]
    if own:
        torch._foreach_copy_([mine[slot] for _, slot in own], [t for t, _ in own])
    if len(own) < per_rank:
        mine[len(own):].zero_()
    if distributed.get_backend(process_group) == "gloo":
        work = distributed.all_gather(list(gathered.chunk(world)), mine.clone(), group=process_group, async_op=True)
    else:
        work = distributed.all_gather_into_tensor(gathered, mine, group=process_group, async_op=True)
    targets = [(t, i) for i, t in enumerate(tensors) if owners[i] != rank]
    return PendingOwnedGather(work, gathered, targets)


def exchange_equal_chunks(input_chunks: Sequence[Tensor], process_group: ProcessGroup) -> list[Tensor]:
    """All-to-all of W equal chunks: output[i] is what rank i sent to this rank (reference :265-275)."""
    world = distributed.get_world_size(process_group)
    if len(input_chunks) != world:
        raise ValueError("exchange needs one chunk per rank")
    chunks = [c.contiguous() for c in input_chunks]
    if distributed.get_backend(process_group) != "gloo":
        outputs = [torch.empty_like(c) for c in chunks]
        distributed.all_to_all(outputs, chunks, group=process_group)
        return outputs
    # gloo has no all-to-all: gather everything and keep the pieces addressed to us.
    rank = distributed.get_rank(process_group)
    stacked = torch.stack(chunks)
    everything = [torch.empty_like(stacked) for _ in range(world)]
    distributed.all_gather(everything, stacked, group=process_group)
    return [everything[src][rank] for src in range(world)]


PARTIAL_GRAM_PIECES = ("frobenius_sumsq", "frobenius_scale", "gram_partial", "gram_iterations", "apply_polynomial")


def supports_partial_gram(orthogonalizer: Orthogonalizer) -> bool:
    """True for a Gram Newton-Schulz orthogonaliser whose backend offers the sharded-chain pieces."""
    backend = getattr(orthogonalizer, "backend", None)
    return bool(getattr(orthogonalizer, "gram", False)) and all(hasattr(backend, n) for n in PARTIAL_GRAM_PIECES)


def shards_long_axis(global_shape: tuple[int, ...], shard_dim: int, local_ndim: int) -> bool:
    """True when the shard dimension is the longer matrix axis of a non-square matrix
    (columns of a wide matrix, rows of a tall one): then the m x m Gram matrix is a
    sum of per-rank partial Grams."""
    rows, cols = global_shape[-2], global_shape[-1]
    if rows == cols:
        return False
    axis = shard_dim - len(global_shape) if shard_dim >= 0 else shard_dim
    return (axis == -1 and rows < cols) or (axis == -2 and rows > cols)


def orthogonalize_long_axis_sharded(
    matrices: Sequence[Tensor],
    global_matrix_shape: tuple[int, ...],
    orthogonalizer: Orthogonalizer,
    process_group: ProcessGroup | None,
) -> list[Tensor]:
    """Gram Newton-Schulz on matrices split along their long axis, without assembling them.

    With X = [X_1 .. X_W] split along its long axis, ||X||^2 = sum ||X_i||^2 and
    G = sum X_i X_i^T, so each rank keeps its shard and the ranks exchange only
    a scalar per matrix and the m x m Gram matrix (fp32 all-reduces). The Gram
    iterations (newton_schulz.py:177-212) run redundantly on every rank; a restart
    (X <- Q X, :164-175) is local to each shard followed by one more Gram
    all-reduce; the output shard is Q X_i. The reference instead gathers whole
    matrices on owner ranks (:278-349), which leaves the other ranks idle when a
    bucket holds one matrix.
    """
    if process_group is None:
        raise ValueError("A sharded DTensor update requires a process group")
    backend = getattr(orthogonalizer, "backend")
    coefficients = orthogonalizer.coefficients  # type: ignore[attr-defined]
    resets = tuple(orthogonalizer.reset_iterations)  # type: ignore[attr-defined]
    epsilon = orthogonalizer.epsilon  # type: ignore[attr-defined]
    if not coefficients:
        raise RuntimeError("Gram Newton--Schulz requires coefficients")
    tall = global_matrix_shape[-2] > global_matrix_shape[-1]
    stacked = torch.stack(list(matrices))
    x = stacked.reshape(-1, stacked.shape[-2], stacked.shape[-1])
    sumsq = backend.frobenius_sumsq(x)
    distributed.all_reduce(sumsq, op=distributed.ReduceOp.SUM, group=process_group)
    normalized = backend.frobenius_scale(x, sumsq, epsilon)
    gram = backend.gram_partial(normalized, tall).contiguous()
    distributed.all_reduce(gram, op=distributed.ReduceOp.SUM, group=process_group)
    n = len(coefficients)
    boundaries = sorted({int(i) for i in resets if 0 < int(i) < n}) + [n]
    begin = 0
    polynomial = None
    for end in boundaries:
        polynomial = backend.gram_iterations(gram, coefficients, begin, end)
        if end < n:
            normalized = backend.apply_polynomial(polynomial, normalized, tall, normalized.dtype)
            gram = backend.gram_partial(normalized, tall).contiguous()
            distributed.all_reduce(gram, op=distributed.ReduceOp.SUM, group=process_group)
        begin = end
    out = backend.apply_polynomial(polynomial, normalized, tall, stacked.dtype)
    return list(out.reshape(stacked.shape).unbind(0))


def pad_matrix_dimension(matrix: Tensor, tensor_dimension: int, padded_size: int) -> Tensor:
    """Zero-pads one dimension up to `padded_size` (reference :352-364)."""
    missing = padded_size - matrix.shape[tensor_dimension]
    if missing <= 0:
        return matrix
    shape = list(matrix.shape)
    shape[tensor_dimension] = missing
    return torch.cat((matrix, matrix.new_zeros(shape)), dim=tensor_dimension)


def orthogonalize_sharded_matrices(
    matrices: Sequence[Tensor],
    global_matrix_shape: tuple[int, ...],
    sharded_tensor_dimension: int,
    orthogonalizer: Orthogonalizer,
    process_group: ProcessGroup | None,
) -> list[Tensor]:
    """Owner scheme for matrices sharded along a matrix axis (reference :278-349).

    Every matrix is padded to W equal shards; an all-to-all delivers all shards
    of matrices [r*k, (r+1)*k) to rank r, which orthogonalises them whole; a
    second all-to-all returns each rank's shard of every result.
    """
    if process_group is None:
        raise ValueError("A sharded DTensor update requires a process group")
    world = distributed.get_world_size(process_group)
    count = len(matrices)
    per_rank = -(-count // world)
    ndim = matrices[0].ndim
    comm_dim = sharded_tensor_dimension - ndim  # negative index into a matrix
    global_size = global_matrix_shape[sharded_tensor_dimension]
    shard_size = -(-global_size // world)
    local_size = matrices[0].shape[sharded_tensor_dimension]
    if local_size > shard_size:
        raise RuntimeError("The local shard exceeds the expected contiguous DTensor shard size")
    padded = [pad_matrix_dimension(m, sharded_tensor_dimension, shard_size) for m in matrices]
    padded += [torch.zeros_like(padded[0]) for _ in range(world * per_rank - count)]
    outgoing = list(torch.stack(padded).unflatten(0, (world, per_rank)).unbind(0))
    incoming = exchange_equal_chunks(outgoing, process_group)
    full = torch.cat(incoming, dim=comm_dim).narrow(comm_dim, 0, global_size)
    result = orthogonalizer(full)
    result = pad_matrix_dimension(result, result.ndim + comm_dim, shard_size * world)
    back = exchange_equal_chunks(list(torch.tensor_split(result, world, dim=comm_dim)), process_group)
    returned = torch.stack(back).narrow(comm_dim, 0, local_size).flatten(0, 1)[:count]
    return list(returned.contiguous().unbind(0))
