"""Type aliases shared by the optimizer modules (mirrors optimizer_types.py of the reference).

The only Newton-Schulz kernel backend of this package is ``"b200"``: the
hand-written sm_100a tensor-core kernels. The reference's ``"torch"``,
``"cutlass"`` and ``"triton"`` names (optimizer_types.py:16 of the reference)
are accepted as well and select the same kernels, so that the reference's
default (``"torch"``) and its saved optimizer state keep working here.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass
from typing import Literal, Protocol

from torch import Tensor
from torch.distributed import ProcessGroup
from torch.distributed.tensor import DeviceMesh
from torch.optim.optimizer import ParamsT

type Coefficients = Sequence[Sequence[float]]
type DistributedMesh = DeviceMesh | ProcessGroup | None
type LearningRate = float | Tensor
type LearningRateAdjustment = Literal["spectral_norm", "rms_norm"] | None
type LossClosure = Callable[[], float]
type NewtonSchulzAlgorithm = Literal["gram_newton_schulz", "standard_newton_schulz"]
type NewtonSchulzBackend = Literal["b200", "torch", "cutlass", "triton"]
type OptimizerAlgorithm = Literal["muon", "dion3", "adamw", "lion"]
type ParameterGroup = dict[str, object]
type ParameterGroupInput = Mapping[str, object]
type OptimizerParameters = ParamsT

SUPPORTED_BACKENDS = frozenset({"b200"})
# The reference package's backend names: accepted, and run on the b200 kernels
# (kernels/interface.py), so that code and checkpoints written for the
# reference keep working.
REFERENCE_BACKEND_NAMES = frozenset({"torch", "cutlass", "triton"})


@dataclass(frozen=True)
class ParameterLayout:
    """How one parameter is laid out across the optimizer's process group."""

    process_group: ProcessGroup | None
    sharded_tensor_dimension: int | None
    batch_sharded: bool


class Orthogonalizer(Protocol):
    def __call__(self, matrix: Tensor, /) -> Tensor: ...
