"""Backend protocols (mirrors kernels/protocols.py:36-61 of the reference).

``MatrixBackend`` is the four-method product interface the Newton-Schulz
algorithms are written against. ``FusedNewtonSchulzBackend`` is the optional
extension a backend may offer to run a whole orthogonalisation in one call;
``NewtonSchulz`` prefers it when present.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Protocol, runtime_checkable

from torch import Tensor


@runtime_checkable
class MatrixBackend(Protocol):
    def symmetric_matmul(self, left: Tensor, right: Tensor) -> Tensor: ...

    def symmetric_batch_matrix_matrix_product(
        self,
        left: Tensor,
        right: Tensor,
        accumulator: Tensor,
        alpha: float = 1.0,
        beta: float = 1.0,
    ) -> Tensor:
        """Return ``alpha * left @ right + beta * accumulator``.

        The caller guarantees that this result is symmetric.
        """
        ...

    def matmul(self, left: Tensor, right: Tensor) -> Tensor: ...

    def matmul_add(self, left: Tensor, right: Tensor, accumulator: Tensor, beta: float) -> Tensor: ...


@runtime_checkable
class FusedNewtonSchulzBackend(Protocol):
    def gram_newton_schulz(
        self,
        matrix: Tensor,
        coefficients: Sequence[Sequence[float]],
        reset_iterations: Sequence[int],
        epsilon: float,
    ) -> Tensor:
        """Normalised Gram Newton-Schulz of a [B, r, c] batch, returned in the input dtype."""
        ...

    def standard_newton_schulz(
        self,
        matrix: Tensor,
        coefficients: Sequence[Sequence[float]],
        epsilon: float,
    ) -> Tensor:
        """Normalised standard Newton-Schulz of a [B, r, c] batch, returned in the input dtype."""
        ...
