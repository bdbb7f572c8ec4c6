"""The ``"b200"`` Newton-Schulz backend: sm_100a tcgen05 kernels behind the
reference's ``MatrixBackend`` protocol (kernels/protocols.py:36-61).

Every product runs in the native library; there is no fallback to torch or the
CPU. Inputs may be strided views (``.mT``) exactly as the reference passes them
(newton_schulz.py:91-93, :146-148). A reference installation can use this class
directly by returning it from ``select_matrix_backend("b200")``.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
from torch import Tensor

from gram_newton_schulz_ampere_b200 import ops


class B200Backend:
    """MatrixBackend + FusedNewtonSchulzBackend on B200 tensor cores."""

    name = "b200"

    def symmetric_matmul(self, left: Tensor, right: Tensor) -> Tensor:
        """``left @ right`` whose result the caller guarantees symmetric (TorchBackend :6-7)."""
        return ops.gemm(left, right, symmetric=True)

    def symmetric_batch_matrix_matrix_product(
        self,
        left: Tensor,
        right: Tensor,
        accumulator: Tensor,
        alpha: float = 1.0,
        beta: float = 1.0,
    ) -> Tensor:
        """``alpha * left @ right + beta * accumulator``, symmetric result (TorchBackend :9-23)."""
        return ops.gemm(left, right, accumulator, alpha=alpha, beta=beta, symmetric=True)

    def matmul(self, left: Tensor, right: Tensor) -> Tensor:
        """``left @ right`` (TorchBackend :25-26)."""
        return ops.gemm(left, right)

    def matmul_add(self, left: Tensor, right: Tensor, accumulator: Tensor, beta: float) -> Tensor:
        """``left @ right + beta * accumulator`` (TorchBackend :28-35)."""
        return ops.gemm(left, right, accumulator, alpha=1.0, beta=beta)

    def gram_newton_schulz(
        self,
        matrix: Tensor,
        coefficients: Sequence[Sequence[float]],
        reset_iterations: Sequence[int],
        epsilon: float,
    ) -> Tensor:
        return ops.newton_schulz_chain(matrix, coefficients, epsilon, gram=True, reset_iterations=reset_iterations)

    def standard_newton_schulz(
        self,
        matrix: Tensor,
        coefficients: Sequence[Sequence[float]],
        epsilon: float,
    ) -> Tensor:
        return ops.newton_schulz_chain(matrix, coefficients, epsilon, gram=False)

    # Pieces of a Gram chain whose long dimension is split across ranks
    # (distributed_orthogonalization.orthogonalize_long_axis_sharded).
    def frobenius_sumsq(self, matrix: Tensor) -> Tensor:
        return ops.frobenius_sumsq(matrix)

    def frobenius_scale(self, matrix: Tensor, sumsq: Tensor, epsilon: float) -> Tensor:
        return ops.frobenius_scale(matrix, sumsq, epsilon)

    def gram_partial(self, normalized: Tensor, tall: bool) -> Tensor:
        """This rank's share of the Gram matrix, fp32 (summed over ranks by the caller)."""
        if tall:
            return ops.gemm(normalized.mT, normalized, symmetric=True, out_dtype=torch.float32)
        return ops.gemm(normalized, normalized.mT, symmetric=True, out_dtype=torch.float32)

    def gram_iterations(
        self,
        gram: Tensor,
        coefficients: Sequence[Sequence[float]],
        it_begin: int,
        it_end: int,
    ) -> Tensor:
        """Q after Gram iterations [it_begin, it_end) between two restarts, from the summed Gram matrix."""
        return ops.gram_iterations(gram, coefficients, it_begin, it_end)

    def apply_polynomial(self, polynomial: Tensor, normalized: Tensor, tall: bool, out_dtype: torch.dtype) -> Tensor:
        """Q X (wide) or X Q (tall) for this rank's shard."""
        if tall:
            return ops.gemm(normalized, polynomial, out_dtype=out_dtype)
        return ops.gemm(polynomial, normalized, out_dtype=out_dtype)
