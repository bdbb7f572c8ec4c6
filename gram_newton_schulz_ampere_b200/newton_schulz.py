"""Newton-Schulz orthogonalisers (mirrors newton_schulz.py of the reference).

``GramNewtonSchulz(...)`` and ``StandardNewtonSchulz(...)`` keep the reference's
constructor signatures (newton_schulz.py:322-355) and call semantics
(:282-319): CUDA input required, any leading batch dims flattened, Gram
iteration for non-square inputs when enabled, standard iteration otherwise,
result returned in the input dtype and shape.

With the ``"b200"`` backend each call is ONE native chain
(``gns_gram_newton_schulz`` / ``gns_standard_newton_schulz``): normalisation,
all products and the output cast run back to back on the caller's stream.
``build_*_operation`` also accepts any other ``MatrixBackend`` and then
composes the reference's sequence of products from its four primitives.
``ns_compile`` is accepted for signature compatibility; as for the
reference's non-torch backends (newton_schulz.py:241) nothing is compiled.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch
from torch import Tensor

from gram_newton_schulz_ampere_b200 import ops
from gram_newton_schulz_ampere_b200.coefficients import polar_express_coefficients
from gram_newton_schulz_ampere_b200.kernels.interface import select_matrix_backend
from gram_newton_schulz_ampere_b200.kernels.protocols import FusedNewtonSchulzBackend, MatrixBackend
from gram_newton_schulz_ampere_b200.optimizer_types import NewtonSchulzBackend


def _freeze(coefficients: Sequence[Sequence[float]]) -> tuple[tuple[float, ...], ...]:
    return tuple(tuple(float(v) for v in triple) for triple in coefficients)


def _normalized(matrix: Tensor, epsilon: float) -> Tensor:
    return ops.frobenius_normalize(matrix, epsilon)


def build_standard_newton_schulz_operation(
    backend: MatrixBackend,
    coefficients: Sequence[Sequence[float]],
    epsilon: float,
    compile_operation: bool = False,
    dynamic_compile: bool = False,
    normalize_input: bool = True,
) -> Callable[[Tensor], Tensor]:
    """Standard Newton-Schulz (reference newton_schulz.py:66-121)."""
    coeffs = _freeze(coefficients)
    if normalize_input and isinstance(backend, FusedNewtonSchulzBackend):

        def fused_standard(matrix: Tensor) -> Tensor:
            return backend.standard_newton_schulz(matrix, coeffs, epsilon)

        return fused_standard

    def standard_newton_schulz(matrix: Tensor) -> Tensor:
        tall = matrix.size(-2) > matrix.size(-1)
        if normalize_input:
            matrix = _normalized(matrix, epsilon)
        for a, b, c in coeffs:
            gram = backend.symmetric_matmul(matrix.mT, matrix) if tall else backend.symmetric_matmul(matrix, matrix.mT)
            poly = backend.symmetric_batch_matrix_matrix_product(gram, gram, accumulator=gram, alpha=c, beta=b)
            if tall:
                matrix = backend.matmul_add(matrix, poly, accumulator=matrix, beta=a)
            else:
                matrix = backend.matmul_add(poly, matrix, accumulator=matrix, beta=a)
        return matrix

    return standard_newton_schulz


def build_gram_newton_schulz_operation(
    backend: MatrixBackend,
    coefficients: Sequence[Sequence[float]],
    reset_iterations: Sequence[int],
    epsilon: float,
    compile_operation: bool = False,
    dynamic_compile: bool = False,
    normalize_input: bool = True,
) -> Callable[[Tensor], Tensor]:
    """Gram Newton-Schulz with restarts (reference newton_schulz.py:124-223)."""
    coeffs = _freeze(coefficients)
    resets = tuple(int(i) for i in reset_iterations)
    if normalize_input and isinstance(backend, FusedNewtonSchulzBackend):

        def fused_gram(matrix: Tensor) -> Tensor:
            return backend.gram_newton_schulz(matrix, coeffs, resets, epsilon)

        return fused_gram

    reset_set = frozenset(resets)

    def gram_newton_schulz(matrix: Tensor) -> Tensor:
        tall = matrix.size(-2) > matrix.size(-1)
        if normalize_input:
            matrix = _normalized(matrix, epsilon)

        def gram_of(x: Tensor) -> Tensor:
            return backend.symmetric_matmul(x.mT, x) if tall else backend.symmetric_matmul(x, x.mT)

        gram = gram_of(matrix)
        eye = torch.eye(gram.shape[-1], device=gram.device, dtype=gram.dtype).expand_as(gram)
        acc: Tensor | None = None
        last = len(coeffs) - 1
        for it, (a, b, c) in enumerate(coeffs):
            if it != 0 and it in reset_set:
                if acc is None:
                    raise RuntimeError("Gram Newton--Schulz reset has no accumulated update")
                matrix = backend.matmul(matrix, acc) if tall else backend.matmul(acc, matrix)
                gram = gram_of(matrix)
                acc = None
            poly = backend.symmetric_batch_matrix_matrix_product(gram, gram, accumulator=gram, alpha=c, beta=b)
            if acc is None:
                acc = poly.add(eye, alpha=a)
            else:
                acc = backend.symmetric_batch_matrix_matrix_product(acc, poly, accumulator=acc, beta=a)
            if it < last and (it + 1) not in reset_set:
                gp = backend.symmetric_batch_matrix_matrix_product(gram, poly, accumulator=gram, beta=a)
                gram = backend.symmetric_batch_matrix_matrix_product(poly, gp, accumulator=gp, beta=a)
        if acc is None:
            raise RuntimeError("Gram Newton--Schulz requires coefficients")
        return backend.matmul(matrix, acc) if tall else backend.matmul(acc, matrix)

    return gram_newton_schulz


class NewtonSchulz:
    """Orthogonaliser: ``NewtonSchulz(...)(X)`` returns the polar factor estimate of X."""

    def __init__(
        self,
        eps: float = 1e-9,
        coeff: Sequence[Sequence[float]] | None = None,
        use_gram: bool = False,
        gns_reset_iters: Sequence[int] | None = None,
        backend: NewtonSchulzBackend = "b200",
        compile: bool = True,
    ) -> None:
        self.epsilon = eps
        self.coefficients = _freeze(coeff if coeff is not None else polar_express_coefficients())
        self.backend = select_matrix_backend(backend)
        self.gram = use_gram
        self.reset_iterations = tuple(gns_reset_iters or ())
        # Nothing is compiled for the native backend (the reference compiles only "torch").
        self.compile_operation = False
        self.standard_operation = build_standard_newton_schulz_operation(
            self.backend, self.coefficients, self.epsilon, normalize_input=True
        )
        self.gram_operation = build_gram_newton_schulz_operation(
            self.backend, self.coefficients, self.reset_iterations, self.epsilon, normalize_input=True
        )
        self.dynamic_standard_operation = self.standard_operation
        self.dynamic_gram_operation = self.gram_operation

    def __call__(self, matrix: Tensor) -> Tensor:
        if not isinstance(matrix, Tensor) or not matrix.is_floating_point():
            raise TypeError("Newton--Schulz expects a floating-point tensor")
        if not matrix.is_cuda:
            raise ValueError("Newton--Schulz requires a CUDA tensor")
        if matrix.ndim < 2:
            raise ValueError("Newton--Schulz expects a matrix or a batch of matrices")
        original_shape = matrix.shape
        original_dtype = matrix.dtype
        batched = matrix.reshape(-1, matrix.shape[-2], matrix.shape[-1])
        use_gram = self.gram and batched.shape[-2] != batched.shape[-1]
        operation = self.gram_operation if use_gram else self.standard_operation
        if torch.compiler.is_compiling():
            # A region torch.compile traces records the native call as a custom op.
            # The opt-in status check synchronises the host, so it is not made
            # here; call ops.check_device_status() after the compiled region.
            return operation(batched).to(original_dtype).reshape(original_shape)
        with ops.status_checked():
            return operation(batched).to(original_dtype).reshape(original_shape)


class GramNewtonSchulz(NewtonSchulz):
    """Gram Newton-Schulz (reference newton_schulz.py:322-338), default reset at iteration 2."""

    def __init__(
        self,
        ns_epsilon: float = 1e-7,
        ns_backend: NewtonSchulzBackend = "b200",
        ns_coefficients: Sequence[Sequence[float]] | None = None,
        gram_newton_schulz_reset_iterations: Sequence[int] = (2,),
        ns_compile: bool = True,
    ) -> None:
        super().__init__(
            eps=ns_epsilon,
            coeff=ns_coefficients,
            use_gram=True,
            gns_reset_iters=gram_newton_schulz_reset_iterations,
            backend=ns_backend,
            compile=ns_compile,
        )


class StandardNewtonSchulz(NewtonSchulz):
    """Standard Newton-Schulz (reference newton_schulz.py:341-355)."""

    def __init__(
        self,
        ns_epsilon: float = 1e-7,
        ns_backend: NewtonSchulzBackend = "b200",
        ns_coefficients: Sequence[Sequence[float]] | None = None,
        ns_compile: bool = True,
    ) -> None:
        super().__init__(
            eps=ns_epsilon,
            coeff=ns_coefficients,
            use_gram=False,
            backend=ns_backend,
            compile=ns_compile,
        )
