"""CPU oracle for Gram / standard Newton-Schulz (numpy). TEST INFRASTRUCTURE ONLY.

This module is a restatement of the reference's torch backend numerics, used as
the checker by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg. The product never imports it.

Reference algorithm (afrenkai/Gram-Newton-Schulz-Ampere):
- coefficients:         gram_newton_schulz_ampere/coefficients.py:1-17
- standard NS:          gram_newton_schulz_ampere/newton_schulz.py:66-121
- Gram NS + reset:      gram_newton_schulz_ampere/newton_schulz.py:124-223
- dispatch / cast:      gram_newton_schulz_ampere/newton_schulz.py:283-319
- torch products:       gram_newton_schulz_ampere/kernels/torch_ns.py:5-35

Numerics restated: the input is normalised in fp32 and cast to fp16; every
product is an fp16 x fp16 GEMM with fp32 accumulation whose result
``beta * C + alpha * (A @ B)`` is rounded to fp16 (cuBLAS / torch.baddbmm
semantics); ``P + a I`` is an fp16 element-wise add; the final result is cast
from fp16 to the caller's dtype. Pinned against outputs of the reference
itself by ``tests/golden/make_golden.py`` (fixtures in ``tests/golden/``).
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np

_UNMODIFIED = (
    (8.28721201814563, -23.595886519098837, 17.300387312530933),
    (4.107059111542203, -2.9478499167379106, 0.5448431082926601),
    (3.9486908534822946, -2.908902115962949, 0.5518191394370137),
    (3.3184196573706015, -2.488488024314874, 0.51004894012372),
    (2.300652019954817, -1.6689039845747493, 0.4188073119525673),
)


def polar_express_coefficients() -> tuple[tuple[float, float, float], ...]:
    """The five (a, b, c) triples divided by (1.05, 1.05**3, 1.05**5) (coefficients.py:1-17)."""
    s = 1.05
    return tuple((a / s, b / s**3, c / s**5) for a, b, c in _UNMODIFIED)


def to_f16(x: np.ndarray) -> np.ndarray:
    """Rounds to fp16 and returns fp32 storage of the rounded values."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def normalize(matrix: np.ndarray, epsilon: float) -> np.ndarray:
    """fp16(X / (||X||_F + eps)) with the norm and division in fp32 (newton_schulz.py:141-144)."""
    x = np.asarray(matrix, dtype=np.float32)
    norm = np.sqrt(np.sum(np.square(x.astype(np.float64)), axis=(-2, -1), keepdims=True)).astype(np.float32)
    return to_f16(x / (norm + np.float32(epsilon)))


def baddbmm(acc: np.ndarray | None, a: np.ndarray, b: np.ndarray, alpha: float = 1.0, beta: float = 0.0) -> np.ndarray:
    """fp16(beta * acc + alpha * (a @ b)), fp32 accumulation (torch_ns.py:9-35)."""
    prod = np.matmul(a.astype(np.float32), b.astype(np.float32))
    out = np.float32(alpha) * prod
    if acc is not None and beta != 0.0:
        out = out + np.float32(beta) * acc.astype(np.float32)
    return to_f16(out)


def _mT(x: np.ndarray) -> np.ndarray:
    return np.swapaxes(x, -1, -2)


def gram_newton_schulz(
    matrix: np.ndarray,
    coefficients: Sequence[Sequence[float]] | None = None,
    reset_iterations: Sequence[int] = (2,),
    epsilon: float = 1e-7,
    identity_alpha_f16: bool = False,
) -> np.ndarray:
    """Gram Newton-Schulz on a [B, r, c] batch; returns fp16 values (as fp32 storage).

    Line-by-line restatement of build_gram_newton_schulz_operation's inner function
    (newton_schulz.py:139-217) with the torch backend. ``P.add(I, alpha=a)``
    (newton_schulz.py:185-188) is evaluated as fp16(P + a) with ``a`` in fp32, as
    torch's CUDA add kernel does; ``identity_alpha_f16=True`` instead rounds ``a``
    to fp16 first, which is what torch's CPU add kernel does (used only to pin this
    oracle bit-for-bit against the reference run on CPU).
    """
    coeffs = coefficients if coefficients is not None else polar_express_coefficients()
    resets = frozenset(int(i) for i in reset_iterations)
    x = np.asarray(matrix, dtype=np.float32)
    tall = x.shape[-2] > x.shape[-1]
    x = normalize(x, epsilon)
    gram = baddbmm(None, _mT(x), x) if tall else baddbmm(None, x, _mT(x))
    eye = np.broadcast_to(np.eye(gram.shape[-1], dtype=np.float32), gram.shape)
    acc = None
    for it, (a, b, c) in enumerate(coeffs):
        if it != 0 and it in resets:
            if acc is None:
                raise RuntimeError("Gram Newton--Schulz reset has no accumulated update")
            if tall:
                x = baddbmm(None, x, acc)
                gram = baddbmm(None, _mT(x), x)
            else:
                x = baddbmm(None, acc, x)
                gram = baddbmm(None, x, _mT(x))
            acc = None
        poly = baddbmm(gram, gram, gram, alpha=c, beta=b)
        if acc is None:
            alpha = to_f16(np.float32(a)) if identity_alpha_f16 else np.float32(a)
            acc = to_f16(poly + alpha * eye)
        else:
            acc = baddbmm(acc, acc, poly, alpha=1.0, beta=a)
        if it < len(coeffs) - 1 and (it + 1) not in resets:
            gp = baddbmm(gram, gram, poly, alpha=1.0, beta=a)
            gram = baddbmm(gp, poly, gp, alpha=1.0, beta=a)
    if acc is None:
        raise RuntimeError("Gram Newton--Schulz requires coefficients")
    return baddbmm(None, x, acc) if tall else baddbmm(None, acc, x)


def gram_iterations(
    gram: np.ndarray,
    coefficients: Sequence[Sequence[float]],
    it_begin: int,
    it_end: int,
    identity_alpha_f16: bool = False,
) -> np.ndarray:
    """Iterations ``[it_begin, it_end)`` of the Gram loop (newton_schulz.py:177-212)
    between two restarts: starts from the Gram matrix of the current X (rounded to
    fp16) with no accumulated update and returns the accumulated polynomial Q (fp16).
    ``gram_newton_schulz`` is these segments split at the reset iterations, with
    X <- X Q / Q X and a fresh Gram between them (newton_schulz.py:164-175)."""
    g = to_f16(gram)
    eye = np.broadcast_to(np.eye(g.shape[-1], dtype=np.float32), g.shape)
    acc = None
    for it in range(it_begin, it_end):
        a, b, c = coefficients[it]
        poly = baddbmm(g, g, g, alpha=c, beta=b)
        if acc is None:
            alpha = to_f16(np.float32(a)) if identity_alpha_f16 else np.float32(a)
            acc = to_f16(poly + alpha * eye)
        else:
            acc = baddbmm(acc, acc, poly, alpha=1.0, beta=a)
        if it + 1 < it_end:
            gp = baddbmm(g, g, poly, alpha=1.0, beta=a)
            g = baddbmm(gp, poly, gp, alpha=1.0, beta=a)
    if acc is None:
        raise ValueError("empty iteration range")
    return acc


def long_axis_sharded_gram_newton_schulz(
    shards: Sequence[np.ndarray],
    tall: bool,
    coefficients: Sequence[Sequence[float]] | None = None,
    reset_iterations: Sequence[int] = (2,),
    epsilon: float = 1e-7,
) -> list[np.ndarray]:
    """Gram Newton-Schulz of X = concat(shards) along its long axis (rows when
    ``tall``, else columns), computed the way the sharded chain computes it: the
    squared norm and the Gram matrix are fp32 sums of per-shard partials (each
    partial Gram an fp32-accumulated product of fp16 operands, the sum rounded to
    fp16), the Gram iterations run on the summed matrix, and each shard is
    multiplied by Q locally. Returns the output shards (fp16 values, fp32 storage).
    Not a reference code path: the reference gathers whole matrices instead
    (distributed_orthogonalization.py:278-349); this is the math it must match."""
    coeffs = coefficients if coefficients is not None else polar_express_coefficients()
    n = len(coeffs)
    xs = [np.asarray(s, dtype=np.float32) for s in shards]
    sumsq = sum(np.sum(np.square(x.astype(np.float64)), axis=(-2, -1), keepdims=True) for x in xs)
    denom = np.sqrt(sumsq).astype(np.float32) + np.float32(epsilon)
    xs = [to_f16(x / denom) for x in xs]

    def gram_of(parts: list[np.ndarray]) -> np.ndarray:
        total = sum(np.matmul(_mT(x), x) if tall else np.matmul(x, _mT(x)) for x in parts)
        return to_f16(total)

    def apply(q: np.ndarray, x: np.ndarray) -> np.ndarray:
        return baddbmm(None, x, q) if tall else baddbmm(None, q, x)

    boundaries = sorted({int(i) for i in reset_iterations if 0 < int(i) < n}) + [n]
    gram = gram_of(xs)
    begin = 0
    q = None
    for end in boundaries:
        q = gram_iterations(gram, coeffs, begin, end)
        if end < n:
            xs = [apply(q, x) for x in xs]
            gram = gram_of(xs)
        begin = end
    return [apply(q, x) for x in xs]


def standard_newton_schulz(
    matrix: np.ndarray,
    coefficients: Sequence[Sequence[float]] | None = None,
    epsilon: float = 1e-7,
) -> np.ndarray:
    """Standard Newton-Schulz (newton_schulz.py:79-115); fp16 values as fp32 storage."""
    coeffs = coefficients if coefficients is not None else polar_express_coefficients()
    x = np.asarray(matrix, dtype=np.float32)
    tall = x.shape[-2] > x.shape[-1]
    x = normalize(x, epsilon)
    for a, b, c in coeffs:
        gram = baddbmm(None, _mT(x), x) if tall else baddbmm(None, x, _mT(x))
        poly = baddbmm(gram, gram, gram, alpha=c, beta=b)
        x = baddbmm(x, x, poly, alpha=1.0, beta=a) if tall else baddbmm(x, poly, x, alpha=1.0, beta=a)
    return x


def orthogonalize(
    matrix: np.ndarray,
    coefficients: Sequence[Sequence[float]] | None = None,
    reset_iterations: Sequence[int] = (2,),
    epsilon: float = 1e-7,
    gram: bool = True,
    identity_alpha_f16: bool = False,
) -> np.ndarray:
    """NewtonSchulz.__call__ dispatch (newton_schulz.py:283-319) without the dtype cast:
    a Gram operation for non-square inputs when ``gram``, else the standard one."""
    x = np.asarray(matrix, dtype=np.float32)
    squeeze = x.ndim == 2
    if squeeze:
        x = x[None]
    lead = x.shape[:-2]
    x = x.reshape((-1, *x.shape[-2:]))
    if gram and x.shape[-2] != x.shape[-1]:
        out = gram_newton_schulz(x, coefficients, reset_iterations, epsilon, identity_alpha_f16)
    else:
        out = standard_newton_schulz(x, coefficients, epsilon)
    out = out.reshape((*lead, *out.shape[-2:]))
    return out[0] if squeeze else out


def relative_error(candidate: np.ndarray, reference: np.ndarray) -> float:
    """||candidate - reference||_F / ||reference||_F (benchmark.py:140-151)."""
    c = np.asarray(candidate, dtype=np.float64)
    r = np.asarray(reference, dtype=np.float64)
    return float(np.linalg.norm(c - r) / max(np.linalg.norm(r), np.finfo(np.float32).tiny))


def orthogonality_residual(output: np.ndarray) -> float:
    """mean over the batch of ||O O^T - I||_F / sqrt(m) (benchmark.py:154-165)."""
    o = np.asarray(output, dtype=np.float64)
    if o.ndim == 2:
        o = o[None]
    g = np.swapaxes(o, -1, -2) @ o if o.shape[-2] > o.shape[-1] else o @ np.swapaxes(o, -1, -2)
    eye = np.eye(g.shape[-1])
    res = np.linalg.norm(g - eye, axis=(-2, -1)) / np.sqrt(g.shape[-1])
    return float(res.mean())


def singular_value_band(output: np.ndarray) -> tuple[float, float]:
    """(min, max) singular value over the batch."""
    o = np.asarray(output, dtype=np.float64)
    if o.ndim == 2:
        o = o[None]
    s = np.linalg.svd(o, compute_uv=False)
    return float(s.min()), float(s.max())
