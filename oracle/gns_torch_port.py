"""TEST INFRASTRUCTURE, not product code: the reference's torch backend restated
with torch CPU operations, used as the timed CPU baseline of bench.py (its
``cpu_baseline`` leg and ``--impl reference``) and pinned against the reference's
own outputs by tests/test_oracle_golden.py.

It follows build_gram_newton_schulz_operation / build_standard_newton_schulz_operation
(newton_schulz.py:49-206) over TorchBackend (kernels/torch_ns.py:5-35): fp32
Frobenius normalisation rounded to fp16, then fp16 ``@`` / ``torch.baddbmm``
products in the same order, and the final cast (newton_schulz.py:302). The numpy
restatement in gns_oracle.py is the parity oracle; this module exists because
torch's CPU fp16 GEMMs are what the reference itself runs on a host, so timing
them gives the honest CPU figure (the numpy restatement emulates fp16 rounding
on fp32 BLAS and runs slower than the reference).
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
from torch import Tensor


def _normalise(x: Tensor, epsilon: float) -> Tensor:
    """newton_schulz.py:124-127."""
    x = x.to(torch.float32)
    return (x / (x.norm(dim=(-2, -1), keepdim=True) + epsilon)).to(torch.float16)


def gram_newton_schulz(
    x: Tensor, coefficients: Sequence[Sequence[float]], resets: Sequence[int] = (2,), epsilon: float = 1e-7
) -> Tensor:
    """Gram iteration (newton_schulz.py:122-200) on a [batch, rows, cols] tensor."""
    out_dtype = x.dtype
    tall = x.size(-2) > x.size(-1)
    reset = frozenset(int(i) for i in resets)
    xs = _normalise(x, epsilon)

    def gram(m: Tensor) -> Tensor:
        return m.mT @ m if tall else m @ m.mT

    g = gram(xs)
    eye = torch.eye(g.shape[-1], dtype=xs.dtype).unsqueeze(0).expand(g.shape[0], -1, -1).contiguous()
    q = None
    n = len(coefficients)
    for it, (a, b, c) in enumerate(coefficients):
        if it != 0 and it in reset:
            xs = xs @ q if tall else q @ xs
            g = gram(xs)
            q = None
        p = torch.baddbmm(g, g, g, alpha=float(c), beta=float(b))
        q = p.add(eye, alpha=float(a)) if q is None else torch.baddbmm(q, q, p, beta=float(a))
        if it < n - 1 and it + 1 not in reset:
            gp = torch.baddbmm(g, g, p, beta=float(a))
            g = torch.baddbmm(gp, p, gp, beta=float(a))
    y = xs @ q if tall else q @ xs
    return y.to(out_dtype)


def standard_newton_schulz(x: Tensor, coefficients: Sequence[Sequence[float]], epsilon: float = 1e-7) -> Tensor:
    """Standard iteration (newton_schulz.py:62-98)."""
    out_dtype = x.dtype
    tall = x.size(-2) > x.size(-1)
    xs = _normalise(x, epsilon)
    for a, b, c in coefficients:
        g = xs.mT @ xs if tall else xs @ xs.mT
        p = torch.baddbmm(g, g, g, alpha=float(c), beta=float(b))
        xs = torch.baddbmm(xs, xs, p, beta=float(a)) if tall else torch.baddbmm(xs, p, xs, beta=float(a))
    return xs.to(out_dtype)


def orthogonalize(x: Tensor, coefficients: Sequence[Sequence[float]], resets: Sequence[int] = (2,),
                  epsilon: float = 1e-7) -> Tensor:
    """NewtonSchulz.__call__'s dispatch (newton_schulz.py:282-302): square matrices
    take the standard iteration."""
    if x.size(-2) == x.size(-1):
        return standard_newton_schulz(x, coefficients, epsilon)
    return gram_newton_schulz(x, coefficients, resets, epsilon)
