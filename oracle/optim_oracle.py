"""CPU oracle for the Muon and Dion3 optimizer-state passes (numpy). TEST INFRASTRUCTURE ONLY.

Used as the checker by ``tests/`` only; the product never imports it.

Restated reference code (afrenkai/Gram-Newton-Schulz-Ampere):
- Muon momentum / Nesterov:    gram_newton_schulz_ampere/muon.py:423-438
- Muon decay + update:         gram_newton_schulz_ampere/muon.py:458-476, lr adjust :500-514
- Dion3 selection:             kernels/dion3_cuda.cu:39-90 + :336-351 (select_rows),
                               torch twin dion3_update.py:14-70
- Dion3 normalise + apply:     kernels/dion3_cuda.cu:92-211 + :353-503,
                               torch twin dion3_update.py:73-148

Rounding points follow the reference: values are rounded to the storage dtype
wherever the reference stores a tensor. Dtypes are named "f32", "bf16", "f16".
Row selection returns indices in ascending order; the reference's
``topk(sorted=False)`` order is unspecified, so index SETS are what is compared.
Pinned by ``tests/golden/make_golden.py`` against the reference's torch twins.
"""

from __future__ import annotations

from math import ceil, sqrt

import numpy as np


def to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bfloat16, returned as float32 storage."""
    u = np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out[nan] = np.nan
    return out


def to_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return to_bf16(x)
    if dtype == "f16":
        return to_f16(x)
    return np.asarray(x, dtype=np.float32)


def promote(a: str, b: str) -> str:
    """torch type promotion among f32 / bf16 / f16."""
    if a == b:
        return a
    return "f32"


# ------------------------------------------------------------------- Muon
def _axpy(x: np.ndarray, alpha: float, y: np.ndarray, dtype: str, cpu_rounding: bool) -> np.ndarray:
    """round(x + alpha * y) as torch.add(x, y, alpha=alpha) computes it in ``dtype``.

    torch's CUDA kernel evaluates x + alpha * y in fp32 and rounds once; its CPU
    kernel for 16-bit dtypes first rounds the scalar ``alpha`` to the dtype
    (``cpu_rounding=True``, used only to pin against reference runs on the CPU).
    """
    a = round_to(np.float32(alpha), dtype) if cpu_rounding else np.float32(alpha)
    return round_to(np.asarray(x, np.float32) + a * np.asarray(y, np.float32), dtype)


def muon_momentum(
    gradient: np.ndarray,
    momentum: np.ndarray,
    mu: float,
    nesterov: bool,
    g_dtype: str,
    m_dtype: str,
    cpu_rounding: bool = False,
) -> tuple[np.ndarray, np.ndarray]:
    """Returns (new momentum, update to orthogonalise) (muon.py:423-438).

    m <- round_m(round_m(g) + mu * m); u = round_u(g + mu * m) if Nesterov, else m;
    mu == 0 copies round_m(g) into m and orthogonalises g itself.
    """
    g = np.asarray(gradient, dtype=np.float32)
    gm = round_to(g, m_dtype)
    if mu == 0.0:
        return gm, g
    m_new = _axpy(gm, mu, momentum, m_dtype, cpu_rounding)
    if not nesterov:
        return m_new, m_new
    return m_new, _axpy(g, mu, m_new, promote(g_dtype, m_dtype), cpu_rounding)


def adjusted_learning_rate(lr: float, shape: tuple[int, ...], adjustment: str | None) -> float:
    """muon.py:500-514."""
    if adjustment is None:
        return lr
    rows, cols = shape[-2], shape[-1]
    if adjustment == "spectral_norm":
        return lr * sqrt(rows / cols)
    if adjustment == "rms_norm":
        return lr * 0.2 * sqrt(max(rows, cols))
    raise ValueError(adjustment)


def muon_apply(
    parameter: np.ndarray,
    update: np.ndarray,
    lr: float,
    weight_decay: float,
    lr_adj: float,
    p_dtype: str,
    cpu_rounding: bool = False,
) -> np.ndarray:
    """p <- round(p * (1 - lr wd)) when wd != 0, then p <- round(p - lr_adj * O) (muon.py:471-476)."""
    p = np.asarray(parameter, dtype=np.float32)
    if weight_decay != 0.0:
        p = round_to(p * np.float32(1.0 - lr * weight_decay), p_dtype)
    return _axpy(p, -lr_adj, update, p_dtype, cpu_rounding)


# ------------------------------------------------------------------ Dion3
def selected_count(rows: int, fraction: float) -> int:
    """k = max(1, ceil(fraction * rows)) (dion3.py:228)."""
    return max(1, ceil(fraction * rows))


def dion3_select(
    momentum: np.ndarray,
    gradient: np.ndarray,
    k: int,
    decay: float,
    parameter: np.ndarray | None = None,
    parameter_decay: float = 1.0,
    dtype: str = "f32",
) -> dict[str, np.ndarray]:
    """Selection pass for a [..., rows, cols] stack (select_rows, kernels/dion3_cuda.cu:336-351).

    Returns momentum/parameter after the pass, the bf16 selected rows, ascending
    indices and the fp64 row L1 norms that ranked them.
    """
    m = round_to(np.asarray(momentum, np.float32) + round_to(np.asarray(gradient, np.float32), dtype), dtype)
    p = None
    if parameter is not None:
        p = np.asarray(parameter, np.float32)
        if parameter_decay != 1.0:
            p = round_to(p * np.float32(parameter_decay), dtype)
    rows = m.shape[-2]
    lead = m.shape[:-2]
    mb = m.reshape(-1, rows, m.shape[-1])
    norms = np.abs(mb.astype(np.float64)).sum(axis=-1)
    k = min(k, rows)
    if k == rows:
        idx = np.broadcast_to(np.arange(rows), (mb.shape[0], rows)).copy()
    else:
        # Stable descending sort: ties resolved towards the lower row index.
        order = np.argsort(-norms, axis=-1, kind="stable")[:, :k]
        idx = np.sort(order, axis=-1)
    sel = np.take_along_axis(mb, idx[..., None], axis=1)
    selected = to_bf16(sel)
    decayed = round_to(sel * np.float32(decay), dtype)
    np.put_along_axis(mb, idx[..., None], decayed, axis=1)
    return {
        "momentum": mb.reshape(m.shape),
        "parameter": p,
        "selected": selected.reshape((*lead, k, m.shape[-1])),
        "indices": idx.reshape((*lead, k)).astype(np.int64),
        "norms": norms.reshape((*lead, rows)),
    }


def dion3_normalize_rows(
    update: np.ndarray,
    variance: np.ndarray,
    indices: np.ndarray,
    beta2: float,
    epsilon: float,
) -> dict[str, np.ndarray]:
    """The normalisation half (kernels/dion3_cuda.cu:92-165): variance EMA of the
    selected rows, n = u / (sqrt(v) + eps) in fp32, per-matrix (sum u^2, sum n^2)."""
    variance = np.asarray(variance, np.float32)
    rows = variance.shape[-2]
    cols = np.asarray(update).shape[-1]
    u = np.asarray(update, np.float32).reshape(-1, np.asarray(update).shape[-2], cols)
    v = variance.reshape(u.shape[0], rows).copy()
    idx = np.asarray(indices).reshape(u.shape[0], -1)
    ss_u = np.sum(u.astype(np.float64) ** 2, axis=-1)
    v_sel = np.take_along_axis(v, idx, axis=1)
    v_new = (np.float32(beta2) * v_sel + np.float32(1.0 - beta2) * (ss_u / cols).astype(np.float32)).astype(np.float32)
    np.put_along_axis(v, idx, v_new, axis=1)
    denom = np.sqrt(v_new) + np.float32(epsilon)
    n = (u / denom[..., None]).astype(np.float32)
    sums = np.stack([ss_u.sum(axis=-1), np.sum(n.astype(np.float64) ** 2, axis=(-2, -1))], axis=-1).astype(np.float32)
    return {
        "variance": v.reshape(variance.shape),
        "normalized": n.reshape(np.asarray(update).shape),
        "squared_norms": sums,
    }


def dion3_normalize_apply(
    parameter: np.ndarray,
    update: np.ndarray,
    variance: np.ndarray,
    indices: np.ndarray,
    beta2: float,
    epsilon: float,
    lr: float,
    weight_decay: float,
    lr_adj: float,
    p_dtype: str = "f32",
) -> dict[str, np.ndarray]:
    """NorMuon normalise + rescale + row update, CUDA-path rounding (kernels/dion3_cuda.cu:92-211)."""
    p = np.asarray(parameter, np.float32).copy()
    rows, cols = p.shape[-2], p.shape[-1]
    pb = p.reshape(-1, rows, cols)
    if weight_decay != 0.0:
        pb = round_to(pb * np.float32(1.0 - lr * weight_decay), p_dtype)
    u = np.asarray(update, np.float32).reshape(pb.shape[0], -1, cols)
    v = np.asarray(variance, np.float32).reshape(pb.shape[0], rows).copy()
    idx = np.asarray(indices).reshape(pb.shape[0], -1)
    ss_u = np.sum(u.astype(np.float64) ** 2, axis=-1)
    v_sel = np.take_along_axis(v, idx, axis=1)
    v_new = (np.float32(beta2) * v_sel + np.float32(1.0 - beta2) * (ss_u / cols).astype(np.float32)).astype(np.float32)
    np.put_along_axis(v, idx, v_new, axis=1)
    denom = np.sqrt(v_new) + np.float32(epsilon)
    n = (u / denom[..., None]).astype(np.float32)
    orig = np.sqrt(ss_u.sum(axis=-1)).astype(np.float32)
    normd = np.maximum(np.sqrt(np.sum(n.astype(np.float64) ** 2, axis=(-2, -1))), epsilon).astype(np.float32)
    rescaled = (n * orig[:, None, None] / normd[:, None, None]).astype(np.float32)
    scaled = round_to(rescaled, p_dtype)
    step = round_to(np.float32(-lr_adj) * scaled, p_dtype)
    rows_now = np.take_along_axis(pb, idx[..., None], axis=1)
    np.put_along_axis(pb, idx[..., None], round_to(rows_now + step, p_dtype), axis=1)
    return {
        "parameter": pb.reshape(p.shape),
        "variance": v.reshape(np.asarray(variance).shape),
        # The update after the norm-preserving rescale (what the reference returns).
        "normalized": rescaled.reshape(np.asarray(update).shape),
    }
