"""Tensor-level wrappers of the sm_100a kernels (C ABI in include/gns_b200.h).

Each function validates its tensors, allocates outputs and workspaces with
torch (so the caching allocator owns all memory), and launches on the current
CUDA stream of the tensors' device. There is no CPU path: non-CUDA tensors are
rejected and a missing native library raises.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
from collections.abc import Iterator, Sequence

import torch
from torch import Tensor

from gram_newton_schulz_ampere_b200 import _native as nat


# ----------------------------------------------------- bounded-wait status
class DeviceWaitError(nat.NativeError):
    """A kernel's bounded wait ran out; its results are invalid (NaN where the
    normalisation gave up)."""


_status = {"enabled": os.environ.get("GNS_B200_CHECK_STATUS", "") not in ("", "0"), "depth": 0}


def set_status_checks(enabled: bool) -> bool:
    """Opt in (or out) of a device-status check after every public call
    (``GramNewtonSchulz.__call__``, ``Muon.step``, ``Dion3.step``; also set by the
    environment variable GNS_B200_CHECK_STATUS=1). Each check synchronises the
    device once per outermost call. Returns the previous setting."""
    previous = bool(_status["enabled"])
    _status["enabled"] = bool(enabled)
    return previous


def check_device_status() -> None:
    """Reads and clears the device status word; raises DeviceWaitError if a
    kernel's bounded wait ran out since the last read."""
    code = nat.device_status(clear=True)
    if code != 0:
        raise DeviceWaitError(f"a kernel's bounded wait ran out (device status {code}); results are invalid")


@contextlib.contextmanager
def status_checked() -> Iterator[None]:
    """Runs the body and, when checks are enabled, checks the device status once
    at the end of the outermost such block."""
    _status["depth"] += 1
    try:
        yield
    finally:
        _status["depth"] -= 1
    if _status["depth"] == 0 and _status["enabled"]:
        check_device_status()


def _require_cuda(*tensors: Tensor | None) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("gram_newton_schulz_ampere_b200 kernels require CUDA tensors")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError("all tensors must be on the same CUDA device")
    if device is None:
        raise ValueError("no tensor given")
    return device


def _workspace(nbytes: int, device: torch.device) -> Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def _as_batched(t: Tensor) -> Tensor:
    if t.ndim == 2:
        return t.unsqueeze(0)
    if t.ndim == 3:
        return t
    raise ValueError("expected a matrix or a batch of matrices")


def _aligned_operand(t: Tensor) -> Tensor:
    """Returns `t` if a TMA tile load can read it (unit stride on one matrix axis,
    16-byte aligned base and strides), else a copy whose row pitch is padded to a
    multiple of 8 elements. The copy is layout plumbing only."""
    es = t.element_size()
    b, r, c = t.shape
    sb, sr, sc = t.stride()
    base_ok = t.data_ptr() % 16 == 0

    def ok_stride(s: int, extent: int) -> bool:
        return extent == 1 or (s * es) % 16 == 0

    if base_ok and (sc == 1 or c == 1) and ok_stride(sr, r) and ok_stride(sb, b):
        return t
    if base_ok and (sr == 1 or r == 1) and ok_stride(sc, c) and ok_stride(sb, b):
        return t
    pitch = (c + 7) // 8 * 8
    padded = torch.empty((b, r, pitch), dtype=t.dtype, device=t.device)
    view = padded[:, :, :c]
    view.copy_(t)
    return view


def gemm(
    left: Tensor,
    right: Tensor,
    accumulator: Tensor | None = None,
    alpha: float = 1.0,
    beta: float = 0.0,
    symmetric: bool = False,
    out_dtype: torch.dtype | None = None,
) -> Tensor:
    """``alpha * left @ right + beta * accumulator`` on tcgen05 tensor cores.

    left [B, m, k] and right [B, k, n] share dtype float16 or bfloat16; either may
    be a transposed view. With ``symmetric=True`` the caller asserts the result is
    symmetric: only its upper triangle is computed and mirrored (exactly symmetric
    output), as the reference's symmetric CUTLASS kernels do
    (kernels/cutlass_ns.cu:167-223 + mirror_lower_triangle :127-165).
    When beta == 0 the accumulator is never read (NaNs in it do not propagate,
    matching torch.baddbmm). Inside a region that torch.compile traces, the call
    is the custom op ``torch.ops.gns_b200.gemm``.
    """
    if torch.compiler.is_compiling():
        return torch.ops.gns_b200.gemm(left, right, accumulator, float(alpha), float(beta), bool(symmetric),
                                       out_dtype)
    return _gemm_eager(left, right, accumulator, alpha, beta, symmetric, out_dtype)


def _gemm_eager(
    left: Tensor,
    right: Tensor,
    accumulator: Tensor | None = None,
    alpha: float = 1.0,
    beta: float = 0.0,
    symmetric: bool = False,
    out_dtype: torch.dtype | None = None,
) -> Tensor:
    device = _require_cuda(left, right, accumulator)
    squeeze = left.ndim == 2
    a = _as_batched(left)
    b = _as_batched(right)
    if a.dtype != b.dtype or a.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("left and right must share dtype float16 or bfloat16")
    if a.shape[0] != b.shape[0] or a.shape[2] != b.shape[1]:
        raise ValueError(f"incompatible shapes {tuple(left.shape)} @ {tuple(right.shape)}")
    batch, m, k = a.shape
    n = b.shape[2]
    if symmetric and m != n:
        raise ValueError("a symmetric product must be square")
    dtype = out_dtype or a.dtype
    out = torch.empty((batch, m, n), dtype=dtype, device=device)
    if batch == 0 or m == 0 or n == 0:
        return out[0] if squeeze else out
    if k == 0:
        out.zero_()
        if accumulator is not None and beta != 0.0:
            out.add_(_as_batched(accumulator).expand(batch, m, n), alpha=beta)
        return out[0] if squeeze else out
    a = _aligned_operand(a)
    b = _aligned_operand(b)
    c = None
    if accumulator is not None and beta != 0.0:
        c = _as_batched(accumulator)
        if c.shape != (batch, m, n):
            c = c.expand(batch, m, n)
        if c.dtype != dtype:
            c = c.to(dtype)
        if c.stride(-1) != 1 or (batch > 1 and c.stride(0) == 0):
            c = c.contiguous()
    lib = nat.load()
    with torch.cuda.device(device):
        rc = lib.gns_gemm(
            nat.dtype_code(a.dtype), batch, m, n, k,
            a.data_ptr(), a.stride(0), a.stride(1), a.stride(2),
            b.data_ptr(), b.stride(0), b.stride(1), b.stride(2),
            nat.ptr(c), nat.dtype_code(c.dtype) if c is not None else 0,
            c.stride(0) if c is not None else 0, c.stride(1) if c is not None else 0,
            out.data_ptr(), nat.dtype_code(dtype), out.stride(0), out.stride(1),
            float(alpha), float(beta) if c is not None else 0.0, 1 if symmetric else 0,
            nat.stream_handle(device),
        )
    nat.check(rc, "gns_gemm")
    return out[0] if squeeze else out


@torch.library.custom_op("gns_b200::gemm", mutates_args=())
def _gemm_op(
    left: Tensor, right: Tensor, accumulator: Tensor | None, alpha: float, beta: float, symmetric: bool,
    out_dtype: torch.dtype | None,
) -> Tensor:
    return _gemm_eager(left, right, accumulator, alpha, beta, symmetric, out_dtype)


@_gemm_op.register_fake
def _(left, right, accumulator, alpha, beta, symmetric, out_dtype):  # type: ignore[no-untyped-def]
    shape = (left.shape[-2], right.shape[-1]) if left.ndim == 2 else (left.shape[0], left.shape[-2], right.shape[-1])
    return torch.empty(shape, dtype=out_dtype or left.dtype, device=left.device)


def frobenius_normalize(matrix: Tensor, epsilon: float) -> Tensor:
    """fp16(X / (||X||_F + eps)) per matrix, norm in fp32 (newton_schulz.py:141-144)."""
    device = _require_cuda(matrix)
    x = _as_batched(matrix)
    if x.stride(-1) != 1:
        x = x.contiguous()
    batch, rows, cols = x.shape
    ld = (cols + 7) // 8 * 8
    out = torch.empty((batch, rows, ld), dtype=torch.float16, device=device)[:, :, :cols]
    lib = nat.load()
    ws = _workspace(lib.gns_normalize_workspace_size(batch, rows, cols), device)
    with torch.cuda.device(device):
        rc = lib.gns_frobenius_normalize(
            nat.dtype_code(x.dtype), batch, rows, cols, x.data_ptr(), x.stride(0), x.stride(1),
            out.data_ptr(), ld, float(epsilon), ws.data_ptr(), ws.numel(), nat.stream_handle(device),
        )
    nat.check(rc, "gns_frobenius_normalize")
    return out if matrix.ndim == 3 else out[0]


def _coefficient_array(coefficients: Sequence[Sequence[float]]) -> ctypes.Array:
    flat = [float(v) for triple in coefficients for v in triple]
    if len(flat) != 3 * len(coefficients):
        raise ValueError("each coefficient entry must be an (a, b, c) triple")
    return (ctypes.c_double * max(len(flat), 1))(*flat)


def _chain_input(matrix: Tensor) -> Tensor:
    x = _as_batched(matrix)
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x


def newton_schulz_chain(
    matrix: Tensor,
    coefficients: Sequence[Sequence[float]],
    epsilon: float,
    gram: bool,
    reset_iterations: Sequence[int] = (),
    out_dtype: torch.dtype | None = None,
) -> Tensor:
    """Whole (Gram) Newton-Schulz orthogonalisation of [B, r, c] in one native call.

    Follows build_gram_newton_schulz_operation / build_standard_newton_schulz_operation
    (newton_schulz.py:66-223): fp32 Frobenius normalisation, fp16 products with fp32
    accumulation, output cast to ``out_dtype`` (default: the input dtype). Inside a
    region that torch.compile traces, the call is the custom op
    ``torch.ops.gns_b200.newton_schulz_chain`` (same kernels, no graph break).
    """
    if torch.compiler.is_compiling():
        return torch.ops.gns_b200.newton_schulz_chain(
            matrix, [float(v) for triple in coefficients for v in triple], float(epsilon), bool(gram),
            [int(i) for i in reset_iterations], out_dtype or matrix.dtype,
        )
    return _newton_schulz_chain_eager(matrix, coefficients, epsilon, gram, reset_iterations, out_dtype)


def _newton_schulz_chain_eager(
    matrix: Tensor,
    coefficients: Sequence[Sequence[float]],
    epsilon: float,
    gram: bool,
    reset_iterations: Sequence[int] = (),
    out_dtype: torch.dtype | None = None,
) -> Tensor:
    device = _require_cuda(matrix)
    x = _chain_input(matrix)
    batch, rows, cols = x.shape
    dtype = out_dtype or matrix.dtype
    out = torch.empty((batch, rows, cols), dtype=dtype, device=device)
    if len(coefficients) > 32:
        raise ValueError("at most 32 Newton-Schulz iterations are supported")
    mask = 0
    for it in reset_iterations:
        if it < 0:
            raise ValueError("reset iterations must be non-negative")
        if it < 32:
            mask |= 1 << int(it)
    coeffs = _coefficient_array(coefficients)
    lib = nat.load()
    ws = _workspace(lib.gns_newton_schulz_workspace_size(batch, rows, cols), device)
    with torch.cuda.device(device):
        if gram:
            rc = lib.gns_gram_newton_schulz(
                nat.dtype_code(x.dtype), batch, rows, cols, x.data_ptr(), x.stride(0), x.stride(1),
                out.data_ptr(), nat.dtype_code(dtype), out.stride(0), out.stride(1),
                coeffs, len(coefficients), mask, float(epsilon), ws.data_ptr(), ws.numel(),
                nat.stream_handle(device),
            )
        else:
            rc = lib.gns_standard_newton_schulz(
                nat.dtype_code(x.dtype), batch, rows, cols, x.data_ptr(), x.stride(0), x.stride(1),
                out.data_ptr(), nat.dtype_code(dtype), out.stride(0), out.stride(1),
                coeffs, len(coefficients), float(epsilon), ws.data_ptr(), ws.numel(),
                nat.stream_handle(device),
            )
    if rc != 0:
        msg = nat.last_error()
        if "requires coefficients" in msg or "no accumulated update" in msg:
            raise RuntimeError(msg)
        nat.check(rc, "Newton-Schulz chain")
    return out if matrix.ndim == 3 else out[0]


@torch.library.custom_op("gns_b200::newton_schulz_chain", mutates_args=())
def _newton_schulz_chain_op(
    matrix: Tensor, coefficients: list[float], epsilon: float, gram: bool, reset_iterations: list[int],
    out_dtype: torch.dtype,
) -> Tensor:
    triples = [coefficients[i:i + 3] for i in range(0, len(coefficients), 3)]
    return _newton_schulz_chain_eager(matrix, triples, epsilon, gram, reset_iterations, out_dtype)


@_newton_schulz_chain_op.register_fake
def _(matrix, coefficients, epsilon, gram, reset_iterations, out_dtype):  # type: ignore[no-untyped-def]
    # The output has the input's shape and is contiguous, like the native call's.
    return torch.empty(matrix.shape, dtype=out_dtype, device=matrix.device)


# ------------------------------------------------ sharded-chain pieces
@contextlib.contextmanager
def small_chain_tactic(enabled: bool) -> Iterator[None]:
    """Within the block, Gram Newton-Schulz calls on matrices with a short side of
    at most 128 run as one fused kernel (``enabled``, the default) or as one GEMM
    launch per product; the previous setting is restored on exit. The switch is
    process-wide (``gns_set_small_chain``)."""
    lib = nat.load()
    previous = lib.gns_set_small_chain(1 if enabled else 0)
    try:
        yield
    finally:
        lib.gns_set_small_chain(previous)


def gemm_sm_limit(sms: int) -> int:
    """Caps the SMs each GEMM launch occupies (0: all), process-wide; returns the
    previous cap (``gns_set_gemm_sm_limit``)."""
    return int(nat.load().gns_set_gemm_sm_limit(int(sms)))


def _padded(batch: int, rows: int, cols: int, dtype: torch.dtype, device: torch.device) -> Tensor:
    """[batch, rows, cols] view of a buffer whose row pitch is a multiple of 8 elements."""
    pitch = (cols + 7) // 8 * 8
    return torch.empty((batch, rows, pitch), dtype=dtype, device=device)[:, :, :cols]


def frobenius_sumsq(matrix: Tensor) -> Tensor:
    """Per-matrix sum of squares in fp32 (fixed summation order), shape [batch]."""
    device = _require_cuda(matrix)
    x = _chain_input(matrix)
    batch, rows, cols = x.shape
    out = torch.empty(batch, dtype=torch.float32, device=device)
    lib = nat.load()
    ws = _workspace(lib.gns_normalize_workspace_size(batch, rows, cols), device)
    with torch.cuda.device(device):
        rc = lib.gns_frobenius_sumsq(
            nat.dtype_code(x.dtype), batch, rows, cols, x.data_ptr(), x.stride(0), x.stride(1), out.data_ptr(),
            ws.data_ptr(), ws.numel(), nat.stream_handle(device),
        )
    nat.check(rc, "gns_frobenius_sumsq")
    return out


def frobenius_scale(matrix: Tensor, sumsq: Tensor, epsilon: float) -> Tensor:
    """fp16(X / (sqrt(sumsq) + eps)) per matrix, for a sum of squares computed elsewhere."""
    device = _require_cuda(matrix, sumsq)
    x = _chain_input(matrix)
    batch, rows, cols = x.shape
    if sumsq.dtype != torch.float32 or sumsq.numel() != batch:
        raise ValueError("sumsq must hold one fp32 value per matrix")
    out = _padded(batch, rows, cols, torch.float16, device)
    lib = nat.load()
    with torch.cuda.device(device):
        rc = lib.gns_frobenius_scale(
            nat.dtype_code(x.dtype), batch, rows, cols, x.data_ptr(), x.stride(0), x.stride(1),
            sumsq.contiguous().data_ptr(), float(epsilon), out.data_ptr(), out.stride(1), nat.stream_handle(device),
        )
    nat.check(rc, "gns_frobenius_scale")
    return out


def gram_iterations(
    gram: Tensor,
    coefficients: Sequence[Sequence[float]],
    it_begin: int,
    it_end: int,
) -> Tensor:
    """Runs Gram iterations [it_begin, it_end) between two restarts from G (fp32 or
    fp16 [B, m, m], rounded to fp16); returns the accumulated polynomial Q in fp16."""
    device = _require_cuda(gram)
    g = _as_batched(gram)
    if g.dtype not in (torch.float32, torch.float16) or g.stride(-1) != 1:
        g = g.float().contiguous()
    batch, m, _ = g.shape
    q = _padded(batch, m, m, torch.float16, device)
    coeffs = _coefficient_array(coefficients)
    lib = nat.load()
    ws = _workspace(lib.gns_gram_iterations_workspace_size(batch, m), device)
    with torch.cuda.device(device):
        rc = lib.gns_gram_iterations(
            batch, m, g.data_ptr(), 1 if g.dtype == torch.float32 else 0, g.stride(0), g.stride(1), coeffs,
            len(coefficients), int(it_begin), int(it_end), q.data_ptr(), q.stride(0), q.stride(1),
            ws.data_ptr(), ws.numel(), nat.stream_handle(device),
        )
    nat.check(rc, "gns_gram_iterations")
    return q if gram.ndim == 3 else q[0]


# ------------------------------------------------------------------- Muon
def _ptr_array(tensors: Sequence[Tensor | None]) -> ctypes.Array:
    return (ctypes.c_void_p * max(len(tensors), 1))(*[0 if t is None else t.data_ptr() for t in tensors])


def muon_momentum(
    gradients: Sequence[Tensor],
    momenta: Sequence[Tensor],
    momentum: float,
    nesterov: bool,
    wanted: Sequence[bool] | None = None,
) -> list[Tensor | None] | None:
    """Fused multi-tensor Muon momentum (muon.py:423-438).

    Updates every momentum buffer in place (m <- g + mu m) and, for Nesterov,
    returns new update tensors u = g + mu m. Returns None when the caller should
    use the gradient (mu == 0) or the momentum buffer itself (no Nesterov).
    ``wanted`` (Nesterov only) limits the update outputs to the marked tensors;
    the others advance their momentum and get None.
    """
    if len(gradients) != len(momenta):
        raise ValueError("gradients and momenta must have equal lengths")
    if not gradients:
        return [] if nesterov and momentum != 0.0 else None
    device = _require_cuda(*gradients, *momenta)
    g_dtype = gradients[0].dtype
    m_dtype = momenta[0].dtype
    for g, m in zip(gradients, momenta, strict=True):
        if g.dtype != g_dtype or m.dtype != m_dtype:
            raise TypeError("all gradients (and all momenta) of one call must share a dtype")
        if g.shape != m.shape:
            raise ValueError("gradient and momentum shapes differ")
        if not (g.is_contiguous() and m.is_contiguous()):
            raise ValueError("gradients and momenta must be contiguous")
    write_update = nesterov and momentum != 0.0
    u_dtype = torch.promote_types(g_dtype, m_dtype)
    if wanted is not None and len(wanted) != len(gradients):
        raise ValueError("wanted must have one flag per gradient")
    updates: list[Tensor | None] | None = None
    if write_update:
        # Updates of one shape are consecutive slices of one buffer, in order, so a
        # bucket of them is already the batch an orthogonaliser takes (no stacking copy).
        by_shape: dict[tuple[int, ...], list[int]] = {}
        for index, g in enumerate(gradients):
            if wanted is None or wanted[index]:
                by_shape.setdefault(tuple(g.shape), []).append(index)
        slots: list[Tensor | None] = [None] * len(gradients)
        for shape, indices in by_shape.items():
            block = torch.empty((len(indices), *shape), dtype=u_dtype, device=device)
            for position, index in enumerate(indices):
                slots[index] = block[position]
        updates = slots
    numel = (ctypes.c_int64 * len(gradients))(*[g.numel() for g in gradients])
    lib = nat.load()
    with torch.cuda.device(device):
        rc = lib.gns_muon_momentum(
            len(gradients), _ptr_array(gradients), _ptr_array(momenta),
            _ptr_array(updates) if updates is not None else None, numel,
            nat.dtype_code(g_dtype), nat.dtype_code(m_dtype), nat.dtype_code(u_dtype),
            float(momentum), 1 if write_update else 0, nat.stream_handle(device),
        )
    nat.check(rc, "gns_muon_momentum")
    return updates


def muon_apply(
    parameters: Sequence[Tensor],
    updates: Sequence[Tensor],
    decay: float | None,
    adjusted_learning_rates: Sequence[float],
) -> None:
    """Fused multi-tensor ``p <- p * decay; p <- p - lr_adj * update`` (muon.py:471-476)."""
    if not parameters:
        return
    if not (len(parameters) == len(updates) == len(adjusted_learning_rates)):
        raise ValueError("parameters, updates and learning rates must have equal lengths")
    device = _require_cuda(*parameters, *updates)
    p_dtype, o_dtype = parameters[0].dtype, updates[0].dtype
    for p, o in zip(parameters, updates, strict=True):
        if p.dtype != p_dtype or o.dtype != o_dtype:
            raise TypeError("all parameters (and all updates) of one call must share a dtype")
        if p.numel() != o.numel():
            raise ValueError("parameter and update sizes differ")
        if not (p.is_contiguous() and o.is_contiguous()):
            raise ValueError("parameters and updates must be contiguous")
    numel = (ctypes.c_int64 * len(parameters))(*[p.numel() for p in parameters])
    lrs = (ctypes.c_float * len(parameters))(*[float(v) for v in adjusted_learning_rates])
    lib = nat.load()
    with torch.cuda.device(device):
        rc = lib.gns_muon_apply(
            len(parameters), _ptr_array(parameters), _ptr_array(updates), numel,
            nat.dtype_code(p_dtype), nat.dtype_code(o_dtype),
            float(decay if decay is not None else 1.0), 0 if decay is None else 1, lrs,
            nat.stream_handle(device),
        )
    nat.check(rc, "gns_muon_apply")


# ------------------------------------------------------------------- Dion3
def _leading(t: Tensor) -> int:
    b = 1
    for s in t.shape[:-2]:
        b *= s
    return b


def dion3_select_rows(
    momentum: Tensor,
    gradient: Tensor,
    parameter: Tensor | None,
    selected_count: int,
    decay: float,
    parameter_decay: float,
) -> tuple[Tensor, Tensor]:
    """Fused momentum + decay + L1 row norm, top-k rows, gather + error-feedback decay.

    Returns (bf16 selected rows [..., k, cols], int64 indices [..., k] ascending).
    Mirrors select_rows (kernels/dion3_cuda.cu:336-351) / select_dion3_rows
    (dion3_update.py:14-70); k == rows selects every row.
    """
    device = _require_cuda(momentum, gradient, parameter)
    if momentum.ndim < 2:
        raise ValueError("momentum must have at least two dimensions")
    if gradient.shape != momentum.shape:
        raise ValueError("momentum and gradient shapes must match")
    if parameter is not None and parameter.shape != momentum.shape:
        raise ValueError("momentum and parameter shapes must match")
    if not momentum.is_contiguous():
        raise ValueError("momentum must be C contiguous")
    grad = gradient.to(dtype=momentum.dtype).contiguous()
    if parameter is not None:
        if parameter.dtype != momentum.dtype or not parameter.is_contiguous():
            raise ValueError("parameter must be contiguous with the momentum dtype")
    rows, cols = momentum.shape[-2], momentum.shape[-1]
    batch = _leading(momentum)
    lead = tuple(momentum.shape[:-2])
    k = int(selected_count)
    if rows == 0:
        momentum.add_(grad)
        if parameter is not None and parameter_decay != 1.0:
            parameter.mul_(parameter_decay)
        return momentum.to(torch.bfloat16), torch.empty((*lead, 0), dtype=torch.long, device=device)
    k = min(k, rows)
    if k < 1:
        raise ValueError("selected_count must be positive")
    selected = torch.empty((*lead, k, cols), dtype=torch.bfloat16, device=device)
    indices = torch.empty((*lead, k), dtype=torch.long, device=device)
    lib = nat.load()
    ws = _workspace(lib.gns_dion3_select_workspace_size(batch, rows), device)
    with torch.cuda.device(device):
        rc = lib.gns_dion3_select_rows(
            nat.dtype_code(momentum.dtype), batch, rows, cols, momentum.data_ptr(), grad.data_ptr(),
            nat.ptr(parameter), k, float(decay),
            float(parameter_decay) if parameter is not None else 1.0,
            selected.data_ptr(), indices.data_ptr(), ws.data_ptr(), ws.numel(), nat.stream_handle(device),
        )
    nat.check(rc, "gns_dion3_select_rows")
    return selected, indices


def dion3_select_rows_multi(
    momenta: Sequence[Tensor],
    gradients: Sequence[Tensor],
    parameters: Sequence[Tensor] | None,
    selected_count: int,
    decay: float,
    parameter_decay: float,
) -> tuple[Tensor, Tensor]:
    """dion3_select_rows over separate same-shape matrices in one set of launches.

    Returns one bf16 stack [n, k, cols] of the selected rows and one int64 stack
    [n, k] of ascending indices (row i is matrix i's selection). Mirrors
    select_dion3_rows_cuda_batch (kernels/dion3_cuda.py:111-149) for a bucket of
    equal shapes and counts.
    """
    count = len(momenta)
    if len(gradients) != count or (parameters is not None and len(parameters) != count):
        raise ValueError("batched selection inputs must have equal lengths")
    if count == 0:
        raise ValueError("batched selection needs at least one matrix")
    device = _require_cuda(*momenta, *gradients, *(parameters or []))
    first = momenta[0]
    if first.ndim != 2:
        raise ValueError("batched selection takes 2-D matrices")
    rows, cols = first.shape
    dtype = first.dtype
    grads = []
    for i, m in enumerate(momenta):
        if m.shape != first.shape or m.dtype != dtype or not m.is_contiguous():
            raise ValueError("batched selection needs contiguous momenta of one shape and dtype")
        if gradients[i].shape != first.shape:
            raise ValueError("momentum and gradient shapes must match")
        grads.append(gradients[i].to(dtype=dtype).contiguous())
        if parameters is not None:
            p = parameters[i]
            if p.shape != first.shape or p.dtype != dtype or not p.is_contiguous():
                raise ValueError("parameters must be contiguous with the momentum shape and dtype")
    k = min(int(selected_count), rows)
    if k < 1 or rows == 0:
        raise ValueError("batched selection requires 1 <= selected_count and rows > 0")
    selected = torch.empty((count, k, cols), dtype=torch.bfloat16, device=device)
    indices = torch.empty((count, k), dtype=torch.long, device=device)
    lib = nat.load()
    ws = _workspace(lib.gns_dion3_select_workspace_size(count, rows), device)
    with torch.cuda.device(device):
        rc = lib.gns_dion3_select_rows_multi(
            nat.dtype_code(dtype), count, rows, cols, _ptr_array(momenta), _ptr_array(grads),
            _ptr_array(parameters) if parameters is not None else None, k, float(decay),
            float(parameter_decay) if parameters is not None else 1.0,
            selected.data_ptr(), indices.data_ptr(), ws.data_ptr(), ws.numel(), nat.stream_handle(device),
        )
    nat.check(rc, "gns_dion3_select_rows_multi")
    return selected, indices


def dion3_normalize_apply_multi(
    parameters: Sequence[Tensor],
    selected_updates: Tensor,
    variances: Sequence[Tensor],
    indices: Tensor,
    beta_two: float,
    epsilon: float,
    learning_rate: float,
    weight_decay: float,
    adjusted_learning_rate: float,
) -> None:
    """dion3_normalize_apply over separate same-shape parameters: ``selected_updates``
    is one [n, k, cols] stack and ``indices`` one [n, k] stack (row i belongs to
    parameter i). Mirrors normalize_apply_rows_cuda_batch (kernels/dion3_cuda.py:220-253)
    for a bucket of equal shapes, counts and adjusted learning rates."""
    count = len(parameters)
    if len(variances) != count or selected_updates.shape[0] != count or indices.shape[0] != count:
        raise ValueError("batched normalization inputs must have equal lengths")
    if count == 0:
        return
    device = _require_cuda(*parameters, *variances, selected_updates, indices)
    first = parameters[0]
    rows, cols = first.shape[-2], first.shape[-1]
    for p, v in zip(parameters, variances, strict=True):
        if p.shape != first.shape or p.dtype != first.dtype or not p.is_contiguous():
            raise ValueError("parameters must be contiguous and share one shape and dtype")
        if v.dtype != torch.float32 or not v.is_contiguous() or v.numel() != rows:
            raise ValueError("variances must be contiguous float32 with one entry per row")
    if indices.dtype != torch.long:
        raise ValueError("indices must be int64")
    k = selected_updates.shape[-2]
    if selected_updates.shape != (count, k, cols) or indices.shape != (count, k):
        raise ValueError("selected_updates must be [n, k, cols] and indices [n, k]")
    u = selected_updates if selected_updates.stride(-1) == 1 else selected_updates.contiguous()
    idx = indices.contiguous()
    lib = nat.load()
    ws = _workspace(lib.gns_dion3_normalize_workspace_size(count, max(k, 1)), device)
    with torch.cuda.device(device):
        rc = lib.gns_dion3_normalize_apply_multi(
            nat.dtype_code(first.dtype), nat.dtype_code(u.dtype), count, rows, cols, k,
            _ptr_array(parameters), u.data_ptr() if k > 0 else None, u.stride(0), u.stride(1),
            _ptr_array(variances), idx.data_ptr() if k > 0 else None,
            float(beta_two), float(epsilon), float(learning_rate), float(weight_decay),
            float(adjusted_learning_rate), ws.data_ptr(), ws.numel(), nat.stream_handle(device),
        )
    nat.check(rc, "gns_dion3_normalize_apply_multi")


def dion3_normalize_apply(
    parameter: Tensor,
    selected_update: Tensor,
    variance: Tensor,
    indices: Tensor,
    beta_two: float,
    epsilon: float,
    learning_rate: float,
    weight_decay: float,
    adjusted_learning_rate: float,
) -> None:
    """NorMuon per-neuron normalisation + norm-preserving rescale + row scatter update
    (kernels/dion3_cuda.cu:353-503; dion3_update.py:73-148)."""
    device = _require_cuda(parameter, selected_update, variance, indices)
    if not parameter.is_contiguous():
        raise ValueError("parameter must be C contiguous")
    if variance.dtype != torch.float32 or not variance.is_contiguous():
        raise ValueError("variance must be contiguous float32")
    if indices.dtype != torch.long:
        raise ValueError("indices must be int64")
    rows, cols = parameter.shape[-2], parameter.shape[-1]
    batch = _leading(parameter)
    k = selected_update.shape[-2]
    if variance.numel() != batch * rows:
        raise ValueError("variance and parameter batch dimensions must match")
    if indices.numel() != batch * k:
        raise ValueError("indices and selected_update shapes must match")
    if selected_update.numel() != batch * k * cols:
        raise ValueError("parameter and selected_update batch dimensions must match")
    u = selected_update.reshape(batch, k, cols)
    if u.stride(-1) != 1:
        u = u.contiguous()
    idx = indices.reshape(batch * k).contiguous() if k > 0 else indices
    lib = nat.load()
    ws = _workspace(lib.gns_dion3_normalize_workspace_size(batch, max(k, 1)), device)
    with torch.cuda.device(device):
        rc = lib.gns_dion3_normalize_apply(
            nat.dtype_code(parameter.dtype), nat.dtype_code(u.dtype), batch, rows, cols, k,
            parameter.data_ptr(), u.data_ptr() if k > 0 else None, u.stride(0), u.stride(1),
            variance.data_ptr(), idx.data_ptr() if k > 0 else None,
            float(beta_two), float(epsilon), float(learning_rate), float(weight_decay),
            float(adjusted_learning_rate), ws.data_ptr(), ws.numel(), nat.stream_handle(device),
        )
    nat.check(rc, "gns_dion3_normalize_apply")


def dion3_normalize_rows(
    selected_update: Tensor,
    variance: Tensor,
    indices: Tensor,
    beta_two: float,
    epsilon: float,
) -> tuple[Tensor, Tensor]:
    """The normalisation half of dion3_normalize_apply (reference kernels/dion3_cuda.cu:353-400):
    updates ``variance`` in place and returns (normalized fp32 [*, k, cols], squared_norms fp32 [batch, 2])."""
    device = _require_cuda(selected_update, variance, indices)
    if variance.dtype != torch.float32 or not variance.is_contiguous():
        raise ValueError("variance must be contiguous float32")
    if indices.dtype != torch.long:
        raise ValueError("indices must be int64")
    k, cols = selected_update.shape[-2], selected_update.shape[-1]
    batch = _leading(selected_update)
    rows = variance.shape[-2]
    if indices.numel() != batch * k:
        raise ValueError("indices and selected_update shapes must match")
    if variance.numel() != batch * rows:
        raise ValueError("variance and selected_update batch dimensions must match")
    normalized = torch.empty(selected_update.shape, dtype=torch.float32, device=device)
    squared_norms = torch.empty((batch, 2), dtype=torch.float32, device=device)
    u = selected_update.reshape(batch, k, cols)
    if u.stride(-1) != 1:
        u = u.contiguous()
    idx = indices.reshape(batch * k).contiguous() if k > 0 else indices
    lib = nat.load()
    ws = _workspace(lib.gns_dion3_normalize_workspace_size(batch, max(k, 1)), device)
    with torch.cuda.device(device):
        rc = lib.gns_dion3_normalize_rows(
            nat.dtype_code(u.dtype), batch, rows, cols, k, u.data_ptr() if k > 0 else None, u.stride(0), u.stride(1),
            variance.data_ptr(), idx.data_ptr() if k > 0 else None, float(beta_two), float(epsilon),
            normalized.data_ptr() if normalized.numel() else None, squared_norms.data_ptr(), ws.data_ptr(),
            ws.numel(), nat.stream_handle(device),
        )
    nat.check(rc, "gns_dion3_normalize_rows")
    return normalized, squared_norms


def dion3_apply_rows(
    parameter: Tensor,
    normalized_update: Tensor,
    indices: Tensor,
    squared_norms: Tensor,
    learning_rate: float,
    weight_decay: float,
    adjusted_learning_rate: float,
    epsilon: float,
) -> None:
    """The update half of dion3_normalize_apply (reference kernels/dion3_cuda.cu:402-470): decays the
    parameter and adds the norm-preserving rescaled ``normalized_update`` to the selected rows."""
    device = _require_cuda(parameter, normalized_update, indices, squared_norms)
    if not parameter.is_contiguous():
        raise ValueError("parameter must be C contiguous")
    if normalized_update.dtype != torch.float32:
        raise ValueError("normalized_update must be float32")
    if indices.dtype != torch.long:
        raise ValueError("indices must be int64")
    if squared_norms.dtype != torch.float32:
        raise ValueError("squared_norms must be float32")
    rows, cols = parameter.shape[-2], parameter.shape[-1]
    batch = _leading(parameter)
    k = normalized_update.shape[-2]
    if normalized_update.numel() != batch * k * cols:
        raise ValueError("parameter and normalized_update batch dimensions must match")
    if indices.numel() != batch * k:
        raise ValueError("indices and normalized_update shapes must match")
    if squared_norms.numel() != batch * 2:
        raise ValueError("squared_norms must contain two values per batch")
    if k == 0 and parameter.numel() != 0:
        raise ValueError("an empty selected update requires an empty parameter shard")
    n = normalized_update.contiguous()
    idx = indices.reshape(batch * k).contiguous() if k > 0 else indices
    sq = squared_norms.contiguous()
    lib = nat.load()
    with torch.cuda.device(device):
        rc = lib.gns_dion3_apply_rows(
            nat.dtype_code(parameter.dtype), batch, rows, cols, k, parameter.data_ptr(),
            n.data_ptr() if n.numel() else None, idx.data_ptr() if k > 0 else None, sq.data_ptr(),
            float(learning_rate), float(weight_decay), float(adjusted_learning_rate), float(epsilon),
            nat.stream_handle(device),
        )
    nat.check(rc, "gns_dion3_apply_rows")


# ------------------------------------------------------------ AdamW / Lion
def _group_check(tensors_by_role: Sequence[Sequence[Tensor]]) -> torch.device:
    first = tensors_by_role[0]
    for role in tensors_by_role:
        if len(role) != len(first):
            raise ValueError("tensor lists must have equal lengths")
        for t, ref in zip(role, first, strict=True):
            if t.numel() != ref.numel():
                raise ValueError("tensor sizes differ within one parameter")
            if not t.is_contiguous():
                raise ValueError("tensors must be contiguous")
        if len({t.dtype for t in role}) > 1:
            raise TypeError("tensors of one role must share a dtype")
    return _require_cuda(*[t for role in tensors_by_role for t in role])


def adamw_step(
    parameters: Sequence[Tensor],
    gradients: Sequence[Tensor],
    exp_avgs: Sequence[Tensor],
    exp_avg_sqs: Sequence[Tensor],
    lr_over_bias_correction1: Sequence[float],
    inverse_sqrt_bias_correction2: Sequence[float],
    beta1: float,
    beta2: float,
    epsilon: float,
    decay: float | None,
) -> None:
    """One multi-tensor AdamW step over a group (muon.py:516-553), in place."""
    if not parameters:
        return
    device = _group_check([parameters, gradients, exp_avgs, exp_avg_sqs])
    count = len(parameters)
    numel = (ctypes.c_int64 * count)(*[t.numel() for t in parameters])
    lr_bc1 = (ctypes.c_float * count)(*[float(v) for v in lr_over_bias_correction1])
    inv_bc2 = (ctypes.c_float * count)(*[float(v) for v in inverse_sqrt_bias_correction2])
    lib = nat.load()
    with torch.cuda.device(device):
        rc = lib.gns_adamw_step(
            count, _ptr_array(parameters), _ptr_array(gradients), _ptr_array(exp_avgs), _ptr_array(exp_avg_sqs),
            numel, nat.dtype_code(parameters[0].dtype), nat.dtype_code(gradients[0].dtype),
            nat.dtype_code(exp_avgs[0].dtype), lr_bc1, inv_bc2, float(beta1), float(beta2), float(1 - beta1),
            float(1 - beta2), float(epsilon),
            float(decay) if decay is not None else 1.0, 1 if decay is not None else 0, nat.stream_handle(device),
        )
    nat.check(rc, "gns_adamw_step")


def lion_step(
    parameters: Sequence[Tensor],
    gradients: Sequence[Tensor],
    buffers: Sequence[Tensor],
    learning_rate: float,
    beta1: float,
    beta2: float,
    decay: float | None,
) -> None:
    """One multi-tensor Lion step over a group (muon.py:555-583), in place."""
    if not parameters:
        return
    device = _group_check([parameters, gradients, buffers])
    count = len(parameters)
    numel = (ctypes.c_int64 * count)(*[t.numel() for t in parameters])
    lib = nat.load()
    with torch.cuda.device(device):
        rc = lib.gns_lion_step(
            count, _ptr_array(parameters), _ptr_array(gradients), _ptr_array(buffers), numel,
            nat.dtype_code(parameters[0].dtype), nat.dtype_code(gradients[0].dtype), nat.dtype_code(buffers[0].dtype),
            float(learning_rate), float(beta1), float(beta2), float(1 - beta1), float(1 - beta2),
            float(decay) if decay is not None else 1.0,
            1 if decay is not None else 0, nat.stream_handle(device),
        )
    nat.check(rc, "gns_lion_step")
