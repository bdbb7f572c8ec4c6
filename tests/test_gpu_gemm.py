"""tcgen05 GEMM / symmetric-product parity against a torch fp32 reference.

Mirrors the reference's CUTLASS kernel tests (tests/test_cutlass_ns.py:123-386):
symmetric products are exactly symmetric, partial tiles (40/136/264), NaN
accumulators ignored when beta == 0, the false-symmetry contract, and general
alpha/beta products. Operands are exercised in every storage order the
tensor-core descriptors support (row-major and transposed views).
"""

from __future__ import annotations

import pytest
import torch

from gram_newton_schulz_ampere_b200 import ops

pytestmark = pytest.mark.gpu

# Same tolerances as the reference's tests (tests/test_cutlass_ns.py:68-71).
TOL = {torch.float16: (5e-3, 2e-2), torch.bfloat16: (2e-2, 2e-1)}


def _reference(left, right, acc=None, alpha=1.0, beta=0.0):
    out = alpha * (left.float() @ right.float())
    if acc is not None and beta != 0.0:
        out = out + beta * acc.float()
    return out


def _operand(batch, rows, cols, dtype, device, gen, transposed):
    if transposed:
        return torch.randn(batch, cols, rows, dtype=dtype, device=device, generator=gen).mT
    return torch.randn(batch, rows, cols, dtype=dtype, device=device, generator=gen)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("shape", [(2, 96, 72, 80), (1, 136, 264, 72), (3, 256, 512, 192), (1, 40, 24, 8)])
def test_general_gemm_matches_torch(cuda_device, dtype, a_t, b_t, shape):
    batch, m, n, k = shape
    gen = torch.Generator(device=cuda_device).manual_seed(131 + m + n + k)
    left = _operand(batch, m, k, dtype, cuda_device, gen, a_t)
    right = _operand(batch, k, n, dtype, cuda_device, gen, b_t)
    acc = torch.randn(batch, m, n, dtype=dtype, device=cuda_device, generator=gen)
    out = ops.gemm(left, right, acc, alpha=0.5, beta=0.25)
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(out.float(), _reference(left, right, acc, 0.5, 0.25), rtol=rtol, atol=atol)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("dimension", [40, 136, 264, 1024])
def test_symmetric_gram_rc_partial_tiles(cuda_device, dtype, dimension):
    gen = torch.Generator(device=cuda_device).manual_seed(109 + dimension)
    matrix = torch.randn(2, dimension, 72, dtype=dtype, device=cuda_device, generator=gen)
    out = ops.gemm(matrix, matrix.mT, symmetric=True)
    assert torch.equal(out, out.mT)
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(out.float(), _reference(matrix, matrix.mT), rtol=rtol, atol=atol)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_symmetric_cr_gram(cuda_device, dtype):
    gen = torch.Generator(device=cuda_device).manual_seed(107)
    matrix = torch.randn(2, 192, 128, dtype=dtype, device=cuda_device, generator=gen)
    out = ops.gemm(matrix.mT, matrix, symmetric=True)
    assert torch.equal(out, out.mT)
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(out.float(), _reference(matrix.mT, matrix), rtol=rtol, atol=atol)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_symmetric_rr_with_accumulator(cuda_device, dtype):
    gen = torch.Generator(device=cuda_device).manual_seed(101)
    src = torch.randn(2, 136, 136, dtype=dtype, device=cuda_device, generator=gen)
    left = ((src + src.mT) * 0.5).contiguous()
    src2 = torch.randn(2, 136, 136, dtype=dtype, device=cuda_device, generator=gen)
    acc = ((src2 + src2.mT) * 0.5).contiguous()
    out = ops.gemm(left, left, acc, alpha=0.75, beta=0.25, symmetric=True)
    assert torch.equal(out, out.mT)
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(out.float(), _reference(left, left, acc, 0.75, 0.25), rtol=rtol, atol=atol)


def test_symmetric_beta_zero_ignores_nan_accumulator(cuda_device):
    gen = torch.Generator(device=cuda_device).manual_seed(127)
    src = torch.randn(1, 64, 64, dtype=torch.float16, device=cuda_device, generator=gen)
    left = ((src + src.mT) * 0.5).contiguous()
    acc = torch.full_like(left, float("nan"))
    out = ops.gemm(left, left, acc, beta=0.0, symmetric=True)
    assert torch.isfinite(out).all()
    assert torch.equal(out, out.mT)


def test_false_symmetry_reflects_upper_triangle(cuda_device):
    gen = torch.Generator(device=cuda_device).manual_seed(149)
    left = torch.randn(1, 64, 64, dtype=torch.float16, device=cuda_device, generator=gen)
    right = torch.randn(1, 64, 64, dtype=torch.float16, device=cuda_device, generator=gen)
    expected = left.float() @ right.float()
    out = ops.gemm(left, right, symmetric=True)
    assert torch.equal(out, out.mT)
    torch.testing.assert_close(torch.triu(out.float()), torch.triu(expected), rtol=5e-3, atol=2e-2)
    assert not torch.allclose(out.float(), expected, rtol=5e-3, atol=2e-2)


def test_large_k_and_fp32_output(cuda_device):
    gen = torch.Generator(device=cuda_device).manual_seed(5)
    x = torch.randn(2, 256, 4096, dtype=torch.float16, device=cuda_device, generator=gen) * 0.02
    out = ops.gemm(x, x.mT, symmetric=True, out_dtype=torch.float32)
    assert out.dtype == torch.float32
    assert torch.equal(out, out.mT)
    torch.testing.assert_close(out, x.float() @ x.float().mT, rtol=1e-3, atol=1e-3)


def test_unaligned_rows_are_repacked(cuda_device):
    # 5 x 4 fp16 rows (8-byte pitch) cannot be a TMA operand as-is.
    gen = torch.Generator(device=cuda_device).manual_seed(7)
    a = torch.randn(3, 5, 4, dtype=torch.float16, device=cuda_device, generator=gen)
    out = ops.gemm(a, a.mT, symmetric=True)
    assert torch.equal(out, out.mT)
    torch.testing.assert_close(out.float(), a.float() @ a.float().mT, rtol=5e-3, atol=2e-2)


def test_direct_api_rejects_unsupported_inputs(cuda_device):
    # tests/test_cutlass_ns.py:258-322 of the reference: the Python entry point
    # rejects bad dtypes and shapes before any launch, and the C ABI refuses
    # operands a TMA tile load cannot address (unaligned base, unaligned batch
    # stride) with GNS_ERR_LAYOUT instead of launching.
    from gram_newton_schulz_ampere_b200 import _native as nat

    valid = torch.zeros(1, 64, 64, dtype=torch.float16, device=cuda_device)
    with pytest.raises(TypeError, match="float16 or bfloat16"):
        ops.gemm(valid.float(), valid.float())
    with pytest.raises(TypeError, match="float16 or bfloat16"):
        ops.gemm(valid, valid.to(torch.bfloat16))
    with pytest.raises(ValueError, match="matrix or a batch"):
        ops.gemm(valid[None], valid[None])
    with pytest.raises(ValueError, match="incompatible"):
        ops.gemm(valid, valid[..., :32, :])
    with pytest.raises(ValueError, match="square"):
        ops.gemm(valid, torch.zeros(1, 64, 72, dtype=torch.float16, device=cuda_device), symmetric=True)
    with pytest.raises(ValueError, match="CUDA"):
        ops.gemm(valid.cpu(), valid.cpu())

    lib = nat.load()
    base = torch.randn(1 + 64 * 64, dtype=torch.float16, device=cuda_device)
    unaligned = base[1:].view(1, 64, 64)
    assert unaligned.data_ptr() % 16 != 0
    strided = torch.randn(2 * (64 * 64 + 4), dtype=torch.float16, device=cuda_device)
    odd_batch = torch.as_strided(strided, (2, 64, 64), (64 * 64 + 4, 64, 1))
    out = torch.empty(2, 64, 64, dtype=torch.float16, device=cuda_device)
    for operand, batch in ((unaligned, 1), (odd_batch, 2)):
        s = operand.stride()
        rc = lib.gns_gemm(
            nat.dtype_code(torch.float16), batch, 64, 64, 64,
            operand.data_ptr(), s[0], s[1], s[2], operand.data_ptr(), s[0], s[2], s[1],
            None, 0, 0, 0, out.data_ptr(), nat.dtype_code(torch.float16), 64 * 64, 64,
            1.0, 0.0, 1, nat.stream_handle(cuda_device),
        )
        assert nat.ERROR_NAMES.get(rc) == "layout", (rc, nat.last_error())
        assert "16" in nat.last_error()
        # The Python entry point repacks the same operand and computes the product.
        got = ops.gemm(operand, operand.mT, symmetric=True)
        torch.testing.assert_close(got.float(), operand.float() @ operand.float().mT, rtol=5e-3, atol=5e-2)
    torch.cuda.synchronize(cuda_device)
    assert nat.device_status(clear=True) == 0
