"""The long-axis sharded Gram chain's native pieces on one GPU.

The ranks of ``orthogonalize_long_axis_sharded`` are simulated in one process:
the matrix is split along its long axis, each piece goes through the B200
backend's per-shard calls, and the cross-rank sums are plain torch additions in
fp32 (what the NCCL all-reduce computes). The assembled result is compared with
the oracle's restatement of the sharded chain and with the fused single-GPU
chain, both at the 2e-2 relative Frobenius bar of the whole-chain tests.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from gram_newton_schulz_ampere_b200 import ops
from gram_newton_schulz_ampere_b200.kernels.b200_ns import B200Backend
from oracle import gns_oracle as O

pytestmark = pytest.mark.gpu

REL_TOL = 2e-2
COEFFS = O.polar_express_coefficients()


def _simulate_ranks(shards, tall, resets, eps=1e-7):
    be = B200Backend()
    sumsq = sum(be.frobenius_sumsq(s) for s in shards)
    xs = [be.frobenius_scale(s, sumsq, eps) for s in shards]

    def gram(parts):
        return sum(be.gram_partial(x, tall) for x in parts)

    n = len(COEFFS)
    g = gram(xs)
    begin = 0
    q = None
    for end in sorted({i for i in resets if 0 < i < n}) + [n]:
        q = be.gram_iterations(g, COEFFS, begin, end)
        if end < n:
            xs = [be.apply_polynomial(q, x, tall, torch.float16) for x in xs]
            g = gram(xs)
        begin = end
    return [be.apply_polynomial(q, x, tall, shards[0].dtype) for x in xs]


@pytest.mark.parametrize(
    "shape,splits,dtype,resets",
    [
        ((2, 128, 512), (256, 256), torch.bfloat16, (2,)),
        ((1, 96, 392), (200, 192), torch.float32, (2,)),
        ((2, 640, 160), (320, 160, 160), torch.bfloat16, (2,)),
        ((1, 64, 264), (136, 128), torch.float16, (1, 3)),
        ((2, 256, 1024), (512, 512), torch.bfloat16, ()),
    ],
)
def test_sharded_chain_matches_oracle_and_fused(cuda_device, shape, splits, dtype, resets):
    gen = torch.Generator().manual_seed(sum(shape) + len(splits))
    x = torch.randn(shape, generator=gen).to(dtype)
    tall = shape[-2] > shape[-1]
    axis = -2 if tall else -1
    host_shards = list(torch.split(x, list(splits), dim=axis))
    shards = [s.to(cuda_device) for s in host_shards]
    got = torch.cat(_simulate_ranks(shards, tall, resets), dim=axis)
    assert got.dtype == dtype and got.shape == x.shape
    expected = np.concatenate(
        O.long_axis_sharded_gram_newton_schulz([s.float().numpy() for s in host_shards], tall, COEFFS, resets),
        axis=axis,
    )
    err = O.relative_error(got.float().cpu().numpy(), expected)
    assert err < REL_TOL, f"vs oracle: {err:.3e}"
    fused = ops.newton_schulz_chain(x.to(cuda_device), COEFFS, 1e-7, gram=True, reset_iterations=resets)
    err = O.relative_error(got.float().cpu().numpy(), fused.float().cpu().numpy())
    assert err < REL_TOL, f"vs fused chain: {err:.3e}"


def test_frobenius_pieces(cuda_device):
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(3, 72, 200, generator=gen).to(torch.bfloat16)
    xd = x.to(cuda_device)
    be = B200Backend()
    sumsq = be.frobenius_sumsq(xd)
    want = x.double().square().sum(dim=(-2, -1))
    torch.testing.assert_close(sumsq.cpu().double(), want, rtol=1e-5, atol=0)
    scaled = be.frobenius_scale(xd, sumsq, 1e-7)
    assert scaled.dtype == torch.float16 and scaled.shape == x.shape
    ref = (x.float() / (want.float().sqrt()[:, None, None] + 1e-7)).half()
    torch.testing.assert_close(scaled.cpu(), ref, rtol=1e-3, atol=6e-8)
    empty = be.frobenius_sumsq(torch.empty(2, 8, 0, device=cuda_device, dtype=torch.float32))
    assert torch.equal(empty.cpu(), torch.zeros(2))


@pytest.mark.parametrize("begin,end", [(0, 2), (2, 5), (0, 5), (3, 4)])
def test_gram_iterations_match_oracle(cuda_device, begin, end):
    gen = torch.Generator().manual_seed(begin * 10 + end)
    x = O.normalize(torch.randn(2, 96, 256, generator=gen).numpy(), 1e-7)
    g = O.baddbmm(None, x, np.swapaxes(x, -1, -2))
    expected = O.gram_iterations(g, COEFFS, begin, end)
    got = ops.gram_iterations(torch.from_numpy(g).to(cuda_device), COEFFS, begin, end)
    assert got.dtype == torch.float16 and got.shape == g.shape
    err = O.relative_error(got.float().cpu().numpy(), expected)
    assert err < REL_TOL, f"{err:.3e}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_scale_matches_torch_division_bit_for_bit(cuda_device, dtype):
    """fp16(x / (sqrt(s) + eps)) equals torch's IEEE division exactly (the kernel
    divides with one correctly rounded reciprocal and a remainder correction)."""
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(4, 96, 264, generator=gen) * torch.logspace(-6, 3, 264)
    x = x.to(dtype).to(cuda_device)
    sumsq = (torch.rand(4, generator=gen) * torch.tensor([1e-9, 1.0, 37.0, 4e6])).to(cuda_device)
    eps = 1e-7
    got = ops.frobenius_scale(x, sumsq, eps)
    want = (x.float() / (sumsq.sqrt()[:, None, None] + eps)).half()
    assert torch.equal(got.contiguous(), want)
