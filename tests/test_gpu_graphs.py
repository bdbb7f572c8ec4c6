"""CUDA-graph replay of Newton-Schulz calls (graphs.CapturedOrthogonalizer):
a replay computes exactly what the eager call computes, for the fused
small-matrix chain, the multi-launch Gram chain and the standard chain, and a
replay after copying new data in equals the eager call on that data."""

from __future__ import annotations

import pytest
import torch

from gram_newton_schulz_ampere_b200 import GramNewtonSchulz, StandardNewtonSchulz
from gram_newton_schulz_ampere_b200.graphs import CapturedOrthogonalizer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(
    "shape,dtype,gram",
    [
        ((1, 128, 256), torch.float32, True),   # fused small-matrix chain
        ((4, 256, 1024), torch.bfloat16, True),  # one GEMM launch per product
        ((3, 384, 160), torch.float16, True),    # tall
        ((2, 96, 96), torch.float32, True),      # square: standard chain
        ((2, 512, 512), torch.bfloat16, False),
    ],
)
def test_replay_equals_eager(cuda_device, shape, dtype, gram):
    gen = torch.Generator(device=cuda_device).manual_seed(sum(shape))
    ns = GramNewtonSchulz() if gram else StandardNewtonSchulz()
    first = torch.randn(shape, generator=gen, device=cuda_device).to(dtype)
    second = torch.randn(shape, generator=gen, device=cuda_device).to(dtype)
    captured = CapturedOrthogonalizer(ns, first)
    out1 = captured(first).clone()
    assert torch.equal(out1, ns(first))
    out2 = captured(second)
    assert torch.equal(out2, ns(second))
    assert out2.data_ptr() == captured.static_output.data_ptr()  # the graph's buffer, reused


def test_replay_rejects_other_shapes(cuda_device):
    x = torch.randn((1, 64, 128), device=cuda_device)
    captured = CapturedOrthogonalizer(GramNewtonSchulz(), x)
    with pytest.raises(ValueError, match="captured for"):
        captured(torch.randn((1, 64, 64), device=cuda_device))
