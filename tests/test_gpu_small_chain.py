"""The fused single-kernel chains for small matrices (short side <= 128).

``gns_gram_newton_schulz`` routes non-square matrices with a short side of at
most 128 to one kernel that keeps the Gram-space matrices in shared memory.
It computes the same products in the same order and rounding as the
multi-launch chain (one GEMM launch per product), so the two tactics agree bit
for bit; square matrices up to 128 x 128 run the standard chain in the same
kernel, likewise bit for bit; the multi-launch chain is pinned against the oracle and the reference
goldens elsewhere (test_gpu_api.py, test_gpu_chain.py), and cfg1 (128 x 256
fp32) is checked against the oracle here directly.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from gram_newton_schulz_ampere_b200 import GramNewtonSchulz, StandardNewtonSchulz, _native, ops
from oracle import gns_oracle as O

pytestmark = pytest.mark.gpu

CASES = [
    ((1, 128, 256), torch.float32),  # cfg1
    ((3, 96, 320), torch.bfloat16),
    ((2, 40, 1000), torch.float16),  # rows and columns off the tile grid
    ((2, 300, 72), torch.bfloat16),  # tall
    ((4, 128, 130), torch.float32),
    ((2, 1, 64), torch.bfloat16),  # a single row
    ((1, 64, 3072), torch.bfloat16),  # longest long side routed to the fused kernel
    ((300, 32, 96), torch.bfloat16),  # more matrices than SMs: CTAs loop over the batch
    ((2, 2000, 128), torch.float16),  # tall, full 128-wide short side
]


@pytest.mark.parametrize("resets", [(2,), (), (1, 3)])
@pytest.mark.parametrize("shape,dtype", CASES)
def test_fused_small_chain_equals_multi_launch_chain(cuda_device, shape, dtype, resets):
    gen = torch.Generator(device=cuda_device).manual_seed(sum(shape) + len(resets))
    x = torch.randn(shape, generator=gen, device=cuda_device).to(dtype)
    ns = GramNewtonSchulz(gram_newton_schulz_reset_iterations=resets)
    with ops.small_chain_tactic(False):
        want = ns(x)
    got = ns(x)
    torch.cuda.synchronize(cuda_device)
    assert _native.device_status(clear=True) == 0
    assert got.dtype == dtype and got.shape == x.shape
    assert torch.equal(got, want), (got.float() - want.float()).abs().max().item()


SQUARE_CASES = [
    ((1, 128, 128), torch.float32),
    ((3, 96, 96), torch.bfloat16),
    ((2, 40, 40), torch.float16),  # off the 64-element box grid
    ((200, 64, 64), torch.bfloat16),  # more matrices than SMs
    ((2, 1, 1), torch.float32),
]


@pytest.mark.parametrize("iterations", [5, 2])
@pytest.mark.parametrize("shape,dtype", SQUARE_CASES)
def test_fused_square_chain_equals_multi_launch_chain(cuda_device, shape, dtype, iterations):
    gen = torch.Generator(device=cuda_device).manual_seed(sum(shape) + iterations)
    x = torch.randn(shape, generator=gen, device=cuda_device).to(dtype)
    coefficients = O.polar_express_coefficients()[:iterations]
    for ns in (StandardNewtonSchulz(ns_coefficients=coefficients), GramNewtonSchulz(ns_coefficients=coefficients)):
        with ops.small_chain_tactic(False):
            want = ns(x)
        got = ns(x)
        torch.cuda.synchronize(cuda_device)
        assert _native.device_status(clear=True) == 0
        assert got.dtype == dtype and got.shape == x.shape
        assert torch.equal(got, want), (got.float() - want.float()).abs().max().item()


def test_fused_small_chain_cfg1_matches_oracle(cuda_device):
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(1, 128, 256, generator=gen)
    got = GramNewtonSchulz()(x.to(cuda_device)).cpu().numpy()
    want = O.gram_newton_schulz(x.numpy(), O.polar_express_coefficients(), (2,), 1e-7)
    assert O.relative_error(got, want) < 2e-2
    s = np.linalg.svd(got[0].astype(np.float64), compute_uv=False)
    assert 0.7 < s.min() and s.max() < 1.3


def test_tactic_switch_restores_setting(cuda_device):
    lib = _native.load()
    with ops.small_chain_tactic(False):
        with ops.small_chain_tactic(True):
            assert lib.gns_set_small_chain(1) == 1
        assert lib.gns_set_small_chain(0) == 0
    assert lib.gns_set_small_chain(1) == 1
