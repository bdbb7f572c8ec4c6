"""torch.compile over the orthogonaliser and the GEMM primitive.

Inside a traced region the native calls are the custom ops
``gns_b200::newton_schulz_chain`` and ``gns_b200::gemm``, so a compiled region
holds them without a graph break (``fullgraph=True`` fails on a break) and runs
the same kernels: the results equal eager calls bit for bit. ``aot_eager``
traces through AOTAutograd without generating code for the surrounding ops.
"""

from __future__ import annotations

import pytest
import torch

from gram_newton_schulz_ampere_b200 import GramNewtonSchulz, StandardNewtonSchulz, ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(2, 96, 200), (3, 320, 192), (2, 256, 256), (4, 64, 300)])
def test_compiled_orthogonaliser_matches_eager(cuda_device, shape):
    torch._dynamo.reset()
    gen = torch.Generator(device=cuda_device).manual_seed(12)
    x = torch.randn(shape, generator=gen, device=cuda_device).bfloat16()
    ns = GramNewtonSchulz()
    want = ns(x)
    compiled = torch.compile(lambda t: ns(t) * 1.0, backend="aot_eager", fullgraph=True)
    assert torch.equal(compiled(x), want)
    standard = StandardNewtonSchulz()
    compiled_standard = torch.compile(lambda t: standard(t), backend="aot_eager", fullgraph=True)
    assert torch.equal(compiled_standard(x), standard(x))


def test_compiled_gemm_matches_eager(cuda_device):
    torch._dynamo.reset()
    gen = torch.Generator(device=cuda_device).manual_seed(13)
    a = torch.randn(2, 192, 320, generator=gen, device=cuda_device).half()
    c = torch.randn(2, 192, 192, generator=gen, device=cuda_device).half()

    def f(left: torch.Tensor, acc: torch.Tensor) -> torch.Tensor:
        gram = ops.gemm(left, left.mT, symmetric=True)
        return ops.gemm(gram, gram, acc, alpha=0.5, beta=2.0, symmetric=True, out_dtype=torch.float32)

    compiled = torch.compile(f, backend="aot_eager", fullgraph=True)
    assert torch.equal(compiled(a, c), f(a, c))


def test_custom_ops_pass_opcheck(cuda_device):
    gen = torch.Generator(device=cuda_device).manual_seed(14)
    x = torch.randn(2, 96, 200, generator=gen, device=cuda_device).bfloat16()
    coeffs = [float(v) for triple in GramNewtonSchulz().coefficients for v in triple]
    torch.library.opcheck(torch.ops.gns_b200.newton_schulz_chain.default, (x, coeffs, 1e-7, True, [2], torch.bfloat16))
    a = torch.randn(2, 64, 128, generator=gen, device=cuda_device).half()
    b = torch.randn(2, 128, 96, generator=gen, device=cuda_device).half()
    torch.library.opcheck(torch.ops.gns_b200.gemm.default, (a, b, None, 1.0, 0.0, False, None))
