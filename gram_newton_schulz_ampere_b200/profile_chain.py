"""Runs the native Gram Newton-Schulz chain on a seeded batch, for profilers.

    python -m gram_newton_schulz_ampere_b200.profile_chain [batch] [repeats]

Defaults: batch 8 of 1024 x 4096 bf16, N(0, 1) * 1e-2 (the cfg2 statistics),
two repeats, so `ncu -s 18 -c 18` captures exactly the second chain's 18 GEMM
launches.
"""

from __future__ import annotations

import sys

import torch

from gram_newton_schulz_ampere_b200 import ops
from gram_newton_schulz_ampere_b200.coefficients import polar_express_coefficients


def main(argv: list[str]) -> int:
    batch = int(argv[0]) if argv else 8
    repeats = int(argv[1]) if len(argv) > 1 else 2
    gen = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn((batch, 1024, 4096), generator=gen, device="cuda") * 1e-2).to(torch.bfloat16)
    coeffs = polar_express_coefficients()
    out = x
    for _ in range(repeats):
        out = ops.newton_schulz_chain(x, coeffs, 1e-7, gram=True, reset_iterations=(2,))
    torch.cuda.synchronize()
    print(f"chain ok: {tuple(out.shape)} x {repeats}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
