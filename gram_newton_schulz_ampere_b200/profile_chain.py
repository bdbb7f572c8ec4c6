"""Runs the native Gram Newton-Schulz chain on a seeded batch, for profilers.

    python -m gram_newton_schulz_ampere_b200.profile_chain [batch] [repeats] [rows] [cols] [dtype]

Defaults: batch 8 of 1024 x 4096 bf16, N(0, 1) * 1e-2 (the cfg2 statistics),
two repeats, so `ncu -s 18 -c 18` captures exactly the second chain's 18 GEMM
launches. `1 2 128 256 f32` runs cfg1 (1 x 128 x 256 fp32, N(0, 1)), whose
chain is one normalisation and one fused small-matrix chain kernel.
"""

from __future__ import annotations

import sys

import torch

from gram_newton_schulz_ampere_b200 import ops
from gram_newton_schulz_ampere_b200.coefficients import polar_express_coefficients

DTYPES = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def main(argv: list[str]) -> int:
    batch = int(argv[0]) if argv else 8
    repeats = int(argv[1]) if len(argv) > 1 else 2
    rows = int(argv[2]) if len(argv) > 2 else 1024
    cols = int(argv[3]) if len(argv) > 3 else 4096
    dtype = DTYPES[argv[4]] if len(argv) > 4 else torch.bfloat16
    scale = 1e-2 if argv[2:3] == [] else 1.0
    gen = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn((batch, rows, cols), generator=gen, device="cuda") * scale).to(dtype)
    coeffs = polar_express_coefficients()
    out = x
    for _ in range(repeats):
        out = ops.newton_schulz_chain(x, coeffs, 1e-7, gram=True, reset_iterations=(2,))
    torch.cuda.synchronize()
    print(f"chain ok: {tuple(out.shape)} x {repeats}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
