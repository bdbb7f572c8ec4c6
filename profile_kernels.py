"""Runs one native kernel family on a seeded input, for ncu captures.

    python profile_kernels.py chain [batch] [repeats] [rows] [cols] [dtype]
    python profile_kernels.py muon [layers] [repeats]
    python profile_kernels.py dion3 [matrices] [repeats]
    python profile_kernels.py adamw [tensors] [repeats]
    python profile_kernels.py lion [tensors] [repeats]

chain: the Gram Newton-Schulz chain on a batch of 1024 x 4096 bf16 N(0, 1) *
1e-2 (default batch 8, two repeats, so `ncu -s 18 -c 18` captures the second
chain's 18 GEMM launches); `chain 1 2 128 256 f32` runs the 1 x 128 x 256 fp32
case (normalisation + the fused small-matrix chain).
muon: momentum (Nesterov) and update passes over the bf16 matrices of
`layers` Llama-3-8B layers (default 1: 7 tensors, 218 M elements, 2.6 GB of
state and gradients), once per repeat.
dion3: row selection (k = 1024) and normalise + apply on `matrices` 4096 x 4096
fp32 matrices (default 4: 268 MB per tensor).
adamw / lion: one multi-tensor step over `tensors` fp32 tensors of 4 M
elements (default 16: 268 MB per state tensor).
Every input is larger than the 126 MB L2, so DRAM counters mean something.
"""

from __future__ import annotations

import sys

import torch

from gram_newton_schulz_ampere_b200 import ops
from gram_newton_schulz_ampere_b200.coefficients import polar_express_coefficients

DTYPES = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
LLAMA_LAYER = ((4096, 4096), (4096, 4096), (1024, 4096), (1024, 4096), (14336, 4096), (14336, 4096), (4096, 14336))


def chain(argv: list[str]) -> str:
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
    return f"chain {tuple(out.shape)} x {repeats}"


def muon(argv: list[str]) -> str:
    layers = int(argv[0]) if argv else 1
    repeats = int(argv[1]) if len(argv) > 1 else 1
    gen = torch.Generator(device="cuda").manual_seed(1)
    shapes = [s for _ in range(layers) for s in LLAMA_LAYER]
    params = [(torch.randn(s, generator=gen, device="cuda") * 0.02).bfloat16() for s in shapes]
    grads = [(torch.randn(s, generator=gen, device="cuda") * 1e-3).bfloat16() for s in shapes]
    moms = [torch.zeros_like(p) for p in params]
    for _ in range(repeats):
        updates = ops.muon_momentum(grads, moms, 0.95, True)
        ops.muon_apply(params, updates, 1.0 - 3e-3 * 0.01, [3e-3] * len(params))
    return f"muon {len(params)} tensors x {repeats}"


def dion3(argv: list[str]) -> str:
    count = int(argv[0]) if argv else 4
    repeats = int(argv[1]) if len(argv) > 1 else 1
    gen = torch.Generator(device="cuda").manual_seed(2)
    shape = (count, 4096, 4096)
    param = torch.randn(shape, generator=gen, device="cuda") * 0.02
    grad = torch.randn(shape, generator=gen, device="cuda") * 1e-3
    grad.mul_(torch.exp(torch.randn((count, 4096, 1), generator=gen, device="cuda")))
    mom = torch.zeros_like(param)
    var = torch.zeros((count, 4096, 1), device="cuda")
    for _ in range(repeats):
        sel, idx = ops.dion3_select_rows(mom, grad, param, 1024, 0.95, 1.0 - 0.01 * 0.01)
        ops.dion3_normalize_apply(param, sel, var, idx, 0.95, 1e-8, 0.01, 0.0, 0.01)
    return f"dion3 {shape} x {repeats}"


def adamw_or_lion(argv: list[str], lion: bool) -> str:
    count = int(argv[0]) if argv else 16
    repeats = int(argv[1]) if len(argv) > 1 else 1
    gen = torch.Generator(device="cuda").manual_seed(3)
    n = 1 << 22
    params = [torch.randn(n, generator=gen, device="cuda") for _ in range(count)]
    grads = [torch.randn(n, generator=gen, device="cuda") for _ in range(count)]
    m = [torch.zeros(n, device="cuda") for _ in range(count)]
    v = [torch.zeros(n, device="cuda") for _ in range(count)]
    for step in range(1, repeats + 1):
        if lion:
            ops.lion_step(params, grads, m, 1e-4, 0.9, 0.99, 1.0 - 1e-4 * 0.1)
        else:
            bc1 = [1e-3 / (1 - 0.9**step)] * count
            bc2 = [1.0 / (1 - 0.95**step) ** 0.5] * count
            ops.adamw_step(params, grads, m, v, bc1, bc2, 0.9, 0.95, 1e-8, 1.0 - 1e-3 * 0.1)
    return f"{'lion' if lion else 'adamw'} {count} x {n} x {repeats}"


def main(argv: list[str]) -> int:
    kind, rest = (argv[0], argv[1:]) if argv else ("chain", [])
    runners = {
        "chain": chain,
        "muon": muon,
        "dion3": dion3,
        "adamw": lambda a: adamw_or_lion(a, False),
        "lion": lambda a: adamw_or_lion(a, True),
    }
    message = runners[kind](rest)
    torch.cuda.synchronize()
    from gram_newton_schulz_ampere_b200 import _native

    status = _native.device_status(clear=True)
    if status != 0:
        print(f"device status {status}")
        return 1
    print(f"{message}: ok")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
