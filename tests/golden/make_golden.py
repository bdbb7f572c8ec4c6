"""Generates the golden fixtures in this directory from the REFERENCE implementation.

Run in a container where afrenkai/Gram-Newton-Schulz-Ampere is importable:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference /path/to/reference

It imports the reference package read-only and runs its own torch code on the
CPU (the reference rejects CPU tensors at NewtonSchulz.__call__ and in the Muon
constructor, so the harness calls the built operations directly and bypasses
only the CUDA-placement check of the optimizer). Outputs:

* gns_reference.npz   inputs and reference outputs of gram/standard operations
* dion3_reference.npz reference torch-twin selection / normalisation / update
* muon_reference.npz  reference Muon optimizer steps with an identity orthogonaliser
* baseline_shapes.npz reference outputs at full workload sizes (one 1024 x 4096
  Gram case, one 4096 x 4096 standard case, a 16 x 4096 x 4096 Dion3
  selection); only samples, sketches, singular values, index sets and
  checksums are kept, the inputs are regenerated at test time by
  tests/golden/baseline_inputs.py (``--baseline-shapes`` writes this file alone;
  it takes a few minutes and about 8 GB of host memory)

The fixtures are small (< 3 MB) and committed; nothing at test time reads the
reference tree.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).cpu().numpy()


def gns_cases(ref) -> dict[str, np.ndarray]:
    from gram_newton_schulz_ampere.newton_schulz import GramNewtonSchulz, StandardNewtonSchulz

    out: dict[str, np.ndarray] = {}
    coeffs = np.array(
        __import__("gram_newton_schulz_ampere.coefficients", fromlist=["x"]).polar_express_coefficients(),
        dtype=np.float64,
    )
    out["coefficients"] = coeffs
    cases = [
        # name, shape, dtype, seed, gram, resets
        ("cfg1", (1, 128, 256), torch.float32, 0, True, (2,)),
        ("wide_bf16", (2, 64, 160), torch.bfloat16, 1, True, (2,)),
        ("tall_f16", (2, 200, 72), torch.float16, 2, True, (2,)),
        ("tall_bf16", (1, 256, 96), torch.bfloat16, 3, True, (2,)),
        ("square_f32", (2, 96, 96), torch.float32, 4, True, (2,)),
        ("noreset_bf16", (1, 96, 256), torch.bfloat16, 5, True, ()),
        ("resets13_bf16", (1, 96, 256), torch.bfloat16, 6, True, (1, 3)),
        ("standard_wide_bf16", (2, 80, 200), torch.bfloat16, 7, False, ()),
        ("cfg2_like_bf16", (1, 256, 1024), torch.bfloat16, 8, True, (2,)),
    ]
    names = []
    for name, shape, dtype, seed, gram, resets in cases:
        torch.manual_seed(seed)
        x = torch.randn(shape)
        if name.startswith("cfg2"):
            x = x * 1e-2
        x = x.to(dtype)
        if gram:
            ns = GramNewtonSchulz(ns_backend="torch", ns_compile=False, gram_newton_schulz_reset_iterations=resets)
        else:
            ns = StandardNewtonSchulz(ns_backend="torch", ns_compile=False)
        # NewtonSchulz.__call__ dispatch (newton_schulz.py:308-319) without its CUDA guard.
        op = ns.gram_operation if (ns.gram and shape[-2] != shape[-1]) else ns.standard_operation
        y = op(x).to(dtype)
        out[f"{name}__x"] = to_np(x)
        out[f"{name}__y"] = to_np(y)
        out[f"{name}__meta"] = np.array(
            [{torch.float32: 2, torch.bfloat16: 1, torch.float16: 0}[dtype], int(gram), *([-1] + list(resets))],
            dtype=np.int64,
        )
        names.append(name)
    out["case_names"] = np.array(names)
    return out


def dion3_cases() -> dict[str, np.ndarray]:
    from gram_newton_schulz_ampere.dion3_update import apply_dion3_update, normalize_dion3_rows, select_dion3_rows

    out: dict[str, np.ndarray] = {}
    # Known-answer case of the reference's own test (tests/test_dion3.py:21-69).
    grad = torch.tensor([[1.0, 0.0], [4.0, 4.0], [2.0, 0.0], [0.5, 0.0]])
    mom = torch.zeros(4, 2)
    sel, idx = select_dion3_rows(mom, grad, fraction=0.5, error_feedback_decay=0.5)
    var = torch.zeros(4, 1)
    normed = normalize_dion3_rows(sel, var, idx, muon_beta2=0.9, epsilon=1e-8)
    param = torch.ones(4, 2)
    apply_dion3_update(param, normed, idx, learning_rate=0.1, weight_decay=0.2, adjusted_learning_rate=0.1)
    out["kat__grad"] = to_np(grad)
    out["kat__indices"] = np.sort(idx.numpy())
    out["kat__momentum"] = to_np(mom)
    out["kat__selected"] = to_np(sel)[np.argsort(idx.numpy())]
    out["kat__normalized"] = to_np(normed)[np.argsort(idx.numpy())]
    out["kat__variance"] = to_np(var)
    out["kat__parameter"] = to_np(param)

    # Seeded heavy-tailed case (the Dion3 workload's row-scale statistics, reduced size).
    gen = torch.Generator().manual_seed(4242)
    rows, cols, batch = 64, 48, 2
    scale = torch.exp(torch.randn(batch, rows, 1, generator=gen))
    grad = torch.randn(batch, rows, cols, generator=gen) * 1e-3 * scale
    mom = torch.randn(batch, rows, cols, generator=gen) * 1e-3
    param = torch.randn(batch, rows, cols, generator=gen) * 0.02
    var = torch.rand(batch, rows, 1, generator=gen) * 1e-6
    out["rnd__grad"] = to_np(grad)
    out["rnd__momentum_in"] = to_np(mom)
    out["rnd__parameter_in"] = to_np(param)
    out["rnd__variance_in"] = to_np(var)
    mom_after = mom.clone()
    sel, idx = select_dion3_rows(mom_after, grad, fraction=0.25, error_feedback_decay=0.95)
    order = np.argsort(idx.numpy(), axis=-1)
    out["rnd__indices"] = np.sort(idx.numpy(), axis=-1)
    out["rnd__selected"] = np.take_along_axis(to_np(sel), order[..., None], axis=-2)
    out["rnd__momentum"] = to_np(mom_after)
    var_after = var.clone()
    normed = normalize_dion3_rows(sel, var_after, idx, muon_beta2=0.95, epsilon=1e-8)
    param_after = param.clone()
    apply_dion3_update(param_after, normed, idx, learning_rate=0.01, weight_decay=0.0, adjusted_learning_rate=0.01)
    out["rnd__variance"] = to_np(var_after)
    out["rnd__parameter"] = to_np(param_after)
    out["rnd__normalized"] = np.take_along_axis(to_np(normed), order[..., None], axis=-2)
    return out


def muon_cases() -> dict[str, np.ndarray]:
    from gram_newton_schulz_ampere import muon as muon_mod
    from gram_newton_schulz_ampere.muon import Muon

    class Identity:
        def __call__(self, m: torch.Tensor) -> torch.Tensor:
            return m

    # Bypass only the CUDA placement check so the reference runs on the CPU.
    muon_mod.Muon.validate_cuda_configuration = lambda self: None
    out: dict[str, np.ndarray] = {}
    g1 = torch.tensor([[1.0, 2.0], [3.0, 4.0]])
    g2 = torch.tensor([[2.0, -1.0], [0.5, 3.0]])
    for nesterov in (False, True):
        p = torch.nn.Parameter(torch.zeros(2, 2))
        opt = Muon([p], lr=0.1, momentum=0.5, nesterov=nesterov, adjust_lr=None)
        opt.newton_schulz = Identity()
        for g in (g1, g2):
            p.grad = g.clone()
            opt.step()
        tag = "nesterov" if nesterov else "plain"
        out[f"kat_{tag}__parameter"] = to_np(p)
        out[f"kat_{tag}__momentum"] = to_np(opt.state[p]["momentum_buffer"])
    out["kat__g1"] = to_np(g1)
    out["kat__g2"] = to_np(g2)
    # Decay with base lr, update with spectral-norm-adjusted lr (tests/test_muon.py:128-147).
    p = torch.nn.Parameter(torch.ones(8, 2))
    p.grad = torch.ones_like(p)
    opt = Muon([p], lr=0.1, momentum=0.0, nesterov=False, weight_decay=0.2, adjust_lr="spectral_norm")
    opt.newton_schulz = Identity()
    opt.step()
    out["decay__parameter"] = to_np(p)
    # bf16 parameters, Nesterov, three steps of seeded gradients.
    gen = torch.Generator().manual_seed(77)
    p = torch.nn.Parameter((torch.randn(16, 24, generator=gen) * 0.02).bfloat16())
    out["bf16__p0"] = to_np(p)
    opt = Muon([p], lr=3e-3, momentum=0.95, nesterov=True, weight_decay=0.1, adjust_lr="spectral_norm")
    opt.newton_schulz = Identity()
    grads = []
    for _ in range(3):
        g = (torch.randn(16, 24, generator=gen) * 1e-3).bfloat16()
        grads.append(to_np(g))
        p.grad = g
        opt.step()
    out["bf16__grads"] = np.stack(grads)
    out["bf16__parameter"] = to_np(p)
    out["bf16__momentum"] = to_np(opt.state[p]["momentum_buffer"])
    return out


def baseline_shape_cases() -> dict[str, np.ndarray]:
    """The reference at full workload sizes, on inputs from baseline_inputs.py."""
    sys.path.insert(0, str(HERE))
    import baseline_inputs as B
    from gram_newton_schulz_ampere.dion3_update import select_dion3_rows
    from gram_newton_schulz_ampere.newton_schulz import GramNewtonSchulz

    out: dict[str, np.ndarray] = {}
    ns = GramNewtonSchulz(ns_backend="torch", ns_compile=False)
    for name, make, step in (
        ("gram_1024x4096", B.gram_input, B.GRAM_ROW_STEP),
        ("standard_4096", B.standard_input, B.STANDARD_ROW_STEP),
    ):
        x = make()
        # NewtonSchulz.__call__ dispatch and final cast (newton_schulz.py:296-302) without its CUDA guard.
        square = x.shape[-2] == x.shape[-1]
        y = (ns.standard_operation if square else ns.gram_operation)(x).to(x.dtype)
        y64 = y[0].double()
        out[f"{name}__input_checksum"] = B.input_checksum(x)
        out[f"{name}__rows"] = B.bf16_bits(y[0, ::step])
        out[f"{name}__row_step"] = np.array(step)
        out[f"{name}__sketch"] = (y64 @ B.sketch_matrix(y.shape[-1])).numpy()
        out[f"{name}__singular_values"] = torch.linalg.svdvals(y64.float()).double().numpy()
        print(name, "done", flush=True)

    momentum, gradient = B.dion3_inputs()
    out["dion3_16x4096__input_checksum"] = np.stack((B.input_checksum(momentum), B.input_checksum(gradient)))
    count = int(np.ceil(B.DION3_FRACTION * B.DION3_ROWS))
    selected, indices = select_dion3_rows(momentum, gradient, fraction=B.DION3_FRACTION,
                                          error_feedback_decay=B.DION3_DECAY)
    assert indices.shape == (B.DION3_BATCH, count)
    order = torch.argsort(indices, dim=-1)
    out["dion3_16x4096__indices"] = torch.sort(indices, dim=-1).values.numpy().astype(np.int16)
    out["dion3_16x4096__selected_sums"] = B.per_matrix_sums(
        torch.gather(selected, 1, order[..., None].expand(-1, -1, selected.shape[-1]))
    )
    out["dion3_16x4096__momentum_sums"] = B.per_matrix_sums(momentum)
    # How close the k-th and (k+1)-th row norms came (relative gap): a diagnostic
    # of how near a tie the bit-exact index comparison runs.
    norms = torch.sort(B.dion3_inputs()[0].add_(B.dion3_inputs()[1]).norm(p=1, dim=-1), dim=-1, descending=True).values
    out["dion3_16x4096__boundary_gap"] = ((norms[:, count - 1] - norms[:, count]) / norms[:, count - 1]).double().numpy()
    print("dion3 done", flush=True)
    return out


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default="/root/reference")
    parser.add_argument("--baseline-shapes", action="store_true", help="write baseline_shapes.npz only")
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    import gram_newton_schulz_ampere as ref

    if args.baseline_shapes:
        np.savez_compressed(HERE / "baseline_shapes.npz", **baseline_shape_cases())
        print("baseline_shapes.npz", (HERE / "baseline_shapes.npz").stat().st_size)
        return 0

    np.savez_compressed(HERE / "gns_reference.npz", **gns_cases(ref))
    np.savez_compressed(HERE / "dion3_reference.npz", **dion3_cases())
    np.savez_compressed(HERE / "muon_reference.npz", **muon_cases())
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)
    return 0


if __name__ == "__main__":
    sys.exit(main())
