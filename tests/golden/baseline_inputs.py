"""Seeded inputs of the full-size parity cases (tests/golden/baseline_shapes.npz).

The fixtures keep only the reference's outputs (row samples, sketches, singular
values, index sets and checksums); the inputs are regenerated here, at test
time, from torch's CPU generator, which produces the same values on every host
running the same torch version. ``input_checksum`` is stored beside each case so
a test can prove that it regenerated the input the reference consumed.

Cases:
* ``gram_1024x4096``: one 1024 x 4096 bf16 matrix, N(0, 1) * 1e-2 (the batched
  Gram Newton-Schulz workload's matrix shape and value distribution).
* ``standard_4096``: one 4096 x 4096 bf16 matrix, N(0, 1) * 1e-3 (the Muon
  q/o bucket of a Llama-3-8B parameter set, which NewtonSchulz.__call__ routes
  to the standard iteration, newton_schulz.py:308-318).
* ``dion3_16x4096``: 16 x 4096 x 4096 fp32 gradients N(0, 1e-3) times a
  per-row lognormal(sigma = 1) scale, momentum N(0, 1e-3), fraction 0.25
  (k = 1024 rows per matrix), error-feedback decay 0.95.
"""

from __future__ import annotations

import numpy as np
import torch

GRAM_SEED, STANDARD_SEED, DION3_SEED, SKETCH_SEED = 20240, 20241, 20242, 20243
SKETCH_COLUMNS = 16
GRAM_ROW_STEP = 16
STANDARD_ROW_STEP = 64
DION3_BATCH, DION3_ROWS, DION3_COLS = 16, 4096, 4096
DION3_FRACTION, DION3_DECAY = 0.25, 0.95


def gram_input() -> torch.Tensor:
    gen = torch.Generator().manual_seed(GRAM_SEED)
    return (torch.randn((1, 1024, 4096), generator=gen) * 1e-2).to(torch.bfloat16)


def standard_input() -> torch.Tensor:
    gen = torch.Generator().manual_seed(STANDARD_SEED)
    return (torch.randn((1, 4096, 4096), generator=gen) * 1e-3).to(torch.bfloat16)


def dion3_inputs() -> tuple[torch.Tensor, torch.Tensor]:
    """(momentum, gradient), each [16, 4096, 4096] fp32."""
    gen = torch.Generator().manual_seed(DION3_SEED)
    scale = torch.exp(torch.randn((DION3_BATCH, DION3_ROWS, 1), generator=gen))
    gradient = torch.randn((DION3_BATCH, DION3_ROWS, DION3_COLS), generator=gen) * 1e-3
    gradient.mul_(scale)
    momentum = torch.randn((DION3_BATCH, DION3_ROWS, DION3_COLS), generator=gen) * 1e-3
    return momentum, gradient


def sketch_matrix(cols: int) -> torch.Tensor:
    """A fixed Gaussian [cols, 16] test matrix: ||(A - B) R|| / ||B R|| estimates the
    relative Frobenius error of the whole matrix from 16 columns."""
    gen = torch.Generator().manual_seed(SKETCH_SEED)
    return torch.randn((cols, SKETCH_COLUMNS), generator=gen, dtype=torch.float64)


def input_checksum(x: torch.Tensor) -> np.ndarray:
    """(sum, sum |x|, sum x^2) in float64 over the whole tensor."""
    d = x.double()
    return np.array([d.sum().item(), d.abs().sum().item(), (d * d).sum().item()], dtype=np.float64)


def per_matrix_sums(x: torch.Tensor) -> np.ndarray:
    """[batch, 2]: float64 sum and sum of |x| of each matrix."""
    d = x.double().flatten(1)
    return torch.stack((d.sum(1), d.abs().sum(1)), dim=1).numpy()


def bf16_bits(x: torch.Tensor) -> np.ndarray:
    return x.contiguous().to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
