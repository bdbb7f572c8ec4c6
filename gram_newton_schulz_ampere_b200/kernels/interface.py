"""Backend selection (mirrors kernels/interface.py:16-30 of the reference).

One backend exists here: ``"b200"``. The reference's own backend names
(``"torch"``, ``"cutlass"``, ``"triton"``) are accepted so that code and
optimizer checkpoints written for the reference keep working after the switch:
they select the same B200 backend, with a warning (once per name and process)
that says so. Its outputs follow the reference's torch backend within the
parity tolerance; on B200 the reference itself runs its ``"cutlass"`` name
through torch, because its CUTLASS kernels are built for compute capability 8.
Any other name raises.
"""

from __future__ import annotations

import warnings
from functools import cache

from gram_newton_schulz_ampere_b200.kernels.b200_ns import B200Backend
from gram_newton_schulz_ampere_b200.kernels.protocols import MatrixBackend
from gram_newton_schulz_ampere_b200.optimizer_types import REFERENCE_BACKEND_NAMES


@cache
def select_matrix_backend(name: str) -> MatrixBackend:
    if name == "b200":
        return B200Backend()
    if name in REFERENCE_BACKEND_NAMES:
        warnings.warn(
            f"ns_backend={name!r} is a backend of the Ampere reference package; "
            "gram_newton_schulz_ampere_b200 runs it on its B200 kernels (ns_backend='b200')",
            stacklevel=2,
        )
        return select_matrix_backend("b200")
    raise ValueError(f"Unknown Newton--Schulz kernel backend: {name}")
