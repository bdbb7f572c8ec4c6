"""Backend selection (mirrors kernels/interface.py:16-30 of the reference).

One backend exists here: ``"b200"``. The reference's own backend names raise a
ValueError that says so, instead of silently running something else.
"""

from __future__ import annotations

from functools import cache

from gram_newton_schulz_ampere_b200.kernels.b200_ns import B200Backend
from gram_newton_schulz_ampere_b200.kernels.protocols import MatrixBackend
from gram_newton_schulz_ampere_b200.optimizer_types import REFERENCE_ONLY_BACKENDS


@cache
def select_matrix_backend(name: str) -> MatrixBackend:
    if name == "b200":
        return B200Backend()
    if name in REFERENCE_ONLY_BACKENDS:
        raise ValueError(
            f"ns_backend={name!r} belongs to the Ampere reference package; "
            "gram_newton_schulz_ampere_b200 provides ns_backend='b200'"
        )
    raise ValueError(f"Unknown Newton--Schulz kernel backend: {name}")
