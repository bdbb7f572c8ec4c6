"""Polar-express coefficient schedule for Newton-Schulz.

Same constants as the reference (coefficients.py:1-17): five (a, b, c) triples
for the odd polynomial a x + b x^3 + c x^5, each divided by a 1.05 safety factor
raised to the polynomial degree of its term. The numbers are part of the
algorithm's definition, so they must be identical for results to match.
"""

from __future__ import annotations

_RAW_TRIPLES = (
    (8.28721201814563, -23.595886519098837, 17.300387312530933),
    (4.107059111542203, -2.9478499167379106, 0.5448431082926601),
    (3.9486908534822946, -2.908902115962949, 0.5518191394370137),
    (3.3184196573706015, -2.488488024314874, 0.51004894012372),
    (2.300652019954817, -1.6689039845747493, 0.4188073119525673),
)
SAFETY_FACTOR = 1.05


def polar_express_coefficients() -> tuple[tuple[float, float, float], ...]:
    """Returns ((a/s, b/s^3, c/s^5), ...) with s = 1.05."""
    s = SAFETY_FACTOR
    return tuple((a / s, b / s**3, c / s**5) for a, b, c in _RAW_TRIPLES)
