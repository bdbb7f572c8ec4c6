"""B200-native (sm_100a) Gram Newton-Schulz orthogonalisation with Muon and Dion3.

Drop-in for the public API of afrenkai/Gram-Newton-Schulz-Ampere with
``ns_backend="b200"``: ``GramNewtonSchulz``, ``StandardNewtonSchulz``, ``Muon``
and ``Dion3`` keep their constructor signatures and call semantics, and every
product, normalisation and optimizer-state pass runs in the hand-written
kernels of ``lib/libgns_b200.so`` (C ABI: ``include/gns_b200.h``).
"""

from gram_newton_schulz_ampere_b200.dion3 import Dion3 as Dion3
from gram_newton_schulz_ampere_b200.muon import Muon as Muon
from gram_newton_schulz_ampere_b200.newton_schulz import GramNewtonSchulz as GramNewtonSchulz
from gram_newton_schulz_ampere_b200.newton_schulz import StandardNewtonSchulz as StandardNewtonSchulz

__all__ = ["Dion3", "GramNewtonSchulz", "Muon", "StandardNewtonSchulz"]
