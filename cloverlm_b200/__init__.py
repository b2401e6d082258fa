"""cloverlm_b200 -- B200-native (sm_100a) Quartet-II NVFP4 linear layer.

A drop-in for the reference ``quartet2`` package of IST-DASLab/CloverLM:
``cloverlm_b200.linear``, ``cloverlm_b200.quant`` and ``cloverlm_b200.rht``
mirror ``quartet2.linear``, ``quartet2.quant`` and ``quartet2.rht``.
``install_as_quartet2()`` registers this package under the name ``quartet2``
so unmodified callers (``from quartet2.linear import Quartet_II_linear``)
pick it up.

Compute runs only in libq2b.so (hand-written sm_100a CUDA behind the C ABI
of include/q2b.h); there is no CPU or library fallback.
"""
from __future__ import annotations

import sys

from . import _lib  # noqa: F401

__version__ = "0.1.0"


def install_as_quartet2() -> None:
    """Make `import quartet2`, `quartet2.linear`, `quartet2.quant`, `quartet2.rht` resolve to this package."""
    from . import linear, quant, rht
    pkg = sys.modules[__name__]
    sys.modules["quartet2"] = pkg
    sys.modules["quartet2.linear"] = linear
    sys.modules["quartet2.quant"] = quant
    sys.modules["quartet2.rht"] = rht
