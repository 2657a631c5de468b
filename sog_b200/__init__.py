"""sog_b200 — SOG's Gaussian reciprocal-space solver on B200 (sm_100a).

Drop-in for ``sog.Sog`` / ``sog.module.Gaussian`` of the reference package;
all solves run in the CUDA library ``sog_b200/_lib/libsog_b200.so`` through the
C ABI declared in ``include/sog_b200.h``.
"""
from .gaussian import Gaussian
from .grid import next_fft_friendly, resolve_grid
from .heads import BEC, Atomwise
from .sog import Sog

__all__ = ["Sog", "Gaussian", "Atomwise", "BEC", "resolve_grid", "next_fft_friendly"]
