"""Mesh sizing: the reference's grid rules, restated
(src/sog/module/cubes2_fft.py:33-188).

* phi route   n = ceil(L / (phi * r_c)), k^2_max = pi^2 sum 1/Delta^2
* n_dl route  n = 2 floor(L / n_dl) + 1, k^2_max = (2 pi / n_dl)^2 (deprecated)
* auto        phi from Predescu 2020 Table III, linear in b
Every size is at least ``min_grid`` and rounded up to a 2,3,5-smooth number.
"""
from __future__ import annotations

import math
import warnings
from typing import Dict, Optional, Tuple

PHI_MAX_TABLE: Dict[int, Dict[str, float]] = {
    4: {"b2": 0.23, "b163": 0.065},
    6: {"b2": 0.35, "b163": 0.160},
}
_PHI_B_LO = 1.6297670882677647
_PHI_B_HI = 2.0


def next_fft_friendly(n: int) -> int:
    """Smallest 2,3,5-smooth integer >= n (cubes2_fft.py:180-188)."""
    while True:
        m = n
        for p in (2, 3, 5):
            while m % p == 0:
                m //= p
        if m == 1:
            return n
        n += 1


def compute_phi_max(b: float, spline_order: int = 4) -> float:
    """Table III phi_max, linear in b between the anchors (cubes2_fft.py:49-72)."""
    if spline_order not in PHI_MAX_TABLE:
        raise ValueError(f"No φ_max data for spline order {spline_order}. "
                         f"Available: {list(PHI_MAX_TABLE.keys())}")
    entry = PHI_MAX_TABLE[spline_order]
    lo, hi = entry["b163"], entry["b2"]
    if b <= 0:
        raise ValueError(f"b must be positive, got {b}")
    if b <= _PHI_B_LO:
        return lo
    if b >= _PHI_B_HI:
        return hi
    return lo + (hi - lo) * (b - _PHI_B_LO) / (_PHI_B_HI - _PHI_B_LO)


def compute_grid_from_phi(lx: float, ly: float, lz: float, r_c: float, phi: float,
                          min_grid: int = 8) -> Tuple[int, int, int]:
    if r_c <= 0:
        raise ValueError(f"r_c must be positive for φ-based grid, got {r_c}")
    if phi <= 0:
        raise ValueError(f"φ must be positive, got {phi}")
    d = phi * r_c
    return tuple(next_fft_friendly(max(min_grid, int(math.ceil(l / d)))) for l in (lx, ly, lz))


def resolve_grid(lx: float, ly: float, lz: float, n_dl: Optional[float],
                 cubes2_phi_max: Optional[float], r_c: Optional[float], b: float = 2.0,
                 spline_order: int = 4, min_grid: int = 8) -> Tuple[int, int, int, float]:
    """(nx, ny, nz, k_sq_max) for box row lengths lx, ly, lz (cubes2_fft.py:102-175)."""
    if cubes2_phi_max is not None and n_dl is not None:
        raise ValueError("Cannot specify both `cubes2_phi_max` and `n_dl`. "
                         "Use `cubes2_phi_max` (φ = Δ/r_c, recommended) or `n_dl` (legacy).")
    if cubes2_phi_max is not None:
        if r_c is None or r_c <= 0:
            raise ValueError("r_c (real-space cutoff) is required for φ-based grid sizing. "
                             "Set rcut in Gaussian/Sog constructor.")
        nx, ny, nz = compute_grid_from_phi(lx, ly, lz, r_c, float(cubes2_phi_max), min_grid)
        k = math.pi ** 2 * (1.0 / (lx / nx) ** 2 + 1.0 / (ly / ny) ** 2 + 1.0 / (lz / nz) ** 2)
        return nx, ny, nz, k
    if n_dl is not None:
        warnings.warn("`n_dl` is deprecated. Use `cubes2_phi_max` (φ = Δ/r_c) instead. "
                      "See Predescu 2020 Table III: φ_max=0.23 for CubeS₂ 4th/b=2, "
                      "φ_max=0.065 for b≈1.63.", DeprecationWarning, stacklevel=2)
        dims = []
        for l in (lx, ly, lz):
            nk = max(1, int(math.floor(l / n_dl)))
            dims.append(next_fft_friendly(max(min_grid, 2 * nk + 1)))
        return dims[0], dims[1], dims[2], (2.0 * math.pi / n_dl) ** 2
    phi = compute_phi_max(b, spline_order=spline_order)
    if r_c is None or r_c <= 0:
        raise ValueError("r_c is required for auto φ-based grid (neither cubes2_phi_max "
                         "nor n_dl specified). Set rcut in Gaussian/Sog constructor.")
    nx, ny, nz = compute_grid_from_phi(lx, ly, lz, r_c, phi, min_grid)
    k = math.pi ** 2 * (1.0 / (lx / nx) ** 2 + 1.0 / (ly / ny) ** 2 + 1.0 / (lz / nz) ** 2)
    return nx, ny, nz, k
