"""Shared helpers for the parity tests: golden-case loading and grid sizing
written out independently of the product (cubes2_fft.py:142-161 n_dl route)."""
import math
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

MESH_CASES = ["quads4_cubic", "quads6_cubic", "quads4_triclinic", "quads6_triclinic",
              "quads6_2frames_2ch", "quads4_2frames_keepself", "cfg2_quads6"]
CUBES2_CASES = ["cubes2_4_cubic", "cubes2_4_triclinic", "cubes2_6_cubic", "cubes2_6_triclinic",
                "cubes2_4_2frames_2ch"]
REALSPACE_CASES = ["realspace_defaults", "realspace_internal", "realspace_batch_2ch_keepself",
                   "realspace_mixed_cells"]
DIRECT_CASES = ["cfg1_direct", "direct_triclinic_2ch_rsi1", "direct_triclinic_2ch_rsi0",
                "direct_mixed_batch", "direct_rcut", "direct_internal"]


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def friendly(n):
    while True:
        m = n
        for p in (2, 3, 5):
            while m % p == 0:
                m //= p
        if m == 1:
            return n
        n += 1


def grid_ndl(cell, n_dl, min_grid=8):
    lens = np.linalg.norm(np.asarray(cell).reshape(3, 3), axis=1)
    dims = [friendly(max(min_grid, 2 * max(1, int(math.floor(l / n_dl))) + 1)) for l in lens]
    return tuple(dims), (2.0 * math.pi / n_dl) ** 2


def direct_nk(cell, n_dl):
    lens = np.linalg.norm(np.asarray(cell).reshape(3, 3), axis=1)
    return [max(1, int(l / n_dl)) for l in lens]


def direct_n_dl(case):
    if case["n_dl"] > 0:
        return float(case["n_dl"])
    bw_min = float(np.min(case["bw2"]))
    kmax = math.sqrt(2.0 * math.log(1.0 / 1e-5) / max(bw_min, 1e-30))
    return 2.0 * math.pi / max(kmax, 1e-30)
