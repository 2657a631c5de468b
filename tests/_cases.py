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


# ---------------------------------------------------------------------------
# named workloads at full size (seeded numpy inputs; the fixtures store a
# digest of the inputs so a changed generator fails loudly)
# ---------------------------------------------------------------------------
def triclinic(a, b, c, alpha, beta, gamma):
    """Cell rows = lattice vectors; a along x, b in the xy plane."""
    al, be, ga = (math.radians(x) for x in (alpha, beta, gamma))
    cx = c * math.cos(be)
    cy = c * (math.cos(al) - math.cos(be) * math.cos(ga)) / math.sin(ga)
    return np.array([[a, 0.0, 0.0], [b * math.cos(ga), b * math.sin(ga), 0.0],
                     [cx, cy, math.sqrt(c * c - cx * cx - cy * cy)]])


def cfg3_inputs(seed=3):
    """Triclinic cell: 20,000 atoms, a/b/c = 40/42/45 A at 80/95/105 degrees,
    uniform fractional coordinates, neutral N(0, 0.5) charges, 8 Gaussians
    with bandwidths log-spaced 1-20 A and raw amplitudes 1/(bw sqrt(2 pi));
    n_dl = 0.845 gives the 96 x 100 x 108 mesh; order 4."""
    rng = np.random.default_rng(seed)
    cell = triclinic(40.0, 42.0, 45.0, 80.0, 95.0, 105.0)
    n = 20000
    r = rng.random((n, 3)) @ cell
    q = rng.standard_normal(n) * 0.5
    q -= q.mean()
    bw = np.logspace(0.0, math.log10(20.0), 8)
    amp_raw = 1.0 / (bw * math.sqrt(2.0 * math.pi))
    return dict(r=r, q=q, cell=cell, amp_raw=amp_raw, bw=bw, n_dl=0.845, order=4)


def large_system_inputs(natoms, L, seed=0):
    """Large single system (and its scaled-down samples): atoms uniform in a
    cubic box of edge L, neutral N(0, 0.6) charges, 12 Gaussians with
    bandwidths log-spaced 1.2-60 A and raw amplitudes, n_dl = 0.86, order 6.
    The same generator as bench.py's workload."""
    rng = np.random.default_rng(seed)
    r = rng.random((natoms, 3)) * L
    q = rng.standard_normal(natoms) * 0.6
    q -= q.mean()
    bw = np.logspace(math.log10(1.2), math.log10(60.0), 12)
    amp_raw = 1.0 / (bw * math.sqrt(2.0 * math.pi))
    return dict(r=r, q=q, cell=np.eye(3) * L, amp_raw=amp_raw, bw=bw, n_dl=0.86, order=6)


def batch_inputs(nframes=512, seed=0):
    """Batched mixed frames: sizes U{200..5000}, cubic cells at 0.1 atoms/A^3,
    uniform positions, U(-1, 1) charges neutral per frame, 12 Gaussians
    bw 1.2 * 1.62^m with raw amplitudes, n_dl = 1.0, order 6.  The same
    generator as bench.py's batched workload (its first `nframes` frames)."""
    rng = np.random.default_rng(seed)
    ns = rng.integers(200, 5001, 512)
    rs, qs, cells = [], [], []
    for n in ns:
        L = (n / 0.1) ** (1.0 / 3.0)
        rs.append(rng.random((n, 3)) * L)
        qq = rng.uniform(-1.0, 1.0, n)
        qs.append(qq - qq.mean())
        cells.append(np.eye(3) * L)
    bw = 1.2 * 1.62 ** np.arange(12)
    amp_raw = 1.0 / (bw * math.sqrt(2.0 * math.pi))
    ns = [int(n) for n in ns[:nframes]]
    tot = sum(ns)
    return dict(counts=ns, r=np.concatenate(rs)[:tot], q=np.concatenate(qs)[:tot],
                cells=np.stack(cells)[:nframes], amp_raw=amp_raw, bw=bw, n_dl=1.0, order=6)


def digest(*arrays):
    import hashlib
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(np.asarray(a, dtype=np.float64)).tobytes())
    return h.hexdigest()
