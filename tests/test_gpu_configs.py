"""The named workloads at their full sizes, on the GPU, against the reference
(config 3, QuadS order 4) and the oracle (B-spline meshes): the configurations
the benchmark times, not only small cases.

  * config 3: 20,000 atoms, triclinic 40/42/45 A at 80/95/105 degrees, mesh
    96 x 100 x 108, order 4, E + F + dE/dq (+ dE/d(amp, bw2), virial);
  * the large single system (1,048,576 atoms, 220 A, 512^3 mesh, B-spline 6)
    in fp64 and fp32, and its 1/8-scale sample (131,072 atoms, 110 A, 256^3);
  * the first 64 frames of the batched workload (13 mesh buckets, 25^3-75^3).

Tolerances as everywhere: fp64 energy relative 1e-10, forces / dE/dq max-abs
1e-9, parameter gradients and virial relative 1e-10; fp32 relative 1e-5
(forces relative to the largest force component).
"""
import functools
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from sog_b200 import Gaussian
from tests._cases import (batch_inputs, cfg3_inputs, digest, grid_ndl, large_system_inputs,
                          load)

pytestmark = pytest.mark.gpu
DEV = "cuda"
F64, F32 = torch.float64, torch.float32
E_TOL, F_TOL = 1e-10, 1e-9


def _t(a, dtype=F64):
    return torch.as_tensor(np.asarray(a), dtype=dtype, device=DEV)


def _rel(a, b):
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-300))


def _internal(c):
    bw2 = c["bw"] ** 2
    return c["amp_raw"] * bw2, bw2


def _k0(q, cell, amp, bw2):
    e0, dq0, _, _ = O.k0_correction(np.asarray(q)[:, None], cell, amp, bw2,
                                    norm_factor=14.3996454784255, remove_self=True)
    return e0, dq0[:, 0]


# ---------------------------------------------------------------------------
# config 3 at full size
# ---------------------------------------------------------------------------
def test_config3_full_size_quads4_matches_reference():
    c = cfg3_inputs()
    g_ref = load("cfg3_quads4")
    assert str(g_ref["digest"]) == digest(c["r"], c["q"], c["cell"], c["amp_raw"], c["bw"])

    def make():
        return Gaussian(n_dl=c["n_dl"], amp=torch.tensor(c["amp_raw"]), bandwidth=torch.tensor(c["bw"]),
                        use_quads_fft=True, quads_order=4, trainable=True).to(DEV)
    g = make()
    assert g.mesh_k_convention == "reference"
    out = g.compute_bundle(q=_t(c["q"]), r=_t(c["r"]), cell=_t(c["cell"][None]), compute_force=True,
                           compute_virial=True)
    assert _rel(out["energy"].detach().cpu().numpy(), g_ref["energy"]) < E_TOL
    assert np.abs(out["forces"].cpu().numpy() - g_ref["forces"]).max() < F_TOL
    assert _rel(out["virial"].cpu().numpy(), g_ref["virial"]) < E_TOL
    g2 = make()
    q = _t(c["q"]).requires_grad_(True)
    r = _t(c["r"]).requires_grad_(True)
    g2(q=q, r=r, cell=_t(c["cell"][None])).sum().backward()
    assert np.abs(q.grad.cpu().numpy() - g_ref["grad_q"]).max() < F_TOL
    # the reference's autograd force: derivative of its spread weights
    assert np.abs(r.grad.cpu().numpy() - g_ref["grad_r"]).max() < F_TOL
    assert _rel(g2.amp.grad.cpu().numpy(), g_ref["grad_amp"]) < E_TOL
    assert _rel(g2.bandwidth.grad.cpu().numpy(), g_ref["grad_bw2"]) < E_TOL


def test_config3_full_size_bspline4_matches_oracle():
    c = cfg3_inputs()
    amp, bw2 = _internal(c)
    grid, ksm = grid_ndl(c["cell"], c["n_dl"])
    assert grid == (96, 100, 108)
    ref = O.mesh_solve(c["r"], c["q"], c["cell"], amp, bw2, spline=O.BSPLINE, order=4, nx=grid[0],
                       ny=grid[1], nz=grid[2], k_sq_max=ksm, want_force=True, want_pot=True)
    e0, dq0 = _k0(c["q"], c["cell"], amp, bw2)
    g = Gaussian(n_dl=c["n_dl"], amp=torch.tensor(c["amp_raw"]), bandwidth=torch.tensor(c["bw"]),
                 use_bspline_fft=True, bspline_order=4, trainable=False).to(DEV)
    q = _t(c["q"]).requires_grad_(True)
    out = g.compute_bundle(q=q, r=_t(c["r"]), cell=_t(c["cell"][None]), compute_force=True)
    out["energy"].sum().backward()
    assert _rel(out["energy"].detach().cpu().numpy(), ref["energy"] + e0) < E_TOL
    assert np.abs(out["forces"].cpu().numpy() - ref["forces"]).max() < F_TOL
    assert np.abs(q.grad.cpu().numpy() - (ref["potential"] + dq0)).max() < F_TOL


# ---------------------------------------------------------------------------
# the large single system: full size (the benchmark's workload) and 1/8 scale
# ---------------------------------------------------------------------------
@functools.lru_cache(maxsize=2)
def _large_oracle(natoms, L):
    c = large_system_inputs(natoms, L)
    amp, bw2 = _internal(c)
    grid, ksm = grid_ndl(c["cell"], c["n_dl"])
    ref = O.mesh_solve(c["r"], c["q"], c["cell"], amp, bw2, spline=O.BSPLINE, order=6, nx=grid[0],
                       ny=grid[1], nz=grid[2], k_sq_max=ksm, want_force=True)
    e0, _ = _k0(c["q"], c["cell"], amp, bw2)
    return c, grid, ref["energy"] + e0, ref["forces"]


def _large_gpu(c, dtype):
    g = Gaussian(n_dl=c["n_dl"], amp=torch.tensor(c["amp_raw"], dtype=dtype),
                 bandwidth=torch.tensor(c["bw"], dtype=dtype), use_bspline_fft=True, bspline_order=6,
                 trainable=False).to(DEV)
    r, q, cell = _t(c["r"], dtype), _t(c["q"], dtype), _t(c["cell"][None], dtype)
    return [g.compute_bundle(q=q, r=r, cell=cell, compute_force=True) for _ in range(2)]


@pytest.mark.parametrize("dtype", [F64, F32])
def test_large_system_eighth_scale_matches_oracle(dtype):
    c, grid, e_ref, f_ref = _large_oracle(1 << 17, 110.0)
    assert grid == (256, 256, 256)
    outs = _large_gpu(c, dtype)
    e = outs[0]["energy"].double().cpu().numpy()
    f = outs[0]["forces"].double().cpu().numpy()
    if dtype == F64:
        assert _rel(e, e_ref) < E_TOL
        assert np.abs(f - f_ref).max() < F_TOL
    else:
        assert _rel(e, e_ref) < 1e-5
        assert _rel(f, f_ref) < 1e-5
    assert torch.equal(outs[0]["energy"], outs[1]["energy"])
    assert torch.equal(outs[0]["forces"], outs[1]["forces"])


@pytest.mark.slow
@pytest.mark.parametrize("dtype", [F64, F32])
def test_large_system_full_size_matches_oracle(dtype):
    """1,048,576 atoms on the 512^3 mesh: the 512-point x R2C, y, fused z and
    C2R instantiations and the full-size spread / gather the benchmark times.
    Run to run bit-identical as well."""
    c, grid, e_ref, f_ref = _large_oracle(1 << 20, 220.0)
    assert grid == (512, 512, 512)
    outs = _large_gpu(c, dtype)
    e = outs[0]["energy"].double().cpu().numpy()
    f = outs[0]["forces"].double().cpu().numpy()
    if dtype == F64:
        assert _rel(e, e_ref) < E_TOL
        assert np.abs(f - f_ref).max() < F_TOL
    else:
        assert _rel(e, e_ref) < 1e-5
        assert _rel(f, f_ref) < 1e-5
    assert torch.equal(outs[0]["energy"], outs[1]["energy"])
    assert torch.equal(outs[0]["forces"], outs[1]["forces"])
    del outs
    torch.cuda.empty_cache()


# ---------------------------------------------------------------------------
# batched frames: the first 64 frames of the batched workload, 13 mesh buckets
# ---------------------------------------------------------------------------
def test_batched_frames_64_of_workload_match_oracle():
    b = batch_inputs(64)
    amp, bw2 = _internal(b)
    counts = b["counts"]
    batch = np.repeat(np.arange(len(counts)), counts)
    grids, ksm = zip(*[grid_ndl(cl, b["n_dl"]) for cl in b["cells"]])
    assert len(set(grids)) >= 8
    ref = O.bundle(b["r"], b["q"], b["cells"], batch, amp, bw2, solver="mesh", grids=grids,
                   k_sq_max=ksm, spline=O.BSPLINE, order=6)
    g = Gaussian(n_dl=b["n_dl"], amp=torch.tensor(b["amp_raw"]), bandwidth=torch.tensor(b["bw"]),
                 use_bspline_fft=True, bspline_order=6, trainable=False).to(DEV)
    q = _t(b["q"]).requires_grad_(True)
    out = g.compute_bundle(q=q, r=_t(b["r"]), cell=_t(b["cells"]), batch=_t(batch, torch.long),
                           compute_force=True)
    assert len(g._layout["buckets"]) == len(set(grids))
    out["energy"].sum().backward()
    assert _rel(out["energy"].detach().cpu().numpy(), ref["energy"]) < E_TOL
    assert np.abs(out["forces"].cpu().numpy() - ref["forces"]).max() < F_TOL
    assert np.abs(q.grad.cpu().numpy() - ref["potential"][:, 0]).max() < F_TOL
