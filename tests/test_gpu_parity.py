"""CUDA path vs the reference (golden fixtures) and vs the oracle.

Tolerances (fp64): energy relative 1e-10, forces max-abs 1e-9, dE/dq,
dE/d(amp,bw2) and virial at the same level; fp32: relative 1e-5.
"""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from sog_b200 import Gaussian, Sog
from tests._cases import CUBES2_CASES, DIRECT_CASES, MESH_CASES, direct_n_dl, grid_ndl, load

pytestmark = pytest.mark.gpu
DEV = "cuda"
F64 = torch.float64
E_TOL, F_TOL = 1e-10, 1e-9


def _t(a, dtype=F64):
    return torch.as_tensor(np.asarray(a), dtype=dtype, device=DEV)


def _rel(a, b):
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-300))


# --------------------------------------------------------------------------
# QuadS and CubeS2 meshes vs the reference itself (mesh_k_convention="reference")
# --------------------------------------------------------------------------
@pytest.mark.parametrize("name", MESH_CASES + CUBES2_CASES)
def test_quads_matches_reference(name):
    c = load(name)
    lam = None if c["lam"] < 0 else float(c["lam"])
    spline = (dict(use_cubes2_fft=True, cubes2_order=int(c["order"])) if name.startswith("cubes2")
              else dict(use_quads_fft=True, quads_order=int(c["order"])))
    def make():
        return Gaussian(n_dl=float(c["n_dl"]), amp=torch.tensor(c["amp"]), bandwidth=torch.tensor(c["bw2"]),
                        kernel_param_mode="internal",
                        remove_self_interaction=bool(c["remove_self"]), charge_neutral_lambda=lam,
                        mesh_k_convention="reference", trainable=True, **spline).to(DEV)
    g = make()
    out = g.compute_bundle(q=_t(c["q"]), r=_t(c["r"]), cell=_t(c["cell"]), batch=_t(c["batch"], torch.long),
                           compute_force=True, compute_virial=True)
    e = out["energy"].detach().cpu().numpy()
    assert _rel(e, c["energy"]) < E_TOL
    assert np.abs(out["forces"].cpu().numpy() - c["forces"]).max() < F_TOL
    assert _rel(out["virial"].cpu().numpy(), c["virial"]) < E_TOL
    # autograd dE/dq, dE/dr and dE/d(amp, bw2) with per-frame weights (dE/dr:
    # the spline-weight derivative for QuadS, the ik force for CubeS2, as the
    # reference's autograd gives them)
    g2 = make()
    q = _t(c["q"]).requires_grad_(True)
    r = _t(c["r"]).requires_grad_(True)
    en = g2(q=q, r=r, cell=_t(c["cell"]), batch=_t(c["batch"], torch.long))
    (en * _t(c["grad_weights"])).sum().backward()
    assert np.abs(q.grad.cpu().numpy().reshape(c["grad_q"].shape) - c["grad_q"]).max() < F_TOL
    assert np.abs(r.grad.cpu().numpy() - c["grad_r"]).max() < F_TOL
    assert _rel(g2.amp.grad.cpu().numpy(), c["grad_amp"]) < E_TOL
    assert _rel(g2.bandwidth.grad.cpu().numpy(), c["grad_bw2"]) < E_TOL


# --------------------------------------------------------------------------
# direct k-sum vs the reference (autograd forces / dq / params)
# --------------------------------------------------------------------------
@pytest.mark.parametrize("name", DIRECT_CASES)
def test_direct_matches_reference(name):
    c = load(name)
    lam = None if c["lam"] < 0 else float(c["lam"])
    g = Gaussian(n_dl=direct_n_dl(c), amp=torch.tensor(c["amp"]), bandwidth=torch.tensor(c["bw2"]),
                 kernel_param_mode="internal", remove_self_interaction=bool(c["remove_self"]),
                 charge_neutral_lambda=lam, trainable=True).to(DEV)
    g.self_coeff = float(c["self_coeff"])
    r = _t(c["r"]).requires_grad_(True)
    q = _t(c["q"]).requires_grad_(True)
    e = g(q=q, r=r, cell=_t(c["cell"]), batch=_t(c["batch"], torch.long))
    assert _rel(e.detach().cpu().numpy(), c["energy"]) < E_TOL
    (e * _t(c["grad_weights"])).sum().backward()
    assert np.abs(-r.grad.cpu().numpy() - c["forces"]).max() < F_TOL
    assert np.abs(q.grad.cpu().numpy().reshape(c["grad_q"].shape) - c["grad_q"]).max() < F_TOL
    if "grad_amp" in c:
        # the reference's default parameters are float32 tensors; the golden
        # gradients were taken through that cast
        tol = 1e-5 if "float32" in str(c["amp_dtype"]) else E_TOL
        assert _rel(g.amp.grad.cpu().numpy(), c["grad_amp"]) < tol
        assert _rel(g.bandwidth.grad.cpu().numpy(), c["grad_bw2"]) < tol


def test_sog_quickstart_config1():
    """README quickstart through Sog: 16 atoms, 12 A, defaults, E + forces."""
    c = load("cfg1_direct")
    model = Sog({"use_atomwise": False}).to(DEV)
    r = _t(c["r"]).requires_grad_(True)
    out = model(positions=r, cell=_t(c["cell"]), latent_charges=_t(c["q"]), compute_force=True)
    assert _rel(out["E_lr"].detach().cpu().numpy(), c["energy"]) < E_TOL
    assert np.abs(out["forces"].cpu().numpy() - c["forces"]).max() < F_TOL
    out["E_lr"].sum().backward()
    assert np.abs(-r.grad.cpu().numpy() - c["forces"]).max() < F_TOL


# --------------------------------------------------------------------------
# B-spline mesh vs the oracle
# --------------------------------------------------------------------------
def _tri(a, b, c, al, be, ga):
    al, be, ga = (math.radians(x) for x in (al, be, ga))
    cx = c * math.cos(be)
    cy = c * (math.cos(al) - math.cos(be) * math.cos(ga)) / math.sin(ga)
    return np.array([[a, 0, 0], [b * math.cos(ga), b * math.sin(ga), 0],
                     [cx, cy, math.sqrt(c * c - cx * cx - cy * cy)]])


def _system(seed, n, cell, nch=1):
    rng = np.random.default_rng(seed)
    r = rng.random((n, 3)) @ cell
    q = rng.standard_normal((n, nch)) * 0.5
    q -= q.mean(axis=0)
    return r, q


def _oracle_bundle(r, q, cells, batch, amp, bw2, spline, order, n_dl, lam=None, remove_self=True,
                   kconv=0):
    grids, ksm = zip(*[grid_ndl(cl, n_dl) for cl in cells])
    return O.bundle(r, q, cells, batch, amp, bw2, solver="mesh", grids=grids, k_sq_max=ksm,
                    spline=spline, order=order, remove_self=remove_self,
                    charge_neutral_lambda=lam, want_virial=True, kconv=kconv)


BSPLINE_CASES = [
    # (order, cell, n, nch, n_dl)
    (4, np.eye(3) * 12.0, 60, 1, 0.7),
    (5, np.eye(3) * 12.0, 60, 1, 0.7),
    (6, np.eye(3) * 12.0, 60, 1, 0.7),
    (6, _tri(12.0, 12.6, 13.5, 80, 95, 105), 70, 2, 0.7),
    (4, _tri(11.0, 11.5, 12.0, 85, 100, 95), 50, 1, 0.9),
    (6, np.diag([12.0, 8.94, 16.0]), 40, 1, 0.64),  # y mesh 27 < 2 L k_max / 2 pi: alias sums
]


@pytest.mark.parametrize("case", range(len(BSPLINE_CASES)))
def test_bspline_matches_oracle(case):
    order, cell, n, nch, n_dl = BSPLINE_CASES[case]
    r, q = _system(case, n, cell, nch)
    bw = np.array([1.5, 2.5, 4.0])
    amp = 1.0 / (bw * math.sqrt(2 * math.pi)) * bw * bw
    ref = _oracle_bundle(r, q, cell[None], np.zeros(n, int), amp, bw * bw, O.BSPLINE, order, n_dl)
    g = Gaussian(n_dl=n_dl, amp=torch.tensor(amp), bandwidth=torch.tensor(bw * bw),
                 kernel_param_mode="internal", use_bspline_fft=True, bspline_order=order,
                 trainable=True).to(DEV)
    qt = _t(q).requires_grad_(True)
    out = g.compute_bundle(q=qt, r=_t(r), cell=_t(cell[None]), compute_force=True, compute_virial=True)
    assert _rel(out["energy"].detach().cpu().numpy(), ref["energy"]) < E_TOL
    assert np.abs(out["forces"].cpu().numpy() - ref["forces"]).max() < F_TOL
    assert _rel(out["virial"].cpu().numpy(), ref["virial"][0]) < E_TOL
    out["energy"].sum().backward()
    assert np.abs(qt.grad.cpu().numpy() - ref["potential"]).max() < F_TOL
    assert _rel(g.amp.grad.cpu().numpy(), ref["grad_amp"].sum(0)) < E_TOL
    assert _rel(g.bandwidth.grad.cpu().numpy(), ref["grad_bw2"].sum(0)) < E_TOL


def test_bspline_multiframe_buckets_and_unsorted_batch():
    """Frames of different mesh sizes (several buckets), atoms interleaved."""
    cells = np.stack([np.eye(3) * 10.0, _tri(11.0, 10.5, 12.0, 88, 95, 100), np.eye(3) * 10.0])
    rs, qs, bs = [], [], []
    for f, cl in enumerate(cells):
        r, q = _system(10 + f, 30 + 7 * f, cl, 2)
        rs.append(r); qs.append(q); bs.append(np.full(len(r), f))
    r, q, batch = np.concatenate(rs), np.concatenate(qs), np.concatenate(bs)
    perm = np.random.default_rng(3).permutation(len(r))
    r, q, batch = r[perm], q[perm], batch[perm]
    bw = np.array([1.2, 2.0, 3.3, 5.0])
    amp = 1.0 / (bw * math.sqrt(2 * math.pi)) * bw * bw
    ref = _oracle_bundle(r, q, cells, batch, amp, bw * bw, O.BSPLINE, 6, 0.8, lam=0.2)
    g = Gaussian(n_dl=0.8, amp=torch.tensor(amp), bandwidth=torch.tensor(bw * bw),
                 kernel_param_mode="internal", use_bspline_fft=True, bspline_order=6,
                 charge_neutral_lambda=0.2).to(DEV)
    qt = _t(q).requires_grad_(True)
    out = g.compute_bundle(q=qt, r=_t(r), cell=_t(cells), batch=_t(batch, torch.long),
                           compute_force=True, compute_virial=True)
    assert _rel(out["energy"].detach().cpu().numpy(), ref["energy"]) < E_TOL
    assert np.abs(out["forces"].cpu().numpy() - ref["forces"]).max() < F_TOL
    assert _rel(out["virial"].cpu().numpy(), ref["virial"]) < E_TOL
    out["energy"].sum().backward()
    assert np.abs(qt.grad.cpu().numpy() - ref["potential"]).max() < F_TOL


def test_quads_physical_convention_matches_oracle_triclinic():
    cell = _tri(12.0, 12.6, 13.5, 80, 95, 105)
    r, q = _system(7, 60, cell)
    bw = np.array([1.5, 2.5, 4.0])
    amp = 1.0 / (bw * math.sqrt(2 * math.pi)) * bw * bw
    ref = _oracle_bundle(r, q, cell[None], np.zeros(60, int), amp, bw * bw, O.QUADS, 6, 0.7)
    g = Gaussian(n_dl=0.7, amp=torch.tensor(amp), bandwidth=torch.tensor(bw * bw),
                 kernel_param_mode="internal", use_quads_fft=True, quads_order=6,
                 mesh_k_convention="physical").to(DEV)
    out = g.compute_bundle(q=_t(q), r=_t(r), cell=_t(cell[None]), compute_force=True)
    assert _rel(out["energy"].detach().cpu().numpy(), ref["energy"]) < E_TOL
    assert np.abs(out["forces"].cpu().numpy() - ref["forces"]).max() < F_TOL


def test_fp32_mode_within_1e5():
    cell = np.eye(3) * 31.0
    r, q = _system(4, 3000, cell)
    bw = 1.2 * 1.62 ** np.arange(12)
    amp = 1.0 / (bw * math.sqrt(2 * math.pi)) * bw * bw
    ref = _oracle_bundle(r, q, cell[None], np.zeros(3000, int), amp, bw * bw, O.BSPLINE, 6, 1.0)
    g = Gaussian(n_dl=1.0, amp=torch.tensor(amp), bandwidth=torch.tensor(bw * bw),
                 kernel_param_mode="internal", use_bspline_fft=True, bspline_order=6).to(DEV)
    out = g.compute_bundle(q=_t(q, torch.float32), r=_t(r, torch.float32),
                           cell=_t(cell[None], torch.float32), compute_force=True)
    assert out["energy"].dtype == torch.float32
    assert _rel(out["energy"].detach().cpu().numpy(), ref["energy"]) < 1e-5
    assert _rel(out["forces"].cpu().numpy(), ref["forces"]) < 1e-5


@pytest.mark.parametrize("L,n_dl", [(12.0, 0.7), (12.0, 1.0)])   # 36^3 (even: half-length x), 25^3 (odd)
def test_fp32_generic_sizes_within_1e5(L, n_dl):
    cell = np.eye(3) * L
    r, q = _system(6, 500, cell, nch=2)
    bw = np.array([1.2, 2.0, 3.5, 6.0])
    amp = 1.0 / (bw * math.sqrt(2 * math.pi)) * bw * bw
    ref = _oracle_bundle(r, q, cell[None], np.zeros(500, int), amp, bw * bw, O.BSPLINE, 6, n_dl)
    g = Gaussian(n_dl=n_dl, amp=torch.tensor(amp), bandwidth=torch.tensor(bw * bw),
                 kernel_param_mode="internal", use_bspline_fft=True, bspline_order=6).to(DEV)
    qt = _t(q, torch.float32).requires_grad_(True)
    out = g.compute_bundle(q=qt, r=_t(r, torch.float32), cell=_t(cell[None], torch.float32),
                           compute_force=True)
    assert _rel(out["energy"].detach().cpu().numpy(), ref["energy"]) < 1e-5
    assert _rel(out["forces"].cpu().numpy(), ref["forces"]) < 1e-5
    # the potential-only field count (dE/dq without forces) takes the same passes
    (gq,) = torch.autograd.grad(g(q=qt, r=_t(r, torch.float32), cell=_t(cell[None], torch.float32)).sum(), qt)
    assert _rel(gq.cpu().numpy(), ref["potential"]) < 1e-5


def test_config2_full_size_bspline6_vs_oracle_and_deterministic():
    c = load("cfg2_quads6")
    amp, bw2 = c["amp"], c["bw2"]
    ref = _oracle_bundle(c["r"], c["q"], c["cell"], c["batch"], amp, bw2, O.BSPLINE, 6, 1.0)
    g = Gaussian(n_dl=1.0, amp=torch.tensor(amp), bandwidth=torch.tensor(bw2),
                 kernel_param_mode="internal", use_bspline_fft=True, bspline_order=6).to(DEV)
    outs = [g.compute_bundle(q=_t(c["q"]), r=_t(c["r"]), cell=_t(c["cell"]), compute_force=True)
            for _ in range(2)]
    assert _rel(outs[0]["energy"].detach().cpu().numpy(), ref["energy"]) < E_TOL
    assert np.abs(outs[0]["forces"].cpu().numpy() - ref["forces"]).max() < F_TOL
    assert torch.equal(outs[0]["energy"], outs[1]["energy"])
    assert torch.equal(outs[0]["forces"], outs[1]["forces"])


def test_status_word_flags_nonfinite_positions():
    from sog_b200 import _lib
    g = Gaussian(n_dl=1.0, use_bspline_fft=True, bspline_order=4).to(DEV)
    r = torch.rand(20, 3, dtype=F64, device=DEV) * 10
    r[3, 1] = float("nan")
    q = torch.rand(20, dtype=F64, device=DEV) - 0.5
    g(q=q, r=r, cell=torch.eye(3, dtype=F64, device=DEV).unsqueeze(0) * 10)
    torch.cuda.synchronize()
    plan = next(iter(_lib.PLANS.plans.values()))
    bits = [p.status() for p in _lib.PLANS.plans.values()]
    assert any(b & 1 for b in bits)


# --------------------------------------------------------------------------
# CubeS2 in the physical wave-vector convention vs the oracle
# --------------------------------------------------------------------------
@pytest.mark.parametrize("order", [4, 6])
def test_cubes2_physical_convention_matches_oracle_triclinic(order):
    rng = np.random.default_rng(40 + order)
    cell = np.array([[13.0, 0.0, 0.0], [1.1, 12.4, 0.0], [-0.9, 0.7, 12.8]])
    n = 300
    r = rng.random((n, 3)) @ cell
    q = rng.normal(size=n)
    q -= q.mean()
    bw = np.geomspace(1.0, 6.0, 5)
    amp = 1.0 / (bw * np.sqrt(2 * np.pi))
    g = Gaussian(n_dl=0.8, amp=torch.tensor(amp), bandwidth=torch.tensor(bw), use_cubes2_fft=True,
                 cubes2_order=order, trainable=False, mesh_k_convention="physical").to(DEV)
    out = g.compute_bundle(q=_t(q), r=_t(r), cell=_t(cell[None]), compute_force=True, compute_virial=True)
    grid, ksm = grid_ndl(cell, 0.8)
    ref = O.bundle(r, q, cell[None], np.zeros(n, dtype=np.int64), g.amp.detach().cpu().numpy(),
                   g.bandwidth.detach().cpu().numpy(), solver="mesh", grids=[grid], k_sq_max=[ksm],
                   spline=O.CUBES2, order=order, want_virial=True, kconv=0)
    assert _rel(out["energy"].cpu().numpy(), ref["energy"]) < E_TOL
    assert np.abs(out["forces"].cpu().numpy() - ref["forces"]).max() < F_TOL
    assert _rel(out["virial"].cpu().numpy(), ref["virial"]) < E_TOL
