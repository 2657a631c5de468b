"""Real-space pair sum (frames with cell=None or a singular cell) on the GPU.

Against the reference (golden fixtures made by importing it: energy, and
forces / dE/dq / dE/d(amp, bw2) by autograd through its energy), and against
the oracle at sizes where the kernel splits each atom's partner range over
several tiles.  The reference's test_force_fd_realspace.py finite-difference
check is restated on the product.

Tolerances (fp64): energy relative 1e-10, forces / dE/dq max-abs 1e-9 (scaled
by the largest value where the default parameters make energies ~1e9);
fp32: relative 1e-5.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from sog_b200 import Gaussian, Sog
from tests._cases import REALSPACE_CASES, direct_n_dl, load

pytestmark = pytest.mark.gpu
DEV = "cuda"
F64 = torch.float64
E_TOL, F_TOL = 1e-10, 1e-9


def _t(a, dtype=F64):
    return torch.as_tensor(np.asarray(a), dtype=dtype, device=DEV)


def _rel(a, b):
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-300))


def _gauss(c, trainable=True):
    lam = None if c["lam"] < 0 else float(c["lam"])
    g = Gaussian(n_dl=direct_n_dl(c), amp=torch.tensor(c["amp"]), bandwidth=torch.tensor(c["bw2"]),
                 kernel_param_mode="internal", remove_self_interaction=bool(c["remove_self"]),
                 charge_neutral_lambda=lam, trainable=trainable).to(DEV)
    g.self_coeff = float(c["self_coeff"])
    return g


@pytest.mark.parametrize("name", REALSPACE_CASES)
def test_realspace_matches_reference(name):
    c = load(name)
    g = _gauss(c)
    cell = _t(c["cell"]) if int(c["has_cell"]) else None
    batch = _t(c["batch"], torch.long)
    r = _t(c["r"]).requires_grad_(True)
    q = _t(c["q"]).requires_grad_(True)
    e = g(q=q, r=r, cell=cell, batch=batch)
    assert _rel(e.detach().cpu().numpy(), c["energy"]) < E_TOL
    (e * _t(c["grad_weights"])).sum().backward()
    fs = max(1.0, np.abs(c["forces"]).max())
    assert np.abs(-r.grad.cpu().numpy() - c["forces"]).max() < F_TOL * fs
    qs = max(1.0, np.abs(c["grad_q"]).max())
    assert np.abs(q.grad.cpu().numpy().reshape(c["grad_q"].shape) - c["grad_q"]).max() < F_TOL * qs
    if "grad_amp" in c:
        assert _rel(g.amp.grad.cpu().numpy(), c["grad_amp"]) < E_TOL
        assert _rel(g.bandwidth.grad.cpu().numpy(), c["grad_bw2"]) < E_TOL
    # explicit forces of the bundle agree with the autograd ones
    out = g.compute_bundle(q=_t(c["q"]), r=_t(c["r"]), cell=cell, batch=batch, compute_force=True,
                           compute_virial=True)
    w = c["grad_weights"][c["batch"]]
    assert np.abs(out["forces"].cpu().numpy() * w[:, None] - c["forces"]).max() < F_TOL * fs
    v = out["virial"].cpu().numpy()
    if cell is None:
        assert np.all(v == 0.0)


def test_realspace_batch_none_single_frame():
    """cell=None, batch=None: one frame, energy of shape [1]."""
    c = load("realspace_internal")
    g = _gauss(c)
    e = g(q=_t(c["q"]), r=_t(c["r"]), cell=None, batch=None)
    assert e.shape == (1,)
    assert _rel(e.detach().cpu().numpy(), c["energy"]) < E_TOL


def test_sog_force_matches_fd_in_realspace():
    """Restates the reference's test_force_fd_realspace.py on the product."""
    torch.manual_seed(11)
    model = Sog({"use_atomwise": False, "use_nufft": False, "remove_self_interaction": True,
                 "trainable_kernel": False}).to(DEV)
    r = torch.rand(6, 3, dtype=F64, device=DEV)
    q = torch.rand(6, dtype=F64, device=DEV) - 0.5
    q = q - q.mean()
    out = model(positions=r.clone(), cell=None, latent_charges=q, compute_energy=True,
                compute_force=True)
    force = out["forces"]
    assert force is not None
    eps = 1e-6
    r_p, r_m = r.clone(), r.clone()
    r_p[0, 0] += eps
    r_m[0, 0] -= eps
    e_p = model(positions=r_p, cell=None, latent_charges=q, compute_energy=True)["E_lr"]
    e_m = model(positions=r_m, cell=None, latent_charges=q, compute_energy=True)["E_lr"]
    fd = -((e_p[0] - e_m[0]) / (2.0 * eps))
    assert torch.allclose(force[0, 0], fd, rtol=2e-2, atol=2e-3)


def _molecules(seed, sizes, nch, spread=6.0):
    rng = np.random.default_rng(seed)
    r = np.concatenate([rng.standard_normal((n, 3)) * spread * (n / 1000.0) ** (1 / 3) for n in sizes])
    q = rng.standard_normal((sum(sizes), nch)) * 0.5
    batch = np.concatenate([np.full(n, f) for f, n in enumerate(sizes)])
    return r, q, batch


@pytest.mark.parametrize("sizes,nch,rsi,lam", [
    ([3000], 1, True, None),                        # partner range split over tiles
    ([5000, 7, 1, 700], 3, False, 0.3),             # ragged frames, one of one atom
    ([2500, 2500], 2, True, None),
])
def test_realspace_vs_oracle_split_tiles(sizes, nch, rsi, lam):
    r, q, batch = _molecules(sum(sizes) + nch, sizes, nch)
    bw2 = np.geomspace(0.8, 60.0, 9)
    amp = 1.0 / np.sqrt(2 * np.pi * bw2)
    ref = O.bundle(r, q, None, batch, amp, bw2, solver="direct", remove_self=rsi,
                   charge_neutral_lambda=lam)
    g = Gaussian(n_dl=1.0, amp=torch.tensor(amp), bandwidth=torch.tensor(bw2),
                 kernel_param_mode="internal", remove_self_interaction=rsi,
                 charge_neutral_lambda=lam, trainable=True).to(DEV)
    rt = _t(r).requires_grad_(True)
    qt = _t(q).requires_grad_(True)
    out = g.compute_bundle(q=qt, r=rt, cell=None, batch=_t(batch, torch.long), compute_force=True)
    e = out["energy"]
    assert _rel(e.detach().cpu().numpy(), ref["energy"]) < E_TOL
    fs = max(1.0, np.abs(ref["forces"]).max())
    assert np.abs(out["forces"].cpu().numpy() - ref["forces"]).max() < F_TOL * fs
    e.sum().backward()
    ps = max(1.0, np.abs(ref["potential"]).max())
    assert np.abs(qt.grad.cpu().numpy() - ref["potential"]).max() < F_TOL * ps
    assert _rel(g.amp.grad.cpu().numpy(), ref["grad_amp"].sum(0)) < E_TOL
    assert _rel(g.bandwidth.grad.cpu().numpy(), ref["grad_bw2"].sum(0)) < E_TOL
    # fixed-order sums: a second call is bit-identical
    out2 = g.compute_bundle(q=_t(q), r=_t(r), cell=None, batch=_t(batch, torch.long),
                            compute_force=True)
    assert torch.equal(out2["energy"], e.detach())
    assert torch.equal(out2["forces"], out["forces"])


def test_realspace_fp32_within_1e5():
    r, q, batch = _molecules(5, [4000], 1)
    bw2 = np.geomspace(0.8, 60.0, 9)
    amp = 1.0 / np.sqrt(2 * np.pi * bw2)
    ref = O.bundle(r, q, None, batch, amp, bw2, solver="direct")
    g = Gaussian(n_dl=1.0, amp=torch.tensor(amp), bandwidth=torch.tensor(bw2),
                 kernel_param_mode="internal").to(DEV)
    out = g.compute_bundle(q=_t(q, torch.float32), r=_t(r, torch.float32), cell=None,
                           compute_force=True)
    assert out["energy"].dtype == torch.float32
    assert _rel(out["energy"].detach().cpu().numpy(), ref["energy"]) < 1e-5
    assert _rel(out["forces"].cpu().numpy(), ref["forces"]) < 1e-5


def test_mixed_periodic_and_singular_cells_with_mesh():
    """A mesh-solved periodic frame next to a singular cell in one call."""
    rng = np.random.default_rng(9)
    cell = np.eye(3) * 14.0
    na, nb = 200, 50
    r = np.concatenate([rng.random((na, 3)) @ cell, rng.standard_normal((nb, 3)) * 2.0])
    q = rng.standard_normal((na + nb, 1)) * 0.5
    q[:na] -= q[:na].mean()
    batch = np.concatenate([np.zeros(na, int), np.ones(nb, int)])
    cells = np.stack([cell, np.zeros((3, 3))])
    bw2 = np.geomspace(1.0, 20.0, 5)
    amp = 1.0 / np.sqrt(2 * np.pi * bw2)
    g = Gaussian(n_dl=0.8, amp=torch.tensor(amp), bandwidth=torch.tensor(bw2),
                 kernel_param_mode="internal", use_bspline_fft=True, bspline_order=6).to(DEV)
    out = g.compute_bundle(q=_t(q), r=_t(r), cell=_t(cells), batch=_t(batch, torch.long),
                           compute_force=True)
    rs = O.realspace_solve(r[na:], q[na:], amp, bw2)
    assert _rel(out["energy"][1:].detach().cpu().numpy(), [rs["energy"]]) < E_TOL
    assert np.abs(out["forces"][na:].cpu().numpy() - rs["forces"]).max() < F_TOL
    # the periodic frame is the same as solved alone
    alone = g.compute_bundle(q=_t(q[:na]), r=_t(r[:na]), cell=_t(cell[None]), compute_force=True)
    assert torch.equal(alone["energy"], out["energy"][:1])
    assert torch.equal(alone["forces"], out["forces"][:na])
