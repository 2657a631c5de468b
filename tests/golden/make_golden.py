"""Generate the golden fixtures in this folder by running the reference.

Run where the reference tree is checked out, naming it in $SOG_REFERENCE; the
fixtures are committed so the GPU box never needs it:

    SOG_REFERENCE=<path to the sog checkout> python tests/golden/make_golden.py

Every case stores its inputs and the reference's outputs (fp64).  Sources:
  * QuadS and CubeS2 mesh paths: ``Gaussian(use_quads_fft=True)`` /
    ``Gaussian(use_cubes2_fft=True)`` with
    ``_enable_batched_direct=False`` (the switch the reference's own
    test_batched_mixed.py uses), ``compute_bundle(compute_force=True,
    compute_virial=True)`` -> explicit ik forces and virial
    (src/sog/module/gaussian.py:656-704, quads_fft.py:209-326); dE/dq and
    dE/d(amp, bw2) by autograd through the energy-only call.
  * direct k-sum: ``Sog({"use_atomwise": False})`` / ``Gaussian`` default path
    (gaussian.py:444-548, 1180-1337), derivatives by autograd.
  * real-space pair sum: ``cell=None`` or a singular cell
    (gaussian.py:735-746, 822-845), derivatives by autograd.
  * host logic: ``_resolve_grid`` / ``_next_fft_friendly``
    (cubes2_fft.py:75-188) and the kernel-parameter construction of
    ``Gaussian.__init__`` (gaussian.py:89-279).
Parameters passed to the reference are clones: in raw mode it scales the
caller's amp tensor in place (gaussian.py:236).
"""
from __future__ import annotations

import math
import os
import sys
import warnings

import numpy as np
import torch

REF = os.environ.get("SOG_REFERENCE")
if not REF:
    raise SystemExit("set SOG_REFERENCE to the reference checkout (the folder holding src/sog)")
sys.path.insert(0, os.path.join(REF, "src"))
warnings.filterwarnings("ignore", category=DeprecationWarning)

from sog import Sog  # noqa: E402
from sog.module.gaussian import Gaussian  # noqa: E402
from sog.module.cubes2_fft import _next_fft_friendly, _resolve_grid  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
F64 = torch.float64


def triclinic(a, b, c, alpha, beta, gamma):
    """Cell rows = lattice vectors; a along x, b in the xy plane."""
    al, be, ga = (math.radians(x) for x in (alpha, beta, gamma))
    cx = c * math.cos(be)
    cy = c * (math.cos(al) - math.cos(be) * math.cos(ga)) / math.sin(ga)
    cz = math.sqrt(c * c - cx * cx - cy * cy)
    return torch.tensor([[a, 0.0, 0.0], [b * math.cos(ga), b * math.sin(ga), 0.0],
                         [cx, cy, cz]], dtype=F64)


def params_log(m, lo, hi):
    bw = torch.logspace(math.log10(lo), math.log10(hi), m, dtype=F64)
    return 1.0 / (bw * math.sqrt(2.0 * math.pi)), bw


def run_mesh_case(name, r, q, cell, batch, amp_raw, bw_raw, order, n_dl,
                  remove_self=True, lam=None, autograd=True, family="quads"):
    """QuadS (or CubeS2) through the reference compute_bundle, explicit
    E/F/virial, plus autograd dE/dq, dE/damp, dE/dbw2 of the energy-only path."""
    def make():
        spline = (dict(use_quads_fft=True, quads_order=order) if family == "quads"
                  else dict(use_cubes2_fft=True, cubes2_order=order))
        g = Gaussian(n_dl=n_dl, amp=amp_raw.clone(), bandwidth=bw_raw.clone(),
                     trainable=True, remove_self_interaction=remove_self,
                     charge_neutral_lambda=lam, **spline)
        g._enable_batched_direct = False
        return g
    g = make()
    out = g.compute_bundle(q=q, r=r, cell=cell, batch=batch, compute_force=True,
                           compute_virial=True)
    rec = dict(r=r.numpy(), q=q.numpy(), cell=cell.numpy(), batch=batch.numpy(),
               amp=g.amp.detach().numpy(), bw2=g.bandwidth.detach().numpy(),
               order=order, n_dl=n_dl, remove_self=int(remove_self),
               lam=-1.0 if lam is None else float(lam),
               energy=out["energy"].detach().numpy(), forces=out["forces"].detach().numpy(),
               virial=out["virial"].detach().numpy())
    if autograd:
        g2 = make()
        qg = q.clone().requires_grad_(True)
        rg = r.clone().requires_grad_(True)
        e = g2.compute_bundle(q=qg, r=rg, cell=cell, batch=batch)["energy"]
        w = torch.arange(1, e.shape[0] + 1, dtype=F64)  # distinct per-frame weights
        (e * w).sum().backward()
        rec.update(grad_weights=w.numpy(), grad_q=qg.grad.numpy(), grad_r=rg.grad.numpy(),
                   grad_amp=g2.amp.grad.numpy(), grad_bw2=g2.bandwidth.grad.numpy())
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **rec)
    print(name, rec["energy"])


def run_direct_case(name, r, q, cell, batch, sog_args=None, gauss_kwargs=None):
    """Direct k-sum (the reference default), autograd derivatives."""
    torch.manual_seed(0)
    if sog_args is not None:
        model = Sog(dict(sog_args))
        g = model.gaussian
    else:
        g = Gaussian(**gauss_kwargs)
    rg = r.clone().requires_grad_(True)
    qg = q.clone().requires_grad_(True)
    e = g(q=qg, r=rg, cell=cell, batch=batch)
    w = torch.arange(1, e.shape[0] + 1, dtype=F64)
    (e * w).sum().backward()
    amp_grad = g.amp.grad if isinstance(g.amp, torch.nn.Parameter) and g.amp.grad is not None else None
    bw_grad = (g.bandwidth.grad if isinstance(g.bandwidth, torch.nn.Parameter)
               and g.bandwidth.grad is not None else None)
    rec = dict(r=r.numpy(), q=q.numpy(), cell=cell.numpy(), batch=batch.numpy(),
               amp=g.amp.detach().to(F64).numpy(), bw2=g.bandwidth.detach().to(F64).numpy(),
               amp_dtype=str(g.amp.dtype), self_coeff=float(g.self_coeff),
               remove_self=int(g.remove_self_interaction),
               lam=-1.0 if g.charge_neutral_lambda is None else float(g.charge_neutral_lambda),
               n_dl=-1.0 if g.n_dl is None else float(g.n_dl),
               energy=e.detach().numpy(), grad_weights=w.numpy(),
               forces=(-rg.grad).numpy(), grad_q=qg.grad.numpy())
    if amp_grad is not None:
        rec["grad_amp"] = amp_grad.to(F64).numpy()
        rec["grad_bw2"] = bw_grad.to(F64).numpy()
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **rec)
    print(name, rec["energy"])


def main():
    gen = torch.Generator().manual_seed(2024)

    # ---- QuadS mesh cases ----
    amp3, bw3 = params_log(3, 1.5, 4.0)
    for order in (4, 6):
        n = 40
        cell = torch.eye(3, dtype=F64) * 12.0
        r = torch.rand(n, 3, generator=gen, dtype=F64) * 12.0
        q = torch.rand(n, generator=gen, dtype=F64) - 0.5
        q = q - q.mean()
        run_mesh_case(f"quads{order}_cubic", r, q, cell.unsqueeze(0),
                      torch.zeros(n, dtype=torch.int64), amp3, bw3, order, 0.7)
        cell = triclinic(12.0, 12.6, 13.5, 80.0, 95.0, 105.0)
        s = torch.rand(n, 3, generator=gen, dtype=F64)
        r = s @ cell
        q = torch.randn(n, generator=gen, dtype=F64) * 0.5
        q = q - q.mean()
        run_mesh_case(f"quads{order}_triclinic", r, q, cell.unsqueeze(0),
                      torch.zeros(n, dtype=torch.int64), amp3, bw3, order, 0.7)
    # two frames, two channels, one non-neutral channel (k=0 term) + penalty
    cells = torch.stack([triclinic(9.0, 8.8, 9.4, 85.0, 92.0, 98.0),
                         torch.eye(3, dtype=F64) * 10.0])
    na, nb = 30, 22
    ra = torch.rand(na, 3, generator=gen, dtype=F64) @ cells[0]
    rb = torch.rand(nb, 3, generator=gen, dtype=F64) * 10.0
    q = torch.rand(na + nb, 2, generator=gen, dtype=F64) - 0.5
    q[:, 0] -= q[:, 0].mean()
    batch = torch.cat([torch.zeros(na, dtype=torch.int64), torch.ones(nb, dtype=torch.int64)])
    run_mesh_case("quads6_2frames_2ch", torch.cat([ra, rb]), q, cells, batch, amp3, bw3, 6, 0.6,
                  lam=0.3)
    run_mesh_case("quads4_2frames_keepself", torch.cat([ra, rb]), q[:, :1].clone(), cells, batch,
                  amp3, bw3, 4, 0.6, remove_self=False)

    # config 2 (water-like box) with QuadS-6: 3000 atoms, 31 A, 64^3, M=12
    n = 3000
    r = torch.rand(n, 3, generator=gen, dtype=F64) * 31.0
    q = torch.where(torch.arange(n) % 3 == 0, torch.tensor(-0.8, dtype=F64),
                    torch.tensor(0.4, dtype=F64))
    q = q + 0.05 * torch.randn(n, generator=gen, dtype=F64)
    q = q - q.mean()
    bw = 1.2 * torch.pow(torch.tensor(1.62, dtype=F64), torch.arange(12, dtype=F64))
    amp = 1.0 / (bw * math.sqrt(2.0 * math.pi))
    run_mesh_case("cfg2_quads6", r, q, torch.eye(3, dtype=F64).unsqueeze(0) * 31.0,
                  torch.zeros(n, dtype=torch.int64), amp, bw, 6, 1.0)

    # ---- direct k-sum cases ----
    # config 1: README quickstart
    n = 16
    r = torch.rand(n, 3, generator=gen, dtype=F64) * 12.0
    q = torch.rand(n, generator=gen, dtype=F64) - 0.5
    q = q - q.mean()
    run_direct_case("cfg1_direct", r, q, torch.eye(3, dtype=F64).unsqueeze(0) * 12.0,
                    torch.zeros(n, dtype=torch.int64), sog_args={"use_atomwise": False})
    # two identical triclinic frames, two channels (test_gaussian_triclinic.py:28-72)
    n = 24
    r = torch.rand(n, 3, generator=gen, dtype=F64) * 9.0
    q = torch.rand(n, 2, generator=gen, dtype=F64) - 0.5
    q = q - q.mean(dim=0, keepdim=True)
    cell = torch.tensor([[9.0, 0.0, 0.0], [0.8, 8.5, 0.0], [0.4, 0.6, 8.2]], dtype=F64)
    for rsi in (True, False):
        run_direct_case(f"direct_triclinic_2ch_rsi{int(rsi)}", torch.cat([r, r]), torch.cat([q, q]),
                        torch.stack([cell, cell]),
                        torch.cat([torch.zeros(n, dtype=torch.int64), torch.ones(n, dtype=torch.int64)]),
                        gauss_kwargs=dict(n_dl=2.0, remove_self_interaction=rsi, trainable=True))
    # mixed-nloc batch (test_batched_mixed.py:69-100), raw amp/bw, penalty
    nloc = [3, 5, 4, 4, 6, 3, 5]
    nt = sum(nloc)
    r = torch.randn(nt, 3, generator=gen, dtype=F64) * 2.0
    q = torch.randn(nt, 1, generator=gen, dtype=F64)
    batch = torch.cat([torch.full((k,), i, dtype=torch.int64) for i, k in enumerate(nloc)])
    cell = torch.eye(3, dtype=F64).unsqueeze(0).repeat(len(nloc), 1, 1) * 11.0
    run_direct_case("direct_mixed_batch", r, q, cell, batch,
                    gauss_kwargs=dict(amp=torch.tensor([1.0], dtype=F64),
                                      bandwidth=torch.tensor([0.5], dtype=F64),
                                      charge_neutral_lambda=0.25, trainable=True))
    # fastsog convention (rcut given): amp/bw from w0 and a real-space self term
    n = 20
    r = torch.rand(n, 3, generator=gen, dtype=F64) * 10.0
    q = torch.rand(n, generator=gen, dtype=F64) - 0.5
    q = q - q.mean()
    run_direct_case("direct_rcut", r, q, torch.eye(3, dtype=F64).unsqueeze(0) * 10.0,
                    torch.zeros(n, dtype=torch.int64),
                    sog_args={"use_atomwise": False, "r_cut": 5.0, "m": 8})
    # internal-mode parameters
    run_direct_case("direct_internal", r, q, torch.eye(3, dtype=F64).unsqueeze(0) * 10.0,
                    torch.zeros(n, dtype=torch.int64),
                    gauss_kwargs=dict(n_dl=1.5, amp=torch.tensor([0.7, 1.1, 1.4], dtype=F64),
                                      bandwidth=torch.tensor([1.3, 2.1, 3.4], dtype=F64),
                                      kernel_param_mode="internal", trainable=True))

    # ---- host logic ----
    lens = [(31.0, 31.0, 31.0, 1.0), (40.0, 42.0, 45.0, 0.845), (220.0, 220.0, 220.0, 0.86),
            (12.6, 12.6, 12.6, 1.0), (13.8, 13.8, 13.8, 1.0), (36.8, 36.8, 36.8, 1.0),
            (5.0, 6.0, 7.0, 2.0), (9.0, 8.5, 8.2, 0.7)]
    grid_nd = np.array([_resolve_grid(a, b, c, n_dl=d, cubes2_phi_max=None, r_c=None)
                        for a, b, c, d in lens], dtype=np.float64)
    phis = [(31.0, 31.0, 31.0, 0.1, 5.0), (40.0, 42.0, 45.0, 0.2, 6.0), (12.0, 13.0, 14.0, 0.23, 4.0)]
    grid_phi = np.array([_resolve_grid(a, b, c, n_dl=None, cubes2_phi_max=p, r_c=rc)
                         for a, b, c, p, rc in phis], dtype=np.float64)
    grid_auto = np.array([_resolve_grid(a, b, c, n_dl=None, cubes2_phi_max=None, r_c=rc, b=bb,
                                        spline_order=o)
                          for (a, b, c, _, rc), bb, o in zip(phis, (2.0, 1.8, 1.6), (4, 6, 4))],
                         dtype=np.float64)
    friendly = np.array([[k, _next_fft_friendly(k)] for k in range(1, 600)], dtype=np.int64)
    kw_cases = [
        dict(),
        dict(rcut=5.0),
        dict(rcut=4.0, m=6, b=1.8),
        dict(amp=2.0, bandwidth=torch.tensor([1.0, 2.0, 3.0], dtype=F64)),
        dict(amp=torch.tensor([0.5, 0.6], dtype=F64), bandwidth=torch.tensor([1.5, 2.5], dtype=F64),
             kernel_param_mode="internal"),
        dict(amp=torch.tensor([0.5, 0.6], dtype=F64), bandwidth=torch.tensor([1.5, 2.5], dtype=F64),
             rcut=3.0),
        dict(sigma=1.5, b=1.7, m=5),
    ]
    ctor = {}
    for i, kw in enumerate(kw_cases):
        kwc = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in kw.items()}
        g = Gaussian(**kwc)
        ctor[f"amp_{i}"] = g.amp.detach().to(F64).numpy()
        ctor[f"bw2_{i}"] = g.bandwidth.detach().to(F64).numpy()
        ctor[f"self_coeff_{i}"] = np.array(g.self_coeff)
        ctor[f"dtype_{i}"] = np.array(str(g.amp.dtype))
    np.savez_compressed(os.path.join(OUT, "host_logic.npz"), lens=np.array(lens), grid_nd=grid_nd,
                        phis=np.array(phis), grid_phi=grid_phi, grid_auto=grid_auto,
                        friendly=friendly, n_ctor=len(kw_cases), **ctor)
    print("host_logic written")


def cubes2_cases():
    """CubeS2 mesh path (cubes2_fft.py:925-1133 explicit E/F/virial, and
    Cubes2FFTFunction.backward, cubes2_fft.py:747-869, for dE/dq and
    dE/d(amp, bw2)); its own generator, so the other fixtures stay as they are."""
    gen = torch.Generator().manual_seed(2025)
    amp3, bw3 = params_log(3, 1.5, 4.0)
    for order in (4, 6):
        n = 40
        cell = torch.eye(3, dtype=F64) * 12.0
        r = torch.rand(n, 3, generator=gen, dtype=F64) * 12.0
        q = torch.rand(n, generator=gen, dtype=F64) - 0.5
        q = q - q.mean()
        run_mesh_case(f"cubes2_{order}_cubic", r, q, cell.unsqueeze(0),
                      torch.zeros(n, dtype=torch.int64), amp3, bw3, order, 0.7, family="cubes2")
        cell = triclinic(12.0, 12.6, 13.5, 80.0, 95.0, 105.0)
        s = torch.rand(n, 3, generator=gen, dtype=F64)
        r = s @ cell
        q = torch.randn(n, generator=gen, dtype=F64) * 0.5
        q = q - q.mean()
        run_mesh_case(f"cubes2_{order}_triclinic", r, q, cell.unsqueeze(0),
                      torch.zeros(n, dtype=torch.int64), amp3, bw3, order, 0.7, family="cubes2")
    # two frames, two channels (one non-neutral: k=0 term) and the penalty
    cells = torch.stack([triclinic(9.0, 8.8, 9.4, 85.0, 92.0, 98.0),
                         torch.eye(3, dtype=F64) * 10.0])
    na, nb = 30, 22
    ra = torch.rand(na, 3, generator=gen, dtype=F64) @ cells[0]
    rb = torch.rand(nb, 3, generator=gen, dtype=F64) * 10.0
    q = torch.rand(na + nb, 2, generator=gen, dtype=F64) - 0.5
    q[:, 0] -= q[:, 0].mean()
    batch = torch.cat([torch.zeros(na, dtype=torch.int64), torch.ones(nb, dtype=torch.int64)])
    run_mesh_case("cubes2_4_2frames_2ch", torch.cat([ra, rb]), q, cells, batch, amp3, bw3, 4, 0.6,
                  lam=0.3, family="cubes2")


def run_realspace_case(name, r, q, cell, batch, sog_args=None, gauss_kwargs=None):
    """Non-periodic frames (cell=None, or singular cells mixed with periodic
    ones), energy from ``Gaussian.forward``, derivatives by autograd."""
    torch.manual_seed(0)
    if sog_args is not None:
        g = Sog(dict(sog_args)).gaussian
    else:
        g = Gaussian(**gauss_kwargs)
    rg = r.clone().requires_grad_(True)
    qg = q.clone().requires_grad_(True)
    e = g(q=qg, r=rg, cell=cell, batch=batch)
    w = torch.arange(1, e.shape[0] + 1, dtype=F64)
    (e * w).sum().backward()
    rec = dict(r=r.numpy(), q=q.numpy(), has_cell=int(cell is not None),
               cell=np.zeros((0, 3, 3)) if cell is None else cell.numpy(),
               batch=np.zeros(r.shape[0], dtype=np.int64) if batch is None else batch.numpy(),
               amp=g.amp.detach().to(F64).numpy(), bw2=g.bandwidth.detach().to(F64).numpy(),
               amp_dtype=str(g.amp.dtype), self_coeff=float(g.self_coeff),
               remove_self=int(g.remove_self_interaction),
               lam=-1.0 if g.charge_neutral_lambda is None else float(g.charge_neutral_lambda),
               n_dl=-1.0 if g.n_dl is None else float(g.n_dl),
               energy=e.detach().numpy(), grad_weights=w.numpy(),
               forces=(-rg.grad).numpy(), grad_q=qg.grad.numpy())
    if isinstance(g.amp, torch.nn.Parameter) and g.amp.grad is not None:
        rec["grad_amp"] = g.amp.grad.to(F64).numpy()
        rec["grad_bw2"] = g.bandwidth.grad.to(F64).numpy()
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **rec)
    print(name, rec["energy"])


def realspace_cases():
    """Real-space path; its own generator, so the other fixtures stay as they are."""
    gen = torch.Generator().manual_seed(2026)
    # the reference's test_force_fd_realspace.py configuration: defaults, 6 atoms
    r = torch.rand(6, 3, generator=gen, dtype=F64)
    q = torch.rand(6, generator=gen, dtype=F64) - 0.5
    q = q - q.mean()
    run_realspace_case("realspace_defaults", r, q, None, None,
                       sog_args={"use_atomwise": False, "use_nufft": False,
                                 "remove_self_interaction": True, "trainable_kernel": False})
    # one molecule, internal-mode trainable parameters
    n = 40
    r = torch.rand(n, 3, generator=gen, dtype=F64) * 8.0
    q = torch.rand(n, generator=gen, dtype=F64) - 0.5
    q = q - q.mean()
    run_realspace_case("realspace_internal", r, q, None, None,
                       gauss_kwargs=dict(n_dl=2.0, amp=torch.tensor([0.7, 1.1, 1.4], dtype=F64),
                                         bandwidth=torch.tensor([1.3, 2.1, 3.4], dtype=F64),
                                         kernel_param_mode="internal", trainable=True))
    # three molecules (one of a single atom), interleaved batch ids, two
    # channels, self term kept, neutrality penalty
    nloc = [13, 1, 20]
    batch = torch.cat([torch.full((k,), i, dtype=torch.int64) for i, k in enumerate(nloc)])
    batch = batch[torch.randperm(batch.numel(), generator=gen)]
    nt = sum(nloc)
    r = torch.randn(nt, 3, generator=gen, dtype=F64) * 2.5
    q = torch.rand(nt, 2, generator=gen, dtype=F64) - 0.5
    amp4, bw4 = params_log(4, 1.2, 5.0)
    run_realspace_case("realspace_batch_2ch_keepself", r, q, None, batch,
                       gauss_kwargs=dict(n_dl=2.0, amp=amp4.clone(), bandwidth=bw4.clone(),
                                         remove_self_interaction=False,
                                         charge_neutral_lambda=0.2, trainable=True))
    # a periodic frame (direct k-sum) next to a singular cell (real space)
    na, nb = 18, 15
    cells = torch.stack([torch.tensor([[9.0, 0.0, 0.0], [0.8, 8.5, 0.0], [0.4, 0.6, 8.2]], dtype=F64),
                         torch.zeros(3, 3, dtype=F64)])
    r = torch.cat([torch.rand(na, 3, generator=gen, dtype=F64) @ cells[0],
                   torch.randn(nb, 3, generator=gen, dtype=F64) * 2.0])
    q = torch.rand(na + nb, generator=gen, dtype=F64) - 0.5
    q[:na] -= q[:na].mean()
    batch = torch.cat([torch.zeros(na, dtype=torch.int64), torch.ones(nb, dtype=torch.int64)])
    run_realspace_case("realspace_mixed_cells", r, q, cells, batch,
                       gauss_kwargs=dict(n_dl=2.0, amp=amp4.clone(), bandwidth=bw4.clone(),
                                         trainable=True))


def cfg3_case():
    """Config 3 at full size through the reference QuadS order-4 mesh: 20,000
    atoms in the 40/42/45 A, 80/95/105 degree cell, 96 x 100 x 108 mesh.
    Inputs come from tests/_cases.cfg3_inputs (seeded numpy); the fixture
    stores their digest and the reference's outputs only: explicit E, ik
    forces and virial (quads_fft.py:209-326 via compute_bundle), and autograd
    dE/dq, dE/d(amp, bw2) and dE/dr (the derivative of the spread weights)
    of the energy-only call."""
    sys.path.insert(0, os.path.dirname(os.path.dirname(OUT)))
    from tests._cases import cfg3_inputs, digest
    c = cfg3_inputs()
    r = torch.tensor(c["r"], dtype=F64)
    q = torch.tensor(c["q"], dtype=F64)
    cell = torch.tensor(c["cell"], dtype=F64).unsqueeze(0)
    batch = torch.zeros(r.shape[0], dtype=torch.int64)
    amp_raw = torch.tensor(c["amp_raw"], dtype=F64)
    bw = torch.tensor(c["bw"], dtype=F64)

    def make():
        g = Gaussian(n_dl=c["n_dl"], amp=amp_raw.clone(), bandwidth=bw.clone(), trainable=True,
                     use_quads_fft=True, quads_order=c["order"])
        g._enable_batched_direct = False
        return g
    g = make()
    out = g.compute_bundle(q=q, r=r, cell=cell, batch=batch, compute_force=True,
                           compute_virial=True)
    g2 = make()
    qg = q.clone().requires_grad_(True)
    rg = r.clone().requires_grad_(True)
    e = g2.compute_bundle(q=qg, r=rg, cell=cell, batch=batch)["energy"]
    e.sum().backward()
    rec = dict(digest=np.array(digest(c["r"], c["q"], c["cell"], c["amp_raw"], c["bw"])),
               amp=g.amp.detach().numpy(), bw2=g.bandwidth.detach().numpy(),
               energy=out["energy"].detach().numpy(), forces=out["forces"].detach().numpy(),
               virial=out["virial"].detach().numpy(), grad_q=qg.grad.numpy(),
               grad_r=rg.grad.numpy(), grad_amp=g2.amp.grad.numpy(),
               grad_bw2=g2.bandwidth.grad.numpy())
    np.savez_compressed(os.path.join(OUT, "cfg3_quads4.npz"), **rec)
    print("cfg3_quads4", rec["energy"])


def run_hvp_case(name, r, q, cell, batch, sog_args=None, gauss_kwargs=None, seed=0, mesh_order=0):
    """Second derivatives through the reference's direct k-sum (torch autograd
    with create_graph=True, as a force-matching loss needs them): forces F =
    -dE/dr and charge gradients P = dE/dq built with create_graph=True, then
    loss = sum(U * F) + sum(W * F^2) + sum(Z * P) + sum(e_w * E) with fixed
    seeded weights; the fixture holds d loss / d(q, r, amp, bw2)."""
    torch.manual_seed(0)
    if sog_args is not None:
        g = Sog(dict(sog_args)).gaussian
    else:
        g = Gaussian(**gauss_kwargs)
    if mesh_order:
        g._enable_batched_direct = False   # the reference's QuadS path, as test_batched_mixed.py does
    gen = torch.Generator().manual_seed(seed)
    rg = r.clone().requires_grad_(True)
    qg = q.clone().requires_grad_(True)
    e = g(q=qg, r=rg, cell=cell, batch=batch)
    e_w = torch.arange(1, e.shape[0] + 1, dtype=F64)
    gr, gq = torch.autograd.grad((e * e_w).sum(), (rg, qg), create_graph=True)
    F = -gr
    U = torch.randn(F.shape, generator=gen, dtype=F64)
    W = torch.rand(F.shape, generator=gen, dtype=F64)
    Z = torch.randn(gq.shape, generator=gen, dtype=F64)
    loss = (U * F).sum() + (W * F * F).sum() + (Z * gq).sum() + (e * e_w).sum()
    loss.backward()
    rec = dict(r=r.numpy(), q=q.numpy(), has_cell=int(cell is not None),
               cell=np.zeros((0, 3, 3)) if cell is None else cell.numpy(),
               batch=np.zeros(r.shape[0], dtype=np.int64) if batch is None else batch.numpy(),
               amp=g.amp.detach().to(F64).numpy(), bw2=g.bandwidth.detach().to(F64).numpy(),
               amp_dtype=str(g.amp.dtype), self_coeff=float(g.self_coeff),
               remove_self=int(g.remove_self_interaction),
               lam=-1.0 if g.charge_neutral_lambda is None else float(g.charge_neutral_lambda),
               n_dl=-1.0 if g.n_dl is None else float(g.n_dl), e_w=e_w.numpy(), U=U.numpy(),
               W=W.numpy(), Z=Z.numpy(), loss=loss.detach().numpy(), grad_q=qg.grad.numpy(),
               grad_r=rg.grad.numpy(), quads_order=int(mesh_order))
    if isinstance(g.amp, torch.nn.Parameter) and g.amp.grad is not None:
        rec["grad_amp"] = g.amp.grad.to(F64).numpy()
        rec["grad_bw2"] = g.bandwidth.grad.to(F64).numpy()
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **rec)
    print(name, float(loss))


def hvp_realspace_cases():
    """Second-derivative fixtures of the real-space pair sum (cell=None and a
    singular cell next to a periodic frame); own generator."""
    gen = torch.Generator().manual_seed(2028)
    n = 24
    r = torch.rand(n, 3, generator=gen, dtype=F64) * 7.0
    q = torch.rand(n, generator=gen, dtype=F64) - 0.5
    run_hvp_case("hvp_realspace_molecule", r, q, None, None,
                 gauss_kwargs=dict(n_dl=2.0, amp=torch.tensor([0.7, 1.1, 1.4], dtype=F64),
                                   bandwidth=torch.tensor([1.3, 2.1, 3.4], dtype=F64),
                                   kernel_param_mode="internal", trainable=True), seed=5)
    nloc = [9, 1, 13]
    batch = torch.cat([torch.full((k,), i, dtype=torch.int64) for i, k in enumerate(nloc)])
    batch = batch[torch.randperm(batch.numel(), generator=gen)]
    nt = sum(nloc)
    r = torch.randn(nt, 3, generator=gen, dtype=F64) * 2.5
    q = torch.rand(nt, 2, generator=gen, dtype=F64) - 0.5
    amp4, bw4 = params_log(4, 1.2, 5.0)
    run_hvp_case("hvp_realspace_batch_2ch_keepself", r, q, None, batch,
                 gauss_kwargs=dict(n_dl=2.0, amp=amp4.clone(), bandwidth=bw4.clone(),
                                   remove_self_interaction=False, charge_neutral_lambda=0.2,
                                   trainable=True), seed=6)
    na, nb = 14, 12
    cells = torch.stack([torch.tensor([[9.0, 0.0, 0.0], [0.8, 8.5, 0.0], [0.4, 0.6, 8.2]], dtype=F64),
                         torch.zeros(3, 3, dtype=F64)])
    r = torch.cat([torch.rand(na, 3, generator=gen, dtype=F64) @ cells[0],
                   torch.randn(nb, 3, generator=gen, dtype=F64) * 2.0])
    q = torch.rand(na + nb, generator=gen, dtype=F64) - 0.5
    batch = torch.cat([torch.zeros(na, dtype=torch.int64), torch.ones(nb, dtype=torch.int64)])
    run_hvp_case("hvp_realspace_mixed_cells", r, q, cells, batch,
                 gauss_kwargs=dict(n_dl=2.0, amp=amp4.clone(), bandwidth=bw4.clone(), trainable=True), seed=7)


def hvp_cases():
    """Second-derivative fixtures of the direct k-sum; own generator."""
    gen = torch.Generator().manual_seed(2027)
    # README quickstart box, default (fp32-created) trainable parameters
    n = 16
    r = torch.rand(n, 3, generator=gen, dtype=F64) * 12.0
    q = torch.rand(n, generator=gen, dtype=F64) - 0.5
    q = q - q.mean()
    run_hvp_case("hvp_direct_quickstart", r, q, torch.eye(3, dtype=F64).unsqueeze(0) * 12.0,
                 torch.zeros(n, dtype=torch.int64), sog_args={"use_atomwise": False}, seed=1)
    # two triclinic frames, two channels, internal trainable parameters
    na, nb = 14, 11
    cells = torch.stack([triclinic(9.0, 8.6, 9.3, 84.0, 93.0, 101.0),
                         torch.tensor([[8.5, 0.0, 0.0], [0.4, 9.1, 0.0], [-0.3, 0.5, 8.8]], dtype=F64)])
    r = torch.cat([torch.rand(na, 3, generator=gen, dtype=F64) @ cells[0],
                   torch.rand(nb, 3, generator=gen, dtype=F64) @ cells[1]])
    q = torch.rand(na + nb, 2, generator=gen, dtype=F64) - 0.5
    batch = torch.cat([torch.zeros(na, dtype=torch.int64), torch.ones(nb, dtype=torch.int64)])
    run_hvp_case("hvp_direct_triclinic_2ch", r, q, cells, batch,
                 gauss_kwargs=dict(n_dl=1.6, amp=torch.tensor([0.7, 1.1, 1.4], dtype=F64),
                                   bandwidth=torch.tensor([1.3, 2.1, 3.4], dtype=F64),
                                   kernel_param_mode="internal", trainable=True), seed=2)
    # non-neutral charges (k=0 term), self term kept, neutrality penalty, fastsog r_cut convention
    n = 18
    r = torch.rand(n, 3, generator=gen, dtype=F64) * 10.0
    q = torch.rand(n, generator=gen, dtype=F64) - 0.4
    run_hvp_case("hvp_direct_k0_penalty", r, q, torch.eye(3, dtype=F64).unsqueeze(0) * 10.0,
                 torch.zeros(n, dtype=torch.int64),
                 gauss_kwargs=dict(rcut=5.0, m=6, remove_self_interaction=False, charge_neutral_lambda=0.3,
                                   trainable=True), seed=3)
    # the fastsog convention with the self term removed (self_coeff != 0)
    run_hvp_case("hvp_direct_rcut", r, q - q.mean(), torch.eye(3, dtype=F64).unsqueeze(0) * 10.0,
                 torch.zeros(n, dtype=torch.int64),
                 sog_args={"use_atomwise": False, "r_cut": 5.0, "m": 8}, seed=4)


def hvp_quads_cases():
    """Second-derivative fixtures of the reference's QuadS mesh (torch
    autograd through compute_quads_fft, quads_fft.py:209-326, with
    create_graph=True); own generator."""
    gen = torch.Generator().manual_seed(2029)
    n = 20
    cell = triclinic(9.0, 9.4, 8.8, 82.0, 96.0, 104.0).unsqueeze(0)
    r = torch.rand(n, 3, generator=gen, dtype=F64) @ cell[0]
    q = torch.rand(n, generator=gen, dtype=F64) - 0.5
    q = q - q.mean()
    run_hvp_case("hvp_quads4_triclinic", r, q, cell, torch.zeros(n, dtype=torch.int64),
                 gauss_kwargs=dict(n_dl=1.2, amp=torch.tensor([0.7, 1.1, 1.4], dtype=F64),
                                   bandwidth=torch.tensor([1.3, 2.1, 3.4], dtype=F64),
                                   kernel_param_mode="internal", trainable=True,
                                   use_quads_fft=True, quads_order=4), seed=8, mesh_order=4)
    # two frames of different meshes, two channels, charged (k=0 term), self
    # term kept, neutrality penalty
    na, nb = 16, 13
    cells = torch.stack([torch.eye(3, dtype=F64) * 9.0,
                         torch.tensor([[8.5, 0.0, 0.0], [0.4, 9.6, 0.0], [-0.3, 0.5, 10.4]], dtype=F64)])
    r = torch.cat([torch.rand(na, 3, generator=gen, dtype=F64) @ cells[0],
                   torch.rand(nb, 3, generator=gen, dtype=F64) @ cells[1]])
    q = torch.rand(na + nb, 2, generator=gen, dtype=F64) - 0.4
    batch = torch.cat([torch.zeros(na, dtype=torch.int64), torch.ones(nb, dtype=torch.int64)])
    amp4, bw4 = params_log(4, 1.2, 4.0)
    run_hvp_case("hvp_quads6_2frames_2ch", r, q, cells, batch,
                 gauss_kwargs=dict(n_dl=1.1, amp=amp4.clone(), bandwidth=bw4.clone(), trainable=True,
                                   remove_self_interaction=False, charge_neutral_lambda=0.25,
                                   use_quads_fft=True, quads_order=6), seed=9, mesh_order=6)


if __name__ == "__main__":
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    if sys.argv[1:] == ["hvp"]:
        hvp_cases()
        hvp_realspace_cases()
        hvp_quads_cases()
    elif sys.argv[1:] == ["hvp_quads"]:
        hvp_quads_cases()
    elif sys.argv[1:] == ["cfg3"]:
        cfg3_case()
    elif sys.argv[1:] == ["cubes2"]:
        cubes2_cases()
    elif sys.argv[1:] == ["realspace"]:
        realspace_cases()
    else:
        main()
        cubes2_cases()
        realspace_cases()
