"""Second derivatives (double backward) on the GPU.

A force-matching loss differentiates the forces again: F = -dE/dr and the
charge gradients dE/dq are built with create_graph=True and a loss on them is
backpropagated to the charges, positions and kernel parameters.  The
reference gets these derivatives from torch autograd through its direct
k-sum (src/sog/module/gaussian.py:1180-1337); the fixtures hold its values
for the loss  sum(U F) + sum(W F^2) + sum(Z dE/dq) + sum(e_w E), and
likewise through its real-space pair sum for frames without a periodic cell
(gaussian.py:822-845) and through its QuadS mesh (compute_quads_fft,
quads_fft.py:209-326).

Tolerances: fp64 gradients max-abs 1e-9 (relative 1e-10 for the parameter
gradients); parameters created in fp32 by the reference (its defaults) carry
fp32 rounding: relative 1e-5 there.  The B-spline mesh is checked against
central differences of its own first derivatives; CubeS2, whose backward is
the ik force as in the reference, must raise rather than return truncated
second derivatives.
"""
import numpy as np
import pytest
import torch

from sog_b200 import Gaussian, Sog
from tests._cases import direct_n_dl, load

pytestmark = pytest.mark.gpu
DEV = "cuda"
F64 = torch.float64
HVP_CASES = ["hvp_direct_quickstart", "hvp_direct_triclinic_2ch", "hvp_direct_k0_penalty", "hvp_direct_rcut",
             "hvp_realspace_molecule", "hvp_realspace_batch_2ch_keepself", "hvp_realspace_mixed_cells",
             "hvp_quads4_triclinic", "hvp_quads6_2frames_2ch"]


def _t(a, dtype=F64):
    return torch.as_tensor(np.asarray(a), dtype=dtype, device=DEV)


def _rel(a, b):
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-300))


def _model(c):
    lam = None if c["lam"] < 0 else float(c["lam"])
    order = int(c["quads_order"]) if "quads_order" in c else 0
    mesh = dict(use_quads_fft=True, quads_order=order) if order else {}
    g = Gaussian(n_dl=direct_n_dl(c), amp=torch.tensor(c["amp"]), bandwidth=torch.tensor(c["bw2"]),
                 kernel_param_mode="internal", remove_self_interaction=bool(c["remove_self"]),
                 charge_neutral_lambda=lam, trainable=True, **mesh).to(DEV)
    g.self_coeff = float(c["self_coeff"])
    return g


def _loss(g, r, q, c):
    cell = _t(c["cell"]) if int(c.get("has_cell", 1)) else None
    e = g(q=q, r=r, cell=cell, batch=_t(c["batch"], torch.long))
    e_w = _t(c["e_w"])
    gr, gq = torch.autograd.grad((e * e_w).sum(), (r, q), create_graph=True)
    F = -gr
    return (_t(c["U"]) * F).sum() + (_t(c["W"]) * F * F).sum() + (_t(c["Z"]) * gq).sum() + (e * e_w).sum()


@pytest.mark.parametrize("name", HVP_CASES)
def test_second_derivatives_match_reference(name):
    c = load(name)
    g = _model(c)
    r = _t(c["r"]).requires_grad_(True)
    q = _t(c["q"]).requires_grad_(True)
    loss = _loss(g, r, q, c)
    assert abs(float(loss) - float(c["loss"])) <= 1e-10 * max(1.0, abs(float(c["loss"])))
    loss.backward()
    assert np.abs(q.grad.cpu().numpy() - c["grad_q"]).max() < 1e-9
    assert np.abs(r.grad.cpu().numpy() - c["grad_r"]).max() < 1e-9
    if "grad_amp" in c:
        tol = 1e-5 if "float32" in str(c["amp_dtype"]) else 1e-10
        assert _rel(g.amp.grad.cpu().numpy(), c["grad_amp"]) < tol
        assert _rel(g.bandwidth.grad.cpu().numpy(), c["grad_bw2"]) < tol


def _hvp_vs_finite_differences(cells, r0, q0, batch, make, h=1e-4, tol=1e-6, seed=0):
    """H d by double backward against central differences of the GPU's own
    first derivatives along a random direction (charges, positions and
    parameters at once); make(amp, bw2) builds the model."""
    rng = np.random.default_rng(seed)
    amp0, bw0 = np.array([0.6, 1.0, 1.3]), np.array([1.1, 2.4, 4.0])
    dr, dq = rng.standard_normal(r0.shape), rng.standard_normal(q0.shape)
    da, db = rng.standard_normal(3), rng.standard_normal(3)
    nf = int(batch.max()) + 1
    ew = _t(np.linspace(1.0, 0.6, nf))
    bt = _t(batch, torch.long)

    def grads(eps, create_graph=False):
        r = _t(r0 + eps * dr).requires_grad_(True)
        q = _t(q0 + eps * dq).requires_grad_(True)
        g = make(_t(amp0 + eps * da), _t(bw0 + eps * db))
        e = (g(q=q, r=r, cell=None if cells is None else _t(cells), batch=bt) * ew).sum()
        out = torch.autograd.grad(e, (r, q, g.amp, g.bandwidth), create_graph=create_graph)
        return out, (r, q, g)

    (gr, gq, ga, gb), (r, q, g) = grads(0.0, create_graph=True)
    dot = (gr * _t(dr)).sum() + (gq * _t(dq)).sum() + (ga * _t(da)).sum() + (gb * _t(db)).sum()
    hr, hq, ha, hb = torch.autograd.grad(dot, (r, q, g.amp, g.bandwidth))
    (pr, pq, pa, pb), _ = grads(h)
    (mr, mq, ma, mb), _ = grads(-h)
    for an, p, m in ((hr, pr, mr), (hq, pq, mq), (ha, pa, ma), (hb, pb, mb)):
        fd = ((p - m) / (2 * h)).cpu().numpy()
        assert _rel(an.cpu().numpy(), fd) < tol


def test_direct_hvp_matches_finite_differences_of_first_derivatives():
    """Two frames, two channels, neutrality penalty."""
    rng = np.random.default_rng(9)
    cells = np.stack([np.diag([9.0, 9.5, 10.0]), np.array([[8.8, 0, 0], [0.6, 9.2, 0], [-0.4, 0.7, 9.6]])])
    n0, n1 = 12, 15
    r0 = np.concatenate([rng.random((n0, 3)) @ cells[0], rng.random((n1, 3)) @ cells[1]])
    q0 = rng.standard_normal((n0 + n1, 2)) * 0.5
    _hvp_vs_finite_differences(
        cells, r0, q0, np.repeat([0, 1], [n0, n1]),
        lambda a, b: Gaussian(n_dl=1.5, amp=a, bandwidth=b, kernel_param_mode="internal",
                              charge_neutral_lambda=0.2, trainable=True).to(DEV), seed=9)


MESH_HVP_CASES = [
    # (spline kwargs, cells, atoms per frame, n_dl)
    (dict(use_bspline_fft=True, bspline_order=6),
     [np.diag([9.0, 9.5, 10.0]), np.array([[8.8, 0, 0], [0.6, 9.2, 0], [-0.4, 0.7, 9.6]])], (12, 15), 0.9),
    (dict(use_bspline_fft=True, bspline_order=4), [np.array([[9.0, 0, 0], [0.7, 9.4, 0], [-0.5, 0.6, 8.8]])],
     (20,), 0.8),
    # z mesh 25 < 2 L k_max / 2 pi: the B-spline Green function's alias sums
    (dict(use_bspline_fft=True, bspline_order=5), [np.diag([9.0, 8.94, 10.0])], (18,), 0.8),
    (dict(use_quads_fft=True, quads_order=6),
     [np.eye(3) * 9.0, np.array([[8.5, 0, 0], [0.4, 9.6, 0], [-0.3, 0.5, 10.4]])], (14, 11), 1.0),
]


@pytest.mark.parametrize("case", range(len(MESH_HVP_CASES)))
def test_mesh_hvp_matches_finite_differences_of_first_derivatives(case):
    """The B-spline / QuadS mesh Hessian-vector product (charged frames, two
    channels, self term kept, penalty) against central differences of the
    GPU's own exact first derivatives."""
    kw, cells, counts, n_dl = MESH_HVP_CASES[case]
    rng = np.random.default_rng(30 + case)
    r0 = np.concatenate([rng.random((n, 3)) @ cl for n, cl in zip(counts, cells)])
    q0 = rng.standard_normal((sum(counts), 2)) * 0.5 + 0.05
    _hvp_vs_finite_differences(
        np.stack(cells), r0, q0, np.repeat(np.arange(len(counts)), counts),
        lambda a, b: Gaussian(n_dl=n_dl, amp=a, bandwidth=b, kernel_param_mode="internal",
                              remove_self_interaction=False, charge_neutral_lambda=0.2, trainable=True,
                              **kw).to(DEV), seed=40 + case)


def test_realspace_hvp_matches_finite_differences_of_first_derivatives():
    """The pair sum (two molecules, two channels, self term kept)."""
    rng = np.random.default_rng(10)
    n0, n1 = 11, 17
    r0 = rng.standard_normal((n0 + n1, 3)) * 2.0
    q0 = rng.standard_normal((n0 + n1, 2)) * 0.5
    _hvp_vs_finite_differences(
        None, r0, q0, np.repeat([0, 1], [n0, n1]),
        lambda a, b: Gaussian(n_dl=1.5, amp=a, bandwidth=b, kernel_param_mode="internal",
                              remove_self_interaction=False, charge_neutral_lambda=0.2,
                              trainable=True).to(DEV), seed=10)


def test_cubes2_double_backward_raises_instead_of_truncating():
    g = Gaussian(n_dl=1.0, use_cubes2_fft=True, cubes2_order=4).to(DEV)
    r = (torch.rand(30, 3, dtype=F64, device=DEV) * 10).requires_grad_(True)
    q = torch.rand(30, dtype=F64, device=DEV) - 0.5
    e = g(q=q, r=r, cell=torch.eye(3, dtype=F64, device=DEV).unsqueeze(0) * 10)
    (gr,) = torch.autograd.grad(e.sum(), r, create_graph=True)
    with pytest.raises(NotImplementedError):
        (gr * gr).sum().backward()


def test_sog_force_training_step_updates_atomwise_head():
    """A force loss through Sog (Atomwise latent charges, direct k-sum)
    reaches the head's weights: the second derivatives are not dropped."""
    torch.manual_seed(0)
    model = Sog({"n_in": 8, "n_dl": 2.0}).to(DEV).double()
    n = 20
    pos = (torch.rand(n, 3, dtype=F64, device=DEV) * 10).requires_grad_(True)
    desc = torch.randn(n, 8, dtype=F64, device=DEV)
    out = model(positions=pos, cell=torch.eye(3, dtype=F64, device=DEV).unsqueeze(0) * 10, desc=desc)
    (gr,) = torch.autograd.grad(out["E_lr"].sum(), pos, create_graph=True)
    (gr * gr).sum().backward()
    grads = [p.grad for p in model.atomwise.parameters() if p.requires_grad]
    assert any(gg is not None and float(gg.abs().max()) > 0 for gg in grads)
