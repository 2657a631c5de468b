"""The oracle itself, pinned: golden fixtures from the reference and the
reference's own compiled spline header (oracle/_ref)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._cases import (CUBES2_CASES, DIRECT_CASES, MESH_CASES, REALSPACE_CASES, direct_n_dl,
                          direct_nk, grid_ndl, load)


def _mesh_case_vs_oracle(name, spline):
    c = load(name)
    cells = c["cell"].reshape(-1, 3, 3)
    grids, ksm = zip(*[grid_ndl(cl, float(c["n_dl"])) for cl in cells])
    lam = None if c["lam"] < 0 else float(c["lam"])
    res = O.bundle(c["r"], c["q"], cells, c["batch"], c["amp"], c["bw2"], solver="mesh",
                   grids=grids, k_sq_max=ksm, spline=spline, order=int(c["order"]),
                   remove_self=bool(c["remove_self"]), charge_neutral_lambda=lam,
                   want_virial=True, kconv=1)
    return c, res


@pytest.mark.parametrize("name", MESH_CASES + CUBES2_CASES)
def test_oracle_mesh_matches_reference(name):
    c, res = _mesh_case_vs_oracle(name, O.CUBES2 if name.startswith("cubes2") else O.QUADS)
    e_ref = c["energy"]
    assert np.allclose(res["energy"], e_ref, rtol=1e-12, atol=1e-13 * np.abs(e_ref).max())
    assert np.abs(res["forces"] - c["forces"]).max() < 1e-11
    assert np.abs(res["virial"] - c["virial"]).max() < 1e-11 * max(1.0, np.abs(c["virial"]).max())
    w = c["grad_weights"][c["batch"]]
    q = c["q"] if c["q"].ndim == 2 else c["q"][:, None]
    gq = (res["potential"] * w[:, None]).reshape(q.shape)
    assert np.abs(gq - c["grad_q"].reshape(q.shape)).max() < 1e-11
    ga = (res["grad_amp"] * c["grad_weights"][:, None]).sum(0)
    gb = (res["grad_bw2"] * c["grad_weights"][:, None]).sum(0)
    assert np.allclose(ga, c["grad_amp"], rtol=1e-10, atol=1e-12)
    assert np.allclose(gb, c["grad_bw2"], rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("name", DIRECT_CASES)
def test_oracle_direct_matches_reference(name):
    c = load(name)
    cells = c["cell"].reshape(-1, 3, 3)
    n_dl = direct_n_dl(c)
    nks = [direct_nk(cl, n_dl) for cl in cells]
    ksm = [(2.0 * np.pi / n_dl) ** 2] * len(cells)
    lam = None if c["lam"] < 0 else float(c["lam"])
    res = O.bundle(c["r"], c["q"], cells, c["batch"], c["amp"], c["bw2"], solver="direct",
                   nks=nks, k_sq_max=ksm, remove_self=bool(c["remove_self"]),
                   self_coeff=float(c["self_coeff"]), charge_neutral_lambda=lam)
    e_ref = c["energy"]
    assert np.allclose(res["energy"], e_ref, rtol=1e-12, atol=1e-13 * np.abs(e_ref).max())
    w = c["grad_weights"][c["batch"]]
    assert np.abs(res["forces"] * w[:, None] - c["forces"]).max() < 1e-11
    q = c["q"] if c["q"].ndim == 2 else c["q"][:, None]
    gq = res["potential"] * w[:, None]
    assert np.abs(gq - c["grad_q"].reshape(q.shape)).max() < 1e-11
    if "grad_amp" in c:
        ga = (res["grad_amp"] * c["grad_weights"][:, None]).sum(0)
        gb = (res["grad_bw2"] * c["grad_weights"][:, None]).sum(0)
        # reference parameters live in fp32 when created by default (gaussian.py:162-171)
        tol = 1e-5 if "float32" in str(c["amp_dtype"]) else 1e-10
        assert np.allclose(ga, c["grad_amp"], rtol=tol, atol=tol * np.abs(ga).max())
        assert np.allclose(gb, c["grad_bw2"], rtol=tol, atol=tol * np.abs(gb).max())


@pytest.mark.parametrize("name", REALSPACE_CASES)
def test_oracle_realspace_matches_reference(name):
    c = load(name)
    cells = c["cell"].reshape(-1, 3, 3) if int(c["has_cell"]) else None
    n_dl = direct_n_dl(c)
    nks = None if cells is None else [direct_nk(cl, n_dl) for cl in cells]
    ksm = None if cells is None else [(2.0 * np.pi / n_dl) ** 2] * len(cells)
    lam = None if c["lam"] < 0 else float(c["lam"])
    res = O.bundle(c["r"], c["q"], cells, c["batch"], c["amp"], c["bw2"], solver="direct",
                   nks=nks, k_sq_max=ksm, remove_self=bool(c["remove_self"]),
                   self_coeff=float(c["self_coeff"]), charge_neutral_lambda=lam)
    e_ref = c["energy"]
    assert np.allclose(res["energy"], e_ref, rtol=1e-12, atol=1e-13 * np.abs(e_ref).max())
    w = c["grad_weights"][c["batch"]]
    fscale = max(1.0, np.abs(c["forces"]).max())
    assert np.abs(res["forces"] * w[:, None] - c["forces"]).max() < 1e-11 * fscale
    q = c["q"] if c["q"].ndim == 2 else c["q"][:, None]
    gq = res["potential"] * w[:, None]
    assert np.abs(gq - c["grad_q"].reshape(q.shape)).max() < 1e-11 * max(1.0, np.abs(gq).max())
    if "grad_amp" in c:
        ga = (res["grad_amp"] * c["grad_weights"][:, None]).sum(0)
        gb = (res["grad_bw2"] * c["grad_weights"][:, None]).sum(0)
        assert np.allclose(ga, c["grad_amp"], rtol=1e-10, atol=1e-12 * np.abs(ga).max())
        assert np.allclose(gb, c["grad_bw2"], rtol=1e-10, atol=1e-12 * np.abs(gb).max())
    # a one-atom molecule has only the self term (or nothing)
    assert np.isfinite(res["energy"]).all()


@pytest.mark.parametrize("order", [4, 5, 6])
def test_bspline_weights_match_reference_header(order):
    ref = O.ref_lib()
    if ref is None:
        pytest.skip("oracle/_ref not built (reference tree absent when building)")
    import ctypes
    rng = np.random.default_rng(order)
    for t in np.concatenate([[0.0, 0.5, 1.0 - 1e-16], rng.random(50)]):
        w = O.bspline_weights(order, float(t))
        wr = np.zeros(order)
        ref.ref_bspline_weights(order, ctypes.c_double(t), wr.ctypes.data_as(ctypes.POINTER(ctypes.c_double)))
        assert np.array_equal(w, wr)
        assert abs(w.sum() - 1.0) < 1e-14


@pytest.mark.parametrize("order", [4, 6])
def test_cubes2_node_table_and_moments(order):
    """32 / 88 nodes (cubes2_spline.py:33-38); the weights reproduce
    polynomials through degree order-1 exactly (the moment conditions
    checked by the reference's verify_order6 / test_cubes2_order6.py)."""
    d = O.cubes2_nodes(order)
    assert len(d) == {4: 32, 6: 88}[order]
    rng = np.random.default_rng(order)
    for t in rng.random((20, 3)):
        w = O.cubes2_weights(order, t)
        assert abs(w.sum() - 1.0) < 1e-13
        # first moments: sum_k w_k (d_k - t) = 0 per axis
        assert np.abs((w[:, None] * (d - t[None, :])).sum(0)).max() < 1e-13


@pytest.mark.parametrize("order", [4, 6])
def test_quads_weights_and_influence_match_reference_header(order):
    ref = O.ref_lib()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    import ctypes
    rng = np.random.default_rng(order)
    for t in rng.random(50):
        w = O.quads_weights(order, float(t))
        wr = np.zeros(order)
        ref.ref_quads_weights(order, ctypes.c_double(t), wr.ctypes.data_as(ctypes.POINTER(ctypes.c_double)))
        assert np.allclose(w, wr, rtol=0, atol=1e-15)
    for n in (8, 25, 64, 100):
        for m in range(-(n // 2), n // 2 + 1):
            assert abs(O.quads_influence_1d(m, n, order) - ref.ref_quads_influence_1d(m, n, order)) < 1e-14


@pytest.mark.parametrize("order", [4, 5, 6])
def test_bspline_moments(order):
    """Partition of unity and vanishing odd moments about the particle
    (cardinal B-splines reproduce polynomials of degree 1 exactly)."""
    first = -((order - 1) // 2)
    for t in np.linspace(0.0, 1.0, 11, endpoint=False):
        w = O.bspline_weights(order, float(t))
        offs = first + np.arange(order)
        assert abs(w.sum() - 1.0) < 1e-14
        # center of mass of the stencil = particle position (even order)
        if order % 2 == 0:
            assert abs((w * (offs - t)).sum()) < 1e-13


def test_oracle_fft_matches_numpy():
    rng = np.random.default_rng(0)
    for n in (8, 12, 25, 27, 45, 64, 75, 100, 108):
        x = rng.standard_normal(n) + 1j * rng.standard_normal(n)
        out = np.zeros(2 * n)
        inp = np.ascontiguousarray(np.stack([x.real, x.imag], 1).reshape(-1))
        import ctypes
        P = ctypes.POINTER(ctypes.c_double)
        O.lib().orc_fft_c2c(inp.ctypes.data_as(P), out.ctypes.data_as(P), n, -1)
        y = out[0::2] + 1j * out[1::2]
        assert np.abs(y - np.fft.fft(x)).max() < 1e-12 * n


def test_bspline_mesh_converges_to_direct():
    """The B-spline mesh energy approaches the direct k-sum as the spline order
    rises (discretisation check; no executable reference for the B-spline)."""
    rng = np.random.default_rng(5)
    L, n = 12.0, 50
    r = rng.random((n, 3)) * L
    q = rng.random(n) - 0.5
    q -= q.mean()
    bw = np.array([1.5, 2.5, 4.0])
    amp = 1.0 / (bw * np.sqrt(2 * np.pi)) * bw * bw
    cell = np.eye(3) * L
    (nx, ny, nz), ksm = grid_ndl(cell, 0.7)
    d = O.direct_solve(r, q, cell, amp, bw * bw, nk=direct_nk(cell, 0.7), k_sq_max=ksm)
    errs = []
    for order in (4, 6):
        m = O.mesh_solve(r, q, cell, amp, bw * bw, spline=O.BSPLINE, order=order, nx=nx, ny=ny,
                         nz=nz, k_sq_max=ksm)
        errs.append(abs(m["energy"] - d["energy"]) / abs(d["energy"]))
        assert np.abs(m["forces"] - d["forces"]).max() < 1e-3
    assert errs[1] < errs[0] < 1e-3


def test_oracle_config3_full_size_matches_reference_quads4():
    """20,000-atom triclinic cell on the 96 x 100 x 108 mesh: the oracle's
    QuadS-4 (reference wave vector) against the reference itself."""
    from tests._cases import cfg3_inputs, digest
    c = cfg3_inputs()
    g = load("cfg3_quads4")
    assert str(g["digest"]) == digest(c["r"], c["q"], c["cell"], c["amp_raw"], c["bw"])
    grid, ksm = grid_ndl(c["cell"], c["n_dl"])
    assert grid == (96, 100, 108)
    res = O.bundle(c["r"], c["q"], c["cell"][None], np.zeros(len(c["r"]), int), g["amp"], g["bw2"],
                   solver="mesh", grids=[grid], k_sq_max=[ksm], spline=O.QUADS, order=4,
                   want_virial=True, kconv=1)
    assert abs(res["energy"][0] - g["energy"][0]) < 1e-12 * abs(g["energy"][0])
    assert np.abs(res["forces"] - g["forces"]).max() < 1e-11
    assert np.abs(res["virial"] - g["virial"]).max() < 1e-11 * np.abs(g["virial"]).max()
    assert np.abs(res["potential"][:, 0] - g["grad_q"]).max() < 1e-11
    assert np.allclose(res["grad_amp"][0], g["grad_amp"], rtol=1e-11, atol=0)
    assert np.allclose(res["grad_bw2"][0], g["grad_bw2"], rtol=1e-11, atol=0)


def test_oracle_quads_exact_position_gradient_matches_reference_autograd():
    """The reference's QuadS forces by autograd differentiate its spread
    weights (quads_fft.py:34-73 under torch autograd); the oracle's exact
    gradient reproduces them on the 20,000-atom triclinic system."""
    from tests._cases import cfg3_inputs
    c = cfg3_inputs()
    g = load("cfg3_quads4")
    grid, ksm = grid_ndl(c["cell"], c["n_dl"])
    res = O.mesh_solve(c["r"], c["q"], c["cell"], g["amp"], g["bw2"], spline=O.QUADS, order=4, nx=grid[0],
                       ny=grid[1], nz=grid[2], k_sq_max=ksm, want_force=False, want_dedr=True, kconv=1)
    assert np.abs(res["dedr"] - g["grad_r"]).max() < 1e-11


@pytest.mark.parametrize("spline,order", [(O.BSPLINE, 4), (O.BSPLINE, 5), (O.BSPLINE, 6), (O.QUADS, 6)])
def test_oracle_exact_position_gradient_matches_finite_differences(spline, order):
    rng = np.random.default_rng(order + 10 * spline)
    cell = np.array([[9.0, 0.0, 0.0], [0.7, 9.4, 0.0], [-0.5, 0.6, 8.8]])
    n = 20
    r = rng.random((n, 3)) @ cell
    q = rng.standard_normal(n)
    q -= q.mean()
    amp, bw2 = np.array([0.9, 1.3]), np.array([1.4, 4.0])
    grid, ksm = grid_ndl(cell, 0.8)
    kw = dict(spline=spline, order=order, nx=grid[0], ny=grid[1], nz=grid[2], k_sq_max=ksm, want_force=False)
    res = O.mesh_solve(r, q, cell, amp, bw2, want_dedr=True, **kw)
    h = 1e-5
    for i in (0, 7):
        for b in range(3):
            rp, rm = r.copy(), r.copy()
            rp[i, b] += h
            rm[i, b] -= h
            fd = (O.mesh_solve(rp, q, cell, amp, bw2, **kw)["energy"] -
                  O.mesh_solve(rm, q, cell, amp, bw2, **kw)["energy"]) / (2 * h)
            assert abs(fd - res["dedr"][i, b]) < 1e-7 * max(1.0, abs(fd))


@pytest.mark.parametrize("name", MESH_CASES + CUBES2_CASES)
def test_oracle_position_gradient_matches_reference_autograd(name):
    """The reference's dE/dr by autograd: QuadS differentiates its spread
    weights (the oracle's exact gradient); CubeS2's backward returns the ik
    force (cubes2_fft.py:763-779)."""
    c = load(name)
    cells = c["cell"].reshape(-1, 3, 3)
    q = c["q"] if c["q"].ndim == 2 else c["q"][:, None]
    cubes = name.startswith("cubes2")
    dedr = np.zeros((len(c["r"]), 3))
    for f, cl in enumerate(cells):
        idx = np.nonzero(c["batch"] == f)[0]
        grid, ksm = grid_ndl(cl, float(c["n_dl"]))
        for ch in range(q.shape[1]):
            res = O.mesh_solve(c["r"][idx], q[idx, ch], cl, c["amp"], c["bw2"],
                               spline=O.CUBES2 if cubes else O.QUADS, order=int(c["order"]), nx=grid[0],
                               ny=grid[1], nz=grid[2], k_sq_max=ksm, want_force=cubes,
                               want_dedr=not cubes, kconv=1, remove_self=bool(c["remove_self"]))
            dedr[idx] += (-res["forces"] if cubes else res["dedr"]) * c["grad_weights"][f]
    assert np.abs(dedr - c["grad_r"]).max() < 1e-11


@pytest.mark.parametrize("spline,cell", [
    (O.BSPLINE, np.diag([12.0, 9.0, 16.0])),                                  # coarse: alias sums
    (O.BSPLINE, np.array([[9.0, 0.0, 0.0], [0.7, 9.4, 0.0], [-0.5, 0.6, 8.8]])),
    (O.QUADS, np.array([[9.0, 0.0, 0.0], [0.7, 9.4, 0.0], [-0.5, 0.6, 8.8]]))])
def test_oracle_parameter_gradients_match_finite_differences(spline, cell):
    """dE/d(amp, bw2) are the derivatives of the returned energy, including a
    mesh too coarse for k_max, where every alias term of the B-spline Green
    function brings its own |k + alias|^2 into the bw2 derivative."""
    rng = np.random.default_rng(21 + spline)
    n = 24
    r = rng.random((n, 3)) @ cell
    q = rng.standard_normal(n)
    q -= q.mean()
    amp, bw2 = np.array([0.9, 1.3, 0.7]), np.array([0.8, 1.9, 4.0])
    grid, ksm = grid_ndl(cell, 0.8)
    if cell[0, 0] == 12.0:
        grid = (20, 15, 27)   # below 2 L k_max / 2 pi on every axis
    kw = dict(spline=spline, order=6, nx=grid[0], ny=grid[1], nz=grid[2], k_sq_max=ksm, want_force=False)
    res = O.mesh_solve(r, q, cell, amp, bw2, want_param_grad=True, **kw)
    h = 1e-6
    for m in range(3):
        for arr, key in ((amp, "grad_amp"), (bw2, "grad_bw2")):
            p, mm = arr.copy(), arr.copy()
            p[m] += h
            mm[m] -= h
            args_p = (p, bw2) if key == "grad_amp" else (amp, p)
            args_m = (mm, bw2) if key == "grad_amp" else (amp, mm)
            fd = (O.mesh_solve(r, q, cell, *args_p, **kw)["energy"] -
                  O.mesh_solve(r, q, cell, *args_m, **kw)["energy"]) / (2 * h)
            assert abs(fd - res[key][m]) < 1e-7 * max(1.0, abs(fd)), (key, m)
