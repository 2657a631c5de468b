"""CPU oracle for the SOG reciprocal-space solver — TEST INFRASTRUCTURE ONLY.

This module is the parity checker.  Only ``tests/``, ``__graft_entry__.smoke()``
and the CPU legs of ``bench.py`` may import it; the ``sog_b200`` product never
does, and it is never a fallback for the CUDA path.

It wraps ``libsog_oracle.so`` (the C restatement in ``sog_oracle.c``) with
numpy, and restates in numpy the per-frame host arithmetic of the reference:

* the k=0 correction and charge-neutral penalty of
  ``src/sog/module/gaussian.py:769-798`` (``k0_correction``);
* the per-frame / per-channel orchestration of ``compute_bundle``
  (``gaussian.py:550-820``): channels are solved independently and summed,
  the k=0 term uses the frame's total charge over all channels
  (``bundle``).

Parity is pinned by ``tests/golden`` (fixtures made by importing the reference)
and by ``oracle/_ref`` (the reference's own ``lmp/sog_spline.h`` compiled).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from typing import Dict, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

BSPLINE = 0
QUADS = 1
CUBES2 = 2


def build(reference: Optional[str] = None) -> None:
    """Compile the oracle, and oracle/_ref when ``reference`` (or the
    SOG_REFERENCE environment variable) names the reference tree."""
    ref = reference or os.environ.get("SOG_REFERENCE", "")
    cmd = ["make", "-s", "-C", _HERE]
    if ref:
        cmd.append(f"REF={ref}")
    subprocess.run(cmd, check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "libsog_oracle.so")
        if not os.path.exists(path):
            build()
        _LIB = ctypes.CDLL(path)
        _LIB.orc_quads_influence_1d.restype = ctypes.c_double
        _LIB.orc_bspline_sinc_sum.restype = ctypes.c_double
        _LIB.orc_bspline_sinc2p.restype = ctypes.c_double
        _LIB.orc_quads_xi.restype = ctypes.c_double
        _LIB.orc_cubes2_xi.restype = ctypes.c_double
        _LIB.orc_realspace_solve.restype = ctypes.c_double
        _LIB.orc_realspace_solve.argtypes = [
            ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_double, ctypes.c_int, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return _LIB


def ref_lib():
    """The reference's own lmp/sog_spline.h compiled (oracle/_ref), or None."""
    global _REF
    if _REF is None:
        path = os.path.join(_HERE, "_ref", "libsog_spline_ref.so")
        if not os.path.exists(path):
            return None
        _REF = ctypes.CDLL(path)
        _REF.ref_quads_influence_1d.restype = ctypes.c_double
    return _REF


_dp = ctypes.POINTER(ctypes.c_double)


def _ptr(a: Optional[np.ndarray]):
    if a is None:
        return ctypes.cast(None, _dp)
    assert a.dtype == np.float64 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_dp)


class _MeshIn(ctypes.Structure):
    _fields_ = [
        ("spline", ctypes.c_int), ("order", ctypes.c_int),
        ("nx", ctypes.c_int), ("ny", ctypes.c_int), ("nz", ctypes.c_int),
        ("alias_extent", ctypes.c_int), ("kconv", ctypes.c_int),
        ("natoms", ctypes.c_int), ("r", _dp), ("q", _dp),
        ("cell", ctypes.c_double * 9), ("M", ctypes.c_int),
        ("amp", _dp), ("bw2", _dp),
        ("k_sq_max", ctypes.c_double), ("norm_factor", ctypes.c_double),
        ("self_coeff", ctypes.c_double),
        ("remove_self", ctypes.c_int), ("want_force", ctypes.c_int),
        ("want_pot", ctypes.c_int), ("want_param_grad", ctypes.c_int),
        ("want_virial", ctypes.c_int), ("want_dedr", ctypes.c_int),
    ]


class _MeshOut(ctypes.Structure):
    _fields_ = [
        ("energy", ctypes.c_double), ("diag_sum", ctypes.c_double),
        ("forces", _dp), ("potential", _dp), ("grad_amp", _dp), ("grad_bw2", _dp),
        ("virial", ctypes.c_double * 9), ("dedr", _dp),
    ]


class _DirectIn(ctypes.Structure):
    _fields_ = [
        ("natoms", ctypes.c_int), ("r", _dp), ("q", _dp),
        ("cell", ctypes.c_double * 9), ("nk", ctypes.c_int * 3), ("M", ctypes.c_int),
        ("amp", _dp), ("bw2", _dp),
        ("k_sq_max", ctypes.c_double), ("norm_factor", ctypes.c_double),
        ("self_coeff", ctypes.c_double), ("remove_self", ctypes.c_int),
    ]


class _DirectOut(ctypes.Structure):
    _fields_ = [
        ("energy", ctypes.c_double), ("diag_sum", ctypes.c_double),
        ("nmodes_half", ctypes.c_int),
        ("forces", _dp), ("potential", _dp), ("grad_amp", _dp), ("grad_bw2", _dp),
    ]


def _f64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def bspline_weights(order: int, t: float) -> np.ndarray:
    w = np.zeros(order)
    lib().orc_bspline_weights(order, ctypes.c_double(t), _ptr(w))
    return w


def quads_weights(order: int, t: float) -> np.ndarray:
    w = np.zeros(order)
    lib().orc_quads_weights(order, ctypes.c_double(t), _ptr(w))
    return w


def cubes2_weights(order: int, t) -> np.ndarray:
    """Node weights of CubeS2 order 4 / 6 at fractional offsets t[3], in the
    order of ``cubes2_nodes``."""
    w = np.zeros(216)
    tt = _f64(np.asarray(t, dtype=np.float64).reshape(3))
    n = lib().orc_cubes2_weights(order, _ptr(tt), _ptr(w))
    return w[:n].copy()


def cubes2_nodes(order: int) -> np.ndarray:
    """[n, 3] node offsets of CubeS2 order 4 / 6 (offsets from the floor index)."""
    d = np.zeros(3 * 216, dtype=np.int32)
    n = lib().orc_cubes2_nodes(order, d.ctypes.data_as(ctypes.c_void_p), None)
    return d[:3 * n].reshape(n, 3).copy()


def quads_influence_1d(m: int, n: int, order: int) -> float:
    return lib().orc_quads_influence_1d(m, n, order)


def bspline_deconv_1d(mode: int, n: int, order: int, alias_extent: int = 8) -> float:
    """sinc^(2p)(pi m/N) / (sum_j sinc^(2p)(pi m/N + pi j))^2 (lmp/sog.cpp:1495-1515)."""
    s0 = lib().orc_bspline_sinc2p(mode, n, order, 0)
    ss = lib().orc_bspline_sinc_sum(mode, n, order, alias_extent)
    return s0 / (ss * ss)


def mesh_solve(r, q, cell, amp, bw2, *, spline: int, order: int, nx: int, ny: int,
               nz: int, k_sq_max: float, norm_factor: float = 14.3996454784255,
               self_coeff: float = 0.0, remove_self: bool = True,
               want_force: bool = True, want_pot: bool = False,
               want_param_grad: bool = False, want_virial: bool = False,
               alias_extent: int = 8, kconv: int = 0, want_dedr: bool = False) -> Dict[str, np.ndarray]:
    """One frame, one charge channel.  Energy excludes the k=0 correction.
    want_dedr: the exact gradient of the mesh energy w.r.t. the positions
    (derivatives of the spline weights, B-spline and QuadS), as autograd
    through the reference's QuadS spread gives it."""
    r = _f64(r).reshape(-1, 3)
    q = _f64(q).reshape(-1)
    amp = _f64(amp).reshape(-1)
    bw2 = _f64(bw2).reshape(-1)
    n = r.shape[0]
    M = amp.shape[0]
    inp = _MeshIn()
    inp.spline, inp.order, inp.nx, inp.ny, inp.nz = spline, order, nx, ny, nz
    inp.alias_extent, inp.kconv, inp.natoms = alias_extent, kconv, n
    inp.r, inp.q = _ptr(r), _ptr(q)
    inp.cell[:] = [float(x) for x in np.asarray(cell, dtype=np.float64).reshape(9)]
    inp.M, inp.amp, inp.bw2 = M, _ptr(amp), _ptr(bw2)
    inp.k_sq_max, inp.norm_factor, inp.self_coeff = k_sq_max, norm_factor, self_coeff
    inp.remove_self, inp.want_force, inp.want_pot = int(remove_self), int(want_force), int(want_pot)
    inp.want_param_grad, inp.want_virial = int(want_param_grad), int(want_virial)
    inp.want_dedr = int(want_dedr)
    f = np.zeros((n, 3)) if want_force else None
    dedr = np.zeros((n, 3)) if want_dedr else None
    p = np.zeros(n) if want_pot else None
    ga = np.zeros(M) if want_param_grad else None
    gb = np.zeros(M) if want_param_grad else None
    out = _MeshOut()
    out.forces, out.potential, out.grad_amp, out.grad_bw2 = _ptr(f), _ptr(p), _ptr(ga), _ptr(gb)
    out.dedr = _ptr(dedr)
    lib().orc_mesh_solve(ctypes.byref(inp), ctypes.byref(out))
    res = {"energy": out.energy, "diag_sum": out.diag_sum, "forces": f, "potential": p,
           "grad_amp": ga, "grad_bw2": gb, "dedr": dedr}
    if want_virial:
        res["virial"] = np.array(out.virial[:]).reshape(3, 3)
    return res


def direct_solve(r, q, cell, amp, bw2, *, nk: Sequence[int], k_sq_max: float,
                 norm_factor: float = 14.3996454784255, self_coeff: float = 0.0,
                 remove_self: bool = True) -> Dict[str, np.ndarray]:
    """Direct k-sum of one frame / channel (gaussian.py:1281-1337), explicit
    derivatives.  Energy excludes the k=0 correction."""
    r = _f64(r).reshape(-1, 3)
    q = _f64(q).reshape(-1)
    amp = _f64(amp).reshape(-1)
    bw2 = _f64(bw2).reshape(-1)
    n, M = r.shape[0], amp.shape[0]
    inp = _DirectIn()
    inp.natoms, inp.r, inp.q = n, _ptr(r), _ptr(q)
    inp.cell[:] = [float(x) for x in np.asarray(cell, dtype=np.float64).reshape(9)]
    inp.nk[:] = [int(x) for x in nk]
    inp.M, inp.amp, inp.bw2 = M, _ptr(amp), _ptr(bw2)
    inp.k_sq_max, inp.norm_factor, inp.self_coeff = k_sq_max, norm_factor, self_coeff
    inp.remove_self = int(remove_self)
    f, p, ga, gb = np.zeros((n, 3)), np.zeros(n), np.zeros(M), np.zeros(M)
    out = _DirectOut()
    out.forces, out.potential, out.grad_amp, out.grad_bw2 = _ptr(f), _ptr(p), _ptr(ga), _ptr(gb)
    lib().orc_direct_solve(ctypes.byref(inp), ctypes.byref(out))
    return {"energy": out.energy, "diag_sum": out.diag_sum, "nmodes_half": out.nmodes_half,
            "forces": f, "potential": p, "grad_amp": ga, "grad_bw2": gb}


def realspace_solve(r, q, amp, bw2, *, norm_factor: float = 14.3996454784255,
                    remove_self: bool = True) -> Dict[str, np.ndarray]:
    """Real-space pair sum of one non-periodic frame over all channels
    (compute_potential_realspace, gaussian.py:822-845), explicit derivatives.
    q is [n] or [n, C]; the energy includes the self term when remove_self is
    False and excludes the neutrality penalty."""
    r = np.ascontiguousarray(_f64(r).reshape(-1, 3))
    q = _f64(q)
    if q.ndim == 1:
        q = q[:, None]
    q = np.ascontiguousarray(q)
    amp = np.ascontiguousarray(_f64(amp).reshape(-1))
    bw2 = np.ascontiguousarray(_f64(bw2).reshape(-1))
    n, C = q.shape
    M = amp.shape[0]
    f, p, ga, gb = np.zeros((n, 3)), np.zeros((n, C)), np.zeros(M), np.zeros(M)
    e = lib().orc_realspace_solve(n, C, _ptr(r), _ptr(q), M, _ptr(amp), _ptr(bw2),
                                  float(norm_factor), int(remove_self), _ptr(f), _ptr(p),
                                  _ptr(ga), _ptr(gb))
    return {"energy": float(e), "forces": f, "potential": p, "grad_amp": ga, "grad_bw2": gb}


def penalty(q_frame: np.ndarray, charge_neutral_lambda: Optional[float]):
    """Charge-neutral penalty lambda * sum_c mean_c(q)^2 of one frame
    (gaussian.py:795-798): (energy, dE/dq [n, C])."""
    q_frame = _f64(q_frame)
    if q_frame.ndim == 1:
        q_frame = q_frame[:, None]
    if charge_neutral_lambda is None or not charge_neutral_lambda > 0:
        return 0.0, np.zeros_like(q_frame)
    mean = q_frame.mean(axis=0)
    e = float(charge_neutral_lambda) * float((mean ** 2).sum())
    dq = np.broadcast_to(float(charge_neutral_lambda) * 2.0 * mean[None, :] / q_frame.shape[0],
                         q_frame.shape).copy()
    return e, dq


def k0_correction(q_frame: np.ndarray, cell, amp, bw2, *, norm_factor: float,
                  remove_self: bool, charge_neutral_lambda: Optional[float] = None):
    """k=0 charge / self correction and the optional neutrality penalty of one
    frame (gaussian.py:769-798).  q_frame is [n, C]; returns
    (energy, dE/dq [n,C], dE/damp [M], dE/dbw2 [M])."""
    q_frame = _f64(q_frame)
    if q_frame.ndim == 1:
        q_frame = q_frame[:, None]
    cell = _f64(cell).reshape(3, 3)
    amp = _f64(amp)
    bw2 = _f64(bw2)
    vol = abs(np.linalg.det(cell))
    a1, a2, a3 = cell
    b = [2.0 * math.pi * np.cross(a2, a3) / vol, 2.0 * math.pi * np.cross(a3, a1) / vol,
         2.0 * math.pi * np.cross(a1, a2) / vol]
    kmin2 = min(float(v @ v) for v in b)
    em = np.exp(-0.5 * bw2 * kmin2)
    kfe = float((amp * em).sum())
    qs = float(q_frame.sum())
    qq = float((q_frame ** 2).sum())
    e = kfe * qs * qs / (2.0 * vol) * norm_factor
    dq = np.full_like(q_frame, kfe * 2.0 * qs / (2.0 * vol) * norm_factor)
    c_amp = qs * qs / (2.0 * vol) * norm_factor
    if remove_self:
        e -= kfe * qq / (2.0 * vol) * norm_factor
        dq -= kfe * 2.0 * q_frame / (2.0 * vol) * norm_factor
        c_amp -= qq / (2.0 * vol) * norm_factor
    ga = em * c_amp
    gb = amp * em * (-0.5 * kmin2) * c_amp
    e_p, dq_p = penalty(q_frame, charge_neutral_lambda)
    return e + e_p, dq + dq_p, ga, gb


def bundle(r, q, cell, batch, amp, bw2, *, solver: str, grids=None, nks=None,
           k_sq_max=None, spline: int = BSPLINE, order: int = 6,
           norm_factor: float = 14.3996454784255, self_coeff: float = 0.0,
           remove_self: bool = True, charge_neutral_lambda=None,
           want_virial: bool = False, alias_extent: int = 8, kconv: int = 0):
    """Reference-equivalent per-frame energies and explicit derivatives for a
    batch (compute_bundle, gaussian.py:380-820), solver "mesh" or "direct".
    grids[f] = (nx, ny, nz); nks[f] = (n1, n2, n3); k_sq_max[f] per frame.
    Frames without a cell (cell=None) or with a singular cell take the
    real-space pair sum (gaussian.py:735-746) and no k=0 term."""
    r = _f64(r).reshape(-1, 3)
    q = _f64(q)
    if q.ndim == 1:
        q = q[:, None]
    batch = np.asarray(batch, dtype=np.int64).reshape(-1)
    amp = _f64(amp)
    bw2 = _f64(bw2)
    if cell is None:
        nf = int(batch.max()) + 1 if batch.size else 0
        cell = np.zeros((nf, 3, 3))
    cell = _f64(cell).reshape(-1, 3, 3)
    nf = cell.shape[0]
    n, C = q.shape
    M = amp.shape[0]
    energy = np.zeros(nf)
    forces = np.zeros((n, 3))
    pot = np.zeros((n, C))
    gamp = np.zeros((nf, M))
    gbw2 = np.zeros((nf, M))
    vir = np.zeros((nf, 3, 3))
    for f in range(nf):
        idx = np.nonzero(batch == f)[0]
        if idx.size == 0:
            continue
        if not abs(np.linalg.det(cell[f])) > np.finfo(np.float64).eps:
            res = realspace_solve(r[idx], q[idx], amp, bw2, norm_factor=norm_factor,
                                  remove_self=remove_self)
            e_p, dq_p = penalty(q[idx], charge_neutral_lambda)
            energy[f] = res["energy"] + e_p
            forces[idx] = res["forces"]
            pot[idx] = res["potential"] + dq_p
            gamp[f] = res["grad_amp"]
            gbw2[f] = res["grad_bw2"]
            continue
        for c in range(C):
            if solver == "mesh":
                nx, ny, nz = grids[f]
                res = mesh_solve(r[idx], q[idx, c], cell[f], amp, bw2, spline=spline,
                                 order=order, nx=nx, ny=ny, nz=nz, k_sq_max=k_sq_max[f],
                                 norm_factor=norm_factor, self_coeff=self_coeff,
                                 remove_self=remove_self, want_force=True, want_pot=True,
                                 want_param_grad=True, want_virial=want_virial,
                                 alias_extent=alias_extent, kconv=kconv)
                if want_virial:
                    vir[f] += res["virial"]
            else:
                res = direct_solve(r[idx], q[idx, c], cell[f], amp, bw2, nk=nks[f],
                                   k_sq_max=k_sq_max[f], norm_factor=norm_factor,
                                   self_coeff=self_coeff, remove_self=remove_self)
            energy[f] += res["energy"]
            forces[idx] += res["forces"]
            pot[idx, c] = res["potential"]
            gamp[f] += res["grad_amp"]
            gbw2[f] += res["grad_bw2"]
        e0, dq0, ga0, gb0 = k0_correction(q[idx], cell[f], amp, bw2, norm_factor=norm_factor,
                                          remove_self=remove_self,
                                          charge_neutral_lambda=charge_neutral_lambda)
        energy[f] += e0
        pot[idx] += dq0
        gamp[f] += ga0
        gbw2[f] += gb0
    return {"energy": energy, "forces": forces, "potential": pot, "grad_amp": gamp,
            "grad_bw2": gbw2, "virial": vir}


def num_threads() -> int:
    return int(lib().orc_num_threads())


def set_num_threads(n: int) -> int:
    """Use n OpenMP threads from now on; returns the count in effect."""
    lib().orc_set_num_threads(int(n))
    return num_threads()
