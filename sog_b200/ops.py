"""Autograd functions around the C ABI.

One forward launch computes the energy together with every derivative the
graph will need (forces when positions require grad or explicit forces are
asked for, dE/dq when charges do, dE/d(amp, bw2) when the kernel parameters
do), so the backward is a per-frame scaling of saved results.  This is the
hand-written backward of src/sog/module/cubes2_fft.py:746-869 generalised to
all solvers: dE/dr is the ik-differentiated force (as there), dE/dq the
gathered potential plus self and k=0 terms, dE/d(amp, bw2) the M-vector
k-space reductions.  Non-periodic frames (no cell, or a singular one) take the
real-space pair sum (gaussian.py:822-845) with the same explicit outputs.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch
from torch.autograd.function import once_differentiable

from . import _lib


@dataclass
class Bucket:
    """Frames solved by one C-ABI call (same mesh, or the direct solver)."""
    frames: List[int]            # positions in the output energy vector
    atom_begin: List[int]
    atom_count: List[int]
    k_sq_max: List[float]
    dims: Optional[Tuple[int, int, int]] = None   # mesh
    nk: Optional[List[Tuple[int, int, int]]] = None  # direct
    kind: Optional[str] = None   # "realspace" for non-periodic frames, else the spec's kind
    _host: Optional[dict] = None

    _idx: Optional[torch.Tensor] = None

    def host(self) -> dict:
        """The per-frame arrays as ctypes arrays, converted on first use."""
        if self._host is None:
            self._host = _lib.host_tables(self.atom_begin, self.atom_count, self.k_sq_max, self.nk)
        return self._host

    def frame_index(self, dev: torch.device) -> torch.Tensor:
        """The bucket's output positions on `dev`, uploaded once (a fresh
        upload per call would be a synchronous copy that waits for the
        device)."""
        if self._idx is None or self._idx.device != dev:
            self._idx = torch.tensor(self.frames, device=dev, dtype=torch.long)
        return self._idx


@dataclass
class SolveSpec:
    kind: str                    # "mesh" | "direct" (buckets may say "realspace")
    buckets: List[Bucket]
    nframes: int
    cells: Optional[torch.Tensor]  # [nf, 3, 3] (frames in output order), compute dtype; None: no cell
    frame_of_atom: torch.Tensor  # [N] int64 output-frame index of each (sorted) atom
    spline: int = _lib.SPLINE_BSPLINE
    order: int = 6
    kconv: int = _lib.KCONV_PHYSICAL
    alias_extent: int = 8
    norm_factor: float = 14.3996454784255
    self_coeff: float = 0.0
    remove_self: bool = True
    k0_correction: bool = True
    charge_neutral_lambda: Optional[float] = None
    cache: dict = field(default_factory=dict)
    slab: Optional[object] = None    # sog_b200.slab.SlabGroup: one frame over several ranks


def exact_position_gradient(spec: SolveSpec) -> bool:
    """Whether the mesh buckets of ``spec`` give dE/dr as the exact gradient
    of their energy (spline-weight derivatives: the B-spline and QuadS meshes
    on one device) rather than as the ik-differentiated force.  The
    reference's QuadS solver is plain torch, so autograd differentiates its
    spread weights (quads_fft.py:34-73); its CubeS2 backward returns the ik
    force (cubes2_fft.py:763-779), which CubeS2 keeps here."""
    return (spec.kind == "mesh" and spec.slab is None
            and spec.spline in (_lib.SPLINE_BSPLINE, _lib.SPLINE_QUADS))


def run_solver(spec: SolveSpec, q: torch.Tensor, r: torch.Tensor, amp: torch.Tensor,
               bw2: torch.Tensor, *, want_force: bool, want_pot: bool, want_grad: bool,
               want_virial: bool, want_dedr: bool = False):
    """Launch every bucket of ``spec``; returns (energy, forces, pot, gamp,
    gbw2, virial, dedr).  With want_dedr the mesh buckets also write the exact
    dE/dr of their atoms and the other buckets (frames without a periodic
    cell) their forces, so dE/dr = dedr on mesh atoms and -forces elsewhere
    (see position_gradient)."""
    dev = r.device
    dt = r.dtype
    nf = spec.nframes
    M = amp.numel()
    N = r.shape[0]
    C = q.shape[1]
    r = r.contiguous()
    q = q.contiguous()
    amp = amp.contiguous()
    bw2 = bw2.contiguous()
    energy = torch.empty(nf, dtype=dt, device=dev)
    mixed = want_dedr and any((b.kind or spec.kind) != "mesh" for b in spec.buckets)
    forces = torch.zeros(N, 3, dtype=dt, device=dev) if (want_force or mixed) else None
    dedr = torch.zeros(N, 3, dtype=dt, device=dev) if want_dedr else None
    pot = torch.zeros(N, C, dtype=dt, device=dev) if want_pot else None
    gamp = torch.empty(nf, M, dtype=dt, device=dev) if want_grad else None
    gbw2 = torch.empty(nf, M, dtype=dt, device=dev) if want_grad else None
    vir = torch.empty(nf, 3, 3, dtype=dt, device=dev) if want_virial else None
    dcode = _lib.dtype_code(dt)
    single = len(spec.buckets) == 1 and spec.buckets[0].frames == list(range(nf))
    for b in spec.buckets:
        if single:
            cells_b, e_b, ga_b, gb_b, v_b = spec.cells, energy, gamp, gbw2, vir
        else:
            idx = b.frame_index(dev)
            cells_b = None if spec.cells is None else spec.cells.index_select(0, idx).contiguous()
            e_b = torch.empty(len(b.frames), dtype=dt, device=dev)
            ga_b = torch.empty(len(b.frames), M, dtype=dt, device=dev) if want_grad else None
            gb_b = torch.empty(len(b.frames), M, dtype=dt, device=dev) if want_grad else None
            v_b = torch.empty(len(b.frames), 3, 3, dtype=dt, device=dev) if want_virial else None
        h = b.host()
        common = dict(atom_begin=h["atom_begin"], atom_count=h["atom_count"], k_sq_max=h["k_sq_max"],
                      positions=r, charges=q, cells=cells_b, amp=amp, bw2=bw2,
                      norm_factor=spec.norm_factor, self_coeff=spec.self_coeff,
                      remove_self=spec.remove_self, k0_correction=spec.k0_correction,
                      charge_neutral_lambda=spec.charge_neutral_lambda, energy=e_b,
                      forces=forces, potential=pot, grad_amp=ga_b, grad_bw2=gb_b, virial=v_b)
        kind = b.kind or spec.kind
        if kind == "realspace":
            ctx = _lib.direct_ctx(dev.index if dev.index is not None else torch.cuda.current_device(),
                                  dcode)
            _lib.realspace_forward(ctx, **common)
        elif kind == "mesh" and spec.slab is not None:
            if len(b.frames) != 1 or nf != 1:
                raise NotImplementedError("mesh_decomposition='slab' solves one frame per call")
            if want_grad or want_virial:
                raise NotImplementedError("mesh_decomposition='slab' computes energy, forces and "
                                          "dE/dq; parameter gradients and the virial need 'none'")
            plan = _lib.PLANS.get(dev.index if dev.index is not None else torch.cuda.current_device(),
                                  dcode, spec.spline, spec.order, b.dims, spec.kconv,
                                  spec.alias_extent)
            for k in ("grad_amp", "grad_bw2", "virial"):
                common.pop(k)
            _lib.mesh_slab_forward(plan, spec.slab, **common)
            # each rank holds its slab's atoms; the sum gives every atom's
            if forces is not None:
                spec.slab.sum_(forces)
            if pot is not None:
                spec.slab.sum_(pot)
        elif kind == "mesh":
            plan = _lib.PLANS.get(dev.index if dev.index is not None else torch.cuda.current_device(),
                                  dcode, spec.spline, spec.order, b.dims, spec.kconv,
                                  spec.alias_extent)
            if not want_force:
                common["forces"] = None   # the exact gradient only
            _lib.mesh_forward(plan, dedr=dedr, **common)
        else:
            ctx = _lib.direct_ctx(dev.index if dev.index is not None else torch.cuda.current_device(),
                                  dcode)
            _lib.direct_forward(ctx, nk=h["nk"], **common)
        if not single:
            energy.index_copy_(0, idx, e_b)
            if want_grad:
                gamp.index_copy_(0, idx, ga_b)
                gbw2.index_copy_(0, idx, gb_b)
            if want_virial:
                vir.index_copy_(0, idx, v_b)
    return energy, forces, pot, gamp, gbw2, vir, dedr


def position_gradient(spec: SolveSpec, forces, dedr):
    """dE/dr of every atom from run_solver's outputs."""
    if dedr is None:
        return None if forces is None else -forces
    if forces is None or all((b.kind or spec.kind) == "mesh" for b in spec.buckets):
        return dedr
    exact_frames = torch.zeros(spec.nframes, dtype=torch.bool, device=dedr.device)
    for b in spec.buckets:
        if (b.kind or spec.kind) == "mesh":
            exact_frames[b.frame_index(dedr.device)] = True
    return torch.where(exact_frames.index_select(0, spec.frame_of_atom)[:, None], dedr, -forces)


def run_hvp(spec: SolveSpec, q: torch.Tensor, r: torch.Tensor, amp: torch.Tensor, bw2: torch.Tensor,
            dq: Optional[torch.Tensor], dr: Optional[torch.Tensor], damp: Optional[torch.Tensor],
            dbw2: Optional[torch.Tensor]):
    """Hessian of every frame's energy applied to a direction: dq [N,C] on the
    charges, dr [N,3] on the positions, damp / dbw2 [nf,M] per frame on the
    kernel parameters (None: zero).  Returns (out_q [N,C], out_r [N,3],
    out_amp [nf,M], out_bw2 [nf,M]).  The double backward of the solver."""
    dev, dt = r.device, r.dtype
    nf, M, N, C = spec.nframes, amp.numel(), r.shape[0], q.shape[1]
    out_q = torch.zeros(N, C, dtype=dt, device=dev)
    out_r = torch.zeros(N, 3, dtype=dt, device=dev)
    out_a = torch.zeros(nf, M, dtype=dt, device=dev)
    out_b = torch.zeros(nf, M, dtype=dt, device=dev)
    contig = lambda t: None if t is None else t.contiguous()
    q, r, amp, bw2 = q.contiguous(), r.contiguous(), amp.contiguous(), bw2.contiguous()
    dq, dr, damp, dbw2 = contig(dq), contig(dr), contig(damp), contig(dbw2)
    single = len(spec.buckets) == 1 and spec.buckets[0].frames == list(range(nf))
    for b in spec.buckets:
        kind = b.kind or spec.kind
        if kind == "mesh" and (spec.slab is not None or spec.spline == _lib.SPLINE_CUBES2):
            raise NotImplementedError(
                "second derivatives (create_graph=True through the forces or dE/dq) are implemented "
                "for the direct k-sum, the real-space pair sum and the B-spline / QuadS meshes "
                "without slab decomposition; CubeS2 and slab solves raise here")
        if single:
            cells_b, da_b, db_b, oa_b, ob_b = spec.cells, damp, dbw2, out_a, out_b
        else:
            idx = b.frame_index(dev)
            cells_b = None if spec.cells is None else spec.cells.index_select(0, idx).contiguous()
            da_b = None if damp is None else damp.index_select(0, idx).contiguous()
            db_b = None if dbw2 is None else dbw2.index_select(0, idx).contiguous()
            oa_b = torch.zeros(len(b.frames), M, dtype=dt, device=dev)
            ob_b = torch.zeros(len(b.frames), M, dtype=dt, device=dev)
        h = b.host()
        device = dev.index if dev.index is not None else torch.cuda.current_device()
        # each bucket's atoms get their rows written; the others keep theirs
        common = dict(atom_begin=h["atom_begin"], atom_count=h["atom_count"], positions=r, charges=q,
                      amp=amp, bw2=bw2, norm_factor=spec.norm_factor, remove_self=spec.remove_self,
                      charge_neutral_lambda=spec.charge_neutral_lambda, dir_q=dq, dir_r=dr,
                      dir_amp=da_b, dir_bw2=db_b, out_q=out_q, out_r=out_r, out_amp=oa_b, out_bw2=ob_b)
        if kind == "mesh":
            plan = _lib.PLANS.get(device, _lib.dtype_code(dt), spec.spline, spec.order, b.dims, spec.kconv,
                                  spec.alias_extent)
            _lib.mesh_hvp(plan, k_sq_max=h["k_sq_max"], cells=cells_b, self_coeff=spec.self_coeff,
                          k0_correction=spec.k0_correction, **common)
            if not single:
                out_a.index_copy_(0, idx, oa_b)
                out_b.index_copy_(0, idx, ob_b)
            continue
        ctx = _lib.direct_ctx(device, _lib.dtype_code(dt))
        if kind == "realspace":
            _lib.realspace_hvp(ctx, **common)
        else:
            _lib.direct_hvp(ctx, nk=h["nk"], k_sq_max=h["k_sq_max"], cells=cells_b,
                            self_coeff=spec.self_coeff, k0_correction=spec.k0_correction, **common)
        if not single:
            out_a.index_copy_(0, idx, oa_b)
            out_b.index_copy_(0, idx, ob_b)
    return out_q, out_r, out_a, out_b


class SolveFunction(torch.autograd.Function):
    """energy[nf] = SOG(q, r; amp, bw2); explicit forces / virial as extra,
    non-differentiable outputs.  The backward is differentiable again
    (GradFunction) when a graph is being built (create_graph=True)."""

    @staticmethod
    def forward(ctx, q, r, amp, bw2, spec: SolveSpec, want_force_out: bool, want_virial_out: bool):
        need_q, need_r, need_a, need_b = ctx.needs_input_grad[:4]
        want_grad = bool(need_a or need_b)
        exact = bool(need_r) and exact_position_gradient(spec)
        want_force = bool(want_force_out or (need_r and not exact))
        energy, forces, pot, gamp, gbw2, vir, dedr = run_solver(
            spec, q, r, amp, bw2, want_force=want_force, want_pot=bool(need_q),
            want_grad=want_grad, want_virial=bool(want_virial_out), want_dedr=exact)
        ctx.spec = spec
        dEdr = position_gradient(spec, forces, dedr) if need_r else None
        ctx.save_for_backward(q, r, amp, bw2, dEdr, pot, gamp, gbw2)
        f_out = forces if want_force_out else None
        v_out = vir if want_virial_out else None
        outs = [energy, f_out, v_out]
        nd = [t for t in (f_out, v_out) if t is not None]
        if nd:
            ctx.mark_non_differentiable(*nd)
        return tuple(outs)

    @staticmethod
    def backward(ctx, gE, gF, gV):
        q, r, amp, bw2, dEdr, pot, gamp, gbw2 = ctx.saved_tensors
        if gE is None:
            return None, None, None, None, None, None, None
        needs = tuple(ctx.needs_input_grad[:4])
        if torch.is_grad_enabled():
            # create_graph=True: the gradients are differentiable functions of
            # (gE, q, r, amp, bw2); their own backward is the Hessian-vector
            # product of the solver (run_hvp)
            outs = GradFunction.apply(gE, q, r, amp, bw2, pot, dEdr, gamp, gbw2, ctx.spec, needs)
            gq, gr, ga, gb = outs
        else:
            gq, gr, ga, gb = _first_order(gE, ctx.spec.frame_of_atom, pot, dEdr, gamp, gbw2, needs)
        return gq, gr, ga, gb, None, None, None


def _first_order(gE, frame_of_atom, pot, dEdr, gamp, gbw2, needs):
    """gE-weighted first derivatives: dE/dq, dE/dr per atom (its frame's
    weight) and dE/d(amp, bw2) summed over frames."""
    ga = gE.index_select(0, frame_of_atom)
    gq = pot * ga[:, None] if needs[0] and pot is not None else None
    gr = dEdr * ga[:, None] if needs[1] and dEdr is not None else None
    gam = (gE[:, None] * gamp).sum(0) if needs[2] and gamp is not None else None
    gbw = (gE[:, None] * gbw2).sum(0) if needs[3] and gbw2 is not None else None
    return gq, gr, gam, gbw


class GradFunction(torch.autograd.Function):
    """(dE/dq, dE/dr, dE/damp, dE/dbw2) weighted by the energy cotangent gE, as
    a differentiable function of (gE, q, r, amp, bw2).  Its backward is the
    solver's Hessian-vector product: the second derivatives a force loss needs
    (the reference gets them from torch autograd through its direct k-sum,
    gaussian.py:1180-1337, and through the differentiable ops of its Python
    mesh solvers)."""

    @staticmethod
    def forward(ctx, gE, q, r, amp, bw2, pot, dEdr, gamp, gbw2, spec, needs):
        ctx.spec = spec
        ctx.needs = needs
        ctx.save_for_backward(gE, q, r, amp, bw2, pot, dEdr, gamp, gbw2)
        return _first_order(gE, spec.frame_of_atom, pot, dEdr, gamp, gbw2, needs)

    @staticmethod
    @once_differentiable
    def backward(ctx, uq, ur, ua, ub):
        gE, q, r, amp, bw2, pot, dEdr, gamp, gbw2 = ctx.saved_tensors
        spec = ctx.spec
        fa = spec.frame_of_atom
        ga = gE.index_select(0, fa)
        # d/dgE: the directional derivative of each frame's energy
        d_gE = None
        if ctx.needs_input_grad[0]:
            d_gE = torch.zeros_like(gE)
            if uq is not None and pot is not None:
                d_gE.index_add_(0, fa, (uq * pot).sum(1))
            if ur is not None and dEdr is not None:
                d_gE.index_add_(0, fa, (ur * dEdr).sum(1))
            if ua is not None and gamp is not None:
                d_gE += gamp @ ua
            if ub is not None and gbw2 is not None:
                d_gE += gbw2 @ ub
        want_hvp = any(ctx.needs_input_grad[1:5])
        g_q = g_r = g_a = g_b = None
        if want_hvp:
            dq = None if uq is None else uq * ga[:, None]
            dr = None if ur is None else ur * ga[:, None]
            da = None if ua is None else gE[:, None] * ua[None, :]
            db = None if ub is None else gE[:, None] * ub[None, :]
            oq, orr, oa, ob = run_hvp(spec, q, r, amp, bw2, dq, dr, da, db)
            g_q = oq if ctx.needs_input_grad[1] else None
            g_r = orr if ctx.needs_input_grad[2] else None
            g_a = oa.sum(0) if ctx.needs_input_grad[3] else None
            g_b = ob.sum(0) if ctx.needs_input_grad[4] else None
        return d_gE, g_q, g_r, g_a, g_b, None, None, None, None, None, None
