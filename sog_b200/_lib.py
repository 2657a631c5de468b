"""ctypes binding of the C ABI in ``include/sog_b200.h`` (``_lib/libsog_b200.so``).

The product path has no fallback: if the library is missing or CUDA is not
available, every entry raises.  Plans are cached per (device, dtype, spline,
order, mesh, k-convention) with a small LRU, mirroring the reference's
per-box caches (src/sog/module/gaussian.py:268-329).
"""
from __future__ import annotations

import collections
import ctypes
import os
import threading
from typing import Optional, Sequence

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libsog_b200.so")

SOG_OK = 0
DTYPE_F64, DTYPE_F32 = 0, 1
SPLINE_BSPLINE, SPLINE_QUADS, SPLINE_CUBES2 = 0, 1, 2
KCONV_PHYSICAL, KCONV_REFERENCE = 0, 1

_c_i64p = ctypes.POINTER(ctypes.c_int64)
_c_i32p = ctypes.POINTER(ctypes.c_int32)
_c_dp = ctypes.POINTER(ctypes.c_double)
_vp = ctypes.c_void_p


class PlanDesc(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int), ("spline", ctypes.c_int), ("order", ctypes.c_int),
                ("nx", ctypes.c_int), ("ny", ctypes.c_int), ("nz", ctypes.c_int),
                ("device", ctypes.c_int), ("alias_extent", ctypes.c_int), ("kconv", ctypes.c_int)]


class MeshArgs(ctypes.Structure):
    _fields_ = [("nframes", ctypes.c_int), ("atom_begin", _c_i64p), ("atom_count", _c_i64p),
                ("k_sq_max", _c_dp), ("nchannels", ctypes.c_int), ("positions", _vp),
                ("charges", _vp), ("cells", _vp), ("n_gauss", ctypes.c_int), ("amp", _vp),
                ("bw2", _vp), ("norm_factor", ctypes.c_double), ("self_coeff", ctypes.c_double),
                ("remove_self", ctypes.c_int), ("k0_correction", ctypes.c_int),
                ("charge_neutral_lambda", ctypes.c_double), ("energy", _vp), ("forces", _vp),
                ("potential", _vp), ("grad_amp", _vp), ("grad_bw2", _vp), ("virial", _vp),
                ("dedr", _vp)]


class DirectArgs(ctypes.Structure):
    _fields_ = [("nframes", ctypes.c_int), ("atom_begin", _c_i64p), ("atom_count", _c_i64p),
                ("nk", _c_i32p), ("k_sq_max", _c_dp), ("nchannels", ctypes.c_int),
                ("positions", _vp), ("charges", _vp), ("cells", _vp), ("n_gauss", ctypes.c_int),
                ("amp", _vp), ("bw2", _vp), ("norm_factor", ctypes.c_double),
                ("self_coeff", ctypes.c_double), ("remove_self", ctypes.c_int),
                ("k0_correction", ctypes.c_int), ("charge_neutral_lambda", ctypes.c_double),
                ("energy", _vp), ("forces", _vp), ("potential", _vp), ("grad_amp", _vp),
                ("grad_bw2", _vp), ("virial", _vp)]


class RealspaceArgs(ctypes.Structure):
    _fields_ = [("nframes", ctypes.c_int), ("atom_begin", _c_i64p), ("atom_count", _c_i64p),
                ("nchannels", ctypes.c_int), ("positions", _vp), ("charges", _vp),
                ("n_gauss", ctypes.c_int), ("amp", _vp), ("bw2", _vp),
                ("norm_factor", ctypes.c_double), ("remove_self", ctypes.c_int),
                ("charge_neutral_lambda", ctypes.c_double), ("energy", _vp), ("forces", _vp),
                ("potential", _vp), ("grad_amp", _vp), ("grad_bw2", _vp), ("virial", _vp)]


class HvpArgs(ctypes.Structure):
    _fields_ = [("dir_q", _vp), ("dir_r", _vp), ("dir_amp", _vp), ("dir_bw2", _vp),
                ("out_q", _vp), ("out_r", _vp), ("out_amp", _vp), ("out_bw2", _vp)]


# int exchange(void *ctx, int kind, int64 send_off, int64 recv_off, int64 bytes, void *stream)
EXCHANGE_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                               ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p)
EXCH_ALLTOALL, EXCH_HALO, EXCH_SUM_F64, EXCH_ALLGATHER = 0, 1, 2, 3
SLAB_EXCHANGE, SLAB_PEER = 0, 1


class SlabDesc(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int), ("size", ctypes.c_int), ("transport", ctypes.c_int),
                ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t), ("exchange", EXCHANGE_FN),
                ("ctx", _vp)]


EXPORTS = ["sog_strerror", "sog_last_error", "sog_version", "sog_launch_count", "sog_plan_create",
           "sog_plan_destroy", "sog_plan_status", "sog_plan_set_timing", "sog_plan_timings",
           "sog_mesh_forward", "sog_direct_create", "sog_direct_destroy", "sog_direct_set_timing",
           "sog_direct_timings", "sog_direct_forward", "sog_direct_forward_noalloc",
           "sog_mesh_slab_workspace", "sog_mesh_slab_forward", "sog_realspace_forward",
           "sog_direct_hvp", "sog_realspace_hvp", "sog_mesh_hvp"]

_lib = None
_lock = threading.Lock()


class SogError(RuntimeError):
    pass


def load():
    """Load the library (raises when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise SogError(f"{LIB_PATH} is missing: build it with `python -m sog_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name in ("sog_strerror", "sog_last_error", "sog_version"):
            getattr(lib, name).restype = ctypes.c_char_p
        lib.sog_strerror.argtypes = [ctypes.c_int]
        lib.sog_plan_create.argtypes = [ctypes.POINTER(_vp), ctypes.POINTER(PlanDesc)]
        lib.sog_plan_destroy.argtypes = [_vp]
        lib.sog_plan_status.argtypes = [_vp, ctypes.POINTER(ctypes.c_uint)]
        lib.sog_mesh_forward.argtypes = [_vp, ctypes.POINTER(MeshArgs), _vp]
        lib.sog_mesh_slab_workspace.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                ctypes.POINTER(ctypes.c_size_t)]
        lib.sog_mesh_slab_forward.argtypes = [_vp, ctypes.POINTER(MeshArgs), ctypes.POINTER(SlabDesc),
                                              _vp]
        lib.sog_direct_create.argtypes = [ctypes.POINTER(_vp), ctypes.c_int, ctypes.c_int]
        lib.sog_direct_destroy.argtypes = [_vp]
        lib.sog_direct_forward.argtypes = [_vp, ctypes.POINTER(DirectArgs), _vp]
        lib.sog_realspace_forward.argtypes = [_vp, ctypes.POINTER(RealspaceArgs), _vp]
        lib.sog_direct_hvp.argtypes = [_vp, ctypes.POINTER(DirectArgs), ctypes.POINTER(HvpArgs), _vp]
        lib.sog_mesh_hvp.argtypes = [_vp, ctypes.POINTER(MeshArgs), ctypes.POINTER(HvpArgs), _vp]
        lib.sog_realspace_hvp.argtypes = [_vp, ctypes.POINTER(RealspaceArgs), ctypes.POINTER(HvpArgs), _vp]
        lib.sog_launch_count.restype = ctypes.c_ulonglong
        for name in ("sog_plan_set_timing", "sog_direct_set_timing"):
            getattr(lib, name).argtypes = [_vp, ctypes.c_int]
        for name in ("sog_plan_timings", "sog_direct_timings"):
            getattr(lib, name).argtypes = [_vp, ctypes.POINTER(ctypes.c_char_p),
                                           ctypes.POINTER(ctypes.c_float), ctypes.c_int,
                                           ctypes.POINTER(ctypes.c_int)]
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != SOG_OK:
        lib = load()
        raise SogError(f"{what}: {lib.sog_strerror(rc).decode()} ({lib.sog_last_error().decode()})")


def _require_cuda(t: torch.Tensor) -> None:
    if t.device.type != "cuda":
        raise SogError("sog_b200 runs on CUDA devices only (got a tensor on "
                       f"{t.device}); there is no CPU path")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float64:
        return DTYPE_F64
    if dt == torch.float32:
        return DTYPE_F32
    raise SogError(f"unsupported dtype {dt}; use float64 or float32")


class Plan:
    def __init__(self, device: int, dtype: int, spline: int, order: int, dims, kconv: int,
                 alias_extent: int = 8):
        lib = load()
        self.key = (device, dtype, spline, order, tuple(dims), kconv, alias_extent)
        d = PlanDesc(dtype, spline, order, int(dims[0]), int(dims[1]), int(dims[2]), device,
                     alias_extent, kconv)
        h = _vp()
        check(lib.sog_plan_create(ctypes.byref(h), ctypes.byref(d)), "sog_plan_create")
        self.handle = h

    def close(self):
        if self.handle:
            load().sog_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_timing(self, on, events: int = 0) -> None:
        """Per-kernel event timing on / off; `events` sizes the event pool
        (for calls captured into a CUDA graph)."""
        check(load().sog_plan_set_timing(self.handle, max(int(bool(on)), int(events) if on else 0)),
              "sog_plan_set_timing")

    def timings(self):
        """[(kernel name, ms)] of the latest forward (waits for it)."""
        return _timings(load().sog_plan_timings, self.handle)

    def status(self) -> int:
        bits = ctypes.c_uint(0)
        check(load().sog_plan_status(self.handle, ctypes.byref(bits)), "sog_plan_status")
        return int(bits.value)


class _PlanCache:
    def __init__(self, capacity: int = 16):
        self.capacity = capacity
        self.plans: "collections.OrderedDict" = collections.OrderedDict()

    def get(self, *key) -> Plan:
        p = self.plans.get(key)
        if p is not None:
            self.plans.move_to_end(key)
            return p
        p = Plan(*key)
        self.plans[key] = p
        while len(self.plans) > self.capacity:
            _, old = self.plans.popitem(last=False)
            torch.cuda.synchronize()
            old.close()
        return p

    def clear(self):
        torch.cuda.synchronize()
        for p in self.plans.values():
            p.close()
        self.plans.clear()


def _timings(fn, handle, cap: int = 8192):
    names = (ctypes.c_char_p * cap)()
    ms = (ctypes.c_float * cap)()
    cnt = ctypes.c_int(0)
    check(fn(handle, names, ms, cap, ctypes.byref(cnt)), "timings")
    return [(names[i].decode(), float(ms[i])) for i in range(cnt.value)]


def launch_count() -> int:
    return int(load().sog_launch_count())


PLANS = _PlanCache()
_DIRECT = {}


def direct_ctx(device: int, dtype: int):
    key = (device, dtype)
    h = _DIRECT.get(key)
    if h is None:
        h = _vp()
        check(load().sog_direct_create(ctypes.byref(h), dtype, device), "sog_direct_create")
        _DIRECT[key] = h
    return h


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _host_i64(vals: Sequence[int]):
    if isinstance(vals, ctypes.Array):  # converted once and cached by the caller
        return vals
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def _host_f64(vals: Sequence[float]):
    if isinstance(vals, ctypes.Array):
        return vals
    return (ctypes.c_double * len(vals))(*[float(v) for v in vals])


def _host_nk(nk):
    if isinstance(nk, ctypes.Array):
        return nk
    return (ctypes.c_int32 * (3 * len(nk)))(*[int(v) for row in nk for v in row])


def host_tables(atom_begin, atom_count, k_sq_max, nk=None):
    """ctypes copies of a bucket's per-frame host arrays, made once per frame
    layout so that repeated calls pass them without conversion."""
    return dict(atom_begin=_host_i64(atom_begin), atom_count=_host_i64(atom_count),
                k_sq_max=_host_f64(k_sq_max), nk=None if nk is None else _host_nk(nk))


def _mesh_args(atom_begin, atom_count, k_sq_max, positions, charges, cells, amp, bw2, norm_factor,
               self_coeff, remove_self, k0_correction, charge_neutral_lambda, energy, forces,
               potential, grad_amp, grad_bw2, virial):
    nf = len(atom_begin)
    ab, ac, km = _host_i64(atom_begin), _host_i64(atom_count), _host_f64(k_sq_max)
    args = MeshArgs()
    args.nframes = nf
    args.atom_begin = ctypes.cast(ab, _c_i64p)
    args.atom_count = ctypes.cast(ac, _c_i64p)
    args.k_sq_max = ctypes.cast(km, _c_dp)
    args.nchannels = charges.shape[1]
    args.positions, args.charges, args.cells = _ptr(positions), _ptr(charges), _ptr(cells)
    args.n_gauss = amp.numel()
    args.amp, args.bw2 = _ptr(amp), _ptr(bw2)
    args.norm_factor, args.self_coeff = float(norm_factor), float(self_coeff)
    args.remove_self, args.k0_correction = int(remove_self), int(k0_correction)
    args.charge_neutral_lambda = float(charge_neutral_lambda or 0.0)
    args.energy, args.forces, args.potential = _ptr(energy), _ptr(forces), _ptr(potential)
    args.grad_amp, args.grad_bw2, args.virial = _ptr(grad_amp), _ptr(grad_bw2), _ptr(virial)
    return args, (ab, ac, km)


def slab_workspace_bytes(plan: "Plan", nfield: int, size: int, transport: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().sog_mesh_slab_workspace(plan.handle, int(nfield), int(size), int(transport),
                                         ctypes.byref(out)), "sog_mesh_slab_workspace")
    return int(out.value)


def mesh_slab_forward(plan: "Plan", group, *, atom_begin, atom_count, k_sq_max, positions, charges,
                      cells, amp, bw2, norm_factor, self_coeff, remove_self, k0_correction,
                      charge_neutral_lambda, energy, forces=None, potential=None, stream=None):
    """One frame split over the ranks of ``group`` (a ``sog_b200.slab.SlabGroup``).
    Forces / dE/dq come back for this rank's slab atoms only (others zero)."""
    _require_cuda(positions)
    args, keep = _mesh_args(atom_begin, atom_count, k_sq_max, positions, charges, cells, amp, bw2,
                            norm_factor, self_coeff, remove_self, k0_correction,
                            charge_neutral_lambda, energy, forces, potential, None, None, None)
    nfield = (3 if forces is not None else 0) + (1 if potential is not None else 0)
    ws = group.workspace(slab_workspace_bytes(plan, nfield, group.size, group.transport),
                         positions.device)
    cb = EXCHANGE_FN(group.callback(ws))
    desc = SlabDesc()
    desc.rank, desc.size, desc.transport = group.rank, group.size, group.transport
    desc.workspace, desc.workspace_bytes = ws.data_ptr(), ws.numel()
    desc.exchange, desc.ctx = cb, None
    if stream is None:
        stream = torch.cuda.current_stream(positions.device).cuda_stream
    rc = load().sog_mesh_slab_forward(plan.handle, ctypes.byref(args), ctypes.byref(desc),
                                      ctypes.c_void_p(stream))
    group.raise_pending()
    check(rc, "sog_mesh_slab_forward")
    del keep


def mesh_hvp(plan: Plan, *, atom_begin, atom_count, k_sq_max, positions, charges, cells, amp, bw2,
             norm_factor, self_coeff, remove_self, k0_correction, charge_neutral_lambda, dir_q, dir_r,
             dir_amp, dir_bw2, out_q, out_r, out_amp, out_bw2, stream=None, **_unused):
    """sog_mesh_hvp (B-spline / QuadS plans): the Hessian of every frame's
    mesh energy applied to the direction; outputs written in place."""
    _require_cuda(positions)
    args, keep = _mesh_args(atom_begin, atom_count, k_sq_max, positions, charges, cells, amp, bw2,
                            norm_factor, self_coeff, remove_self, k0_correction, charge_neutral_lambda,
                            None, None, None, None, None, None)
    h = _hvp_args(dir_q, dir_r, dir_amp, dir_bw2, out_q, out_r, out_amp, out_bw2)
    if stream is None:
        stream = torch.cuda.current_stream(positions.device).cuda_stream
    check(load().sog_mesh_hvp(plan.handle, ctypes.byref(args), ctypes.byref(h), ctypes.c_void_p(stream)),
          "sog_mesh_hvp")
    del keep


def mesh_forward(plan: Plan, *, atom_begin, atom_count, k_sq_max, positions, charges, cells, amp,
                 bw2, norm_factor, self_coeff, remove_self, k0_correction, charge_neutral_lambda,
                 energy, forces=None, potential=None, grad_amp=None, grad_bw2=None, virial=None,
                 dedr=None, stream=None):
    """One C-ABI mesh call.  All tensors must be contiguous CUDA tensors of the
    plan dtype; outputs are written in place."""
    _require_cuda(positions)
    args, keep = _mesh_args(atom_begin, atom_count, k_sq_max, positions, charges, cells, amp, bw2,
                            norm_factor, self_coeff, remove_self, k0_correction, charge_neutral_lambda,
                            energy, forces, potential, grad_amp, grad_bw2, virial)
    args.dedr = _ptr(dedr)
    if stream is None:
        stream = torch.cuda.current_stream(positions.device).cuda_stream
    check(load().sog_mesh_forward(plan.handle, ctypes.byref(args), ctypes.c_void_p(stream)),
          "sog_mesh_forward")
    del keep


def direct_forward(ctx, *, atom_begin, atom_count, nk, k_sq_max, positions, charges, cells, amp,
                   bw2, norm_factor, self_coeff, remove_self, k0_correction,
                   charge_neutral_lambda, energy, forces=None, potential=None, grad_amp=None,
                   grad_bw2=None, virial=None, stream=None):
    _require_cuda(positions)
    nf = len(atom_begin)
    ab, ac, km = _host_i64(atom_begin), _host_i64(atom_count), _host_f64(k_sq_max)
    nkflat = _host_nk(nk)
    args = DirectArgs()
    args.nframes = nf
    args.atom_begin = ctypes.cast(ab, _c_i64p)
    args.atom_count = ctypes.cast(ac, _c_i64p)
    args.nk = ctypes.cast(nkflat, _c_i32p)
    args.k_sq_max = ctypes.cast(km, _c_dp)
    args.nchannels = charges.shape[1]
    args.positions, args.charges, args.cells = _ptr(positions), _ptr(charges), _ptr(cells)
    args.n_gauss = amp.numel()
    args.amp, args.bw2 = _ptr(amp), _ptr(bw2)
    args.norm_factor, args.self_coeff = float(norm_factor), float(self_coeff)
    args.remove_self, args.k0_correction = int(remove_self), int(k0_correction)
    args.charge_neutral_lambda = float(charge_neutral_lambda or 0.0)
    args.energy, args.forces, args.potential = _ptr(energy), _ptr(forces), _ptr(potential)
    args.grad_amp, args.grad_bw2, args.virial = _ptr(grad_amp), _ptr(grad_bw2), _ptr(virial)
    if stream is None:
        stream = torch.cuda.current_stream(positions.device).cuda_stream
    check(load().sog_direct_forward(ctx, ctypes.byref(args), ctypes.c_void_p(stream)),
          "sog_direct_forward")


def realspace_forward(ctx, *, atom_begin, atom_count, positions, charges, amp, bw2, norm_factor,
                      remove_self, charge_neutral_lambda, energy, forces=None, potential=None,
                      grad_amp=None, grad_bw2=None, virial=None, stream=None, **_unused):
    """sog_realspace_forward on a direct-solver context (non-periodic frames)."""
    _require_cuda(positions)
    nf = len(atom_begin)
    ab, ac = _host_i64(atom_begin), _host_i64(atom_count)
    args = RealspaceArgs()
    args.nframes = nf
    args.atom_begin = ctypes.cast(ab, _c_i64p)
    args.atom_count = ctypes.cast(ac, _c_i64p)
    args.nchannels = charges.shape[1]
    args.positions, args.charges = _ptr(positions), _ptr(charges)
    args.n_gauss = amp.numel()
    args.amp, args.bw2 = _ptr(amp), _ptr(bw2)
    args.norm_factor = float(norm_factor)
    args.remove_self = int(remove_self)
    args.charge_neutral_lambda = float(charge_neutral_lambda or 0.0)
    args.energy, args.forces, args.potential = _ptr(energy), _ptr(forces), _ptr(potential)
    args.grad_amp, args.grad_bw2, args.virial = _ptr(grad_amp), _ptr(grad_bw2), _ptr(virial)
    if stream is None:
        stream = torch.cuda.current_stream(positions.device).cuda_stream
    check(load().sog_realspace_forward(ctx, ctypes.byref(args), ctypes.c_void_p(stream)),
          "sog_realspace_forward")


def _hvp_args(dir_q, dir_r, dir_amp, dir_bw2, out_q, out_r, out_amp, out_bw2):
    h = HvpArgs()
    h.dir_q, h.dir_r, h.dir_amp, h.dir_bw2 = _ptr(dir_q), _ptr(dir_r), _ptr(dir_amp), _ptr(dir_bw2)
    h.out_q, h.out_r, h.out_amp, h.out_bw2 = _ptr(out_q), _ptr(out_r), _ptr(out_amp), _ptr(out_bw2)
    return h


def direct_hvp(ctx, *, atom_begin, atom_count, nk, k_sq_max, positions, charges, cells, amp, bw2,
               norm_factor, self_coeff, remove_self, k0_correction, charge_neutral_lambda, dir_q, dir_r,
               dir_amp, dir_bw2, out_q, out_r, out_amp, out_bw2, stream=None, **_unused):
    """sog_direct_hvp: the Hessian of every frame's energy applied to the
    direction (dir_q, dir_r, dir_amp[f], dir_bw2[f]); outputs written in place."""
    _require_cuda(positions)
    nf = len(atom_begin)
    ab, ac, km = _host_i64(atom_begin), _host_i64(atom_count), _host_f64(k_sq_max)
    nkflat = _host_nk(nk)
    args = DirectArgs()
    args.nframes = nf
    args.atom_begin = ctypes.cast(ab, _c_i64p)
    args.atom_count = ctypes.cast(ac, _c_i64p)
    args.nk = ctypes.cast(nkflat, _c_i32p)
    args.k_sq_max = ctypes.cast(km, _c_dp)
    args.nchannels = charges.shape[1]
    args.positions, args.charges, args.cells = _ptr(positions), _ptr(charges), _ptr(cells)
    args.n_gauss = amp.numel()
    args.amp, args.bw2 = _ptr(amp), _ptr(bw2)
    args.norm_factor, args.self_coeff = float(norm_factor), float(self_coeff)
    args.remove_self, args.k0_correction = int(remove_self), int(k0_correction)
    args.charge_neutral_lambda = float(charge_neutral_lambda or 0.0)
    h = _hvp_args(dir_q, dir_r, dir_amp, dir_bw2, out_q, out_r, out_amp, out_bw2)
    if stream is None:
        stream = torch.cuda.current_stream(positions.device).cuda_stream
    check(load().sog_direct_hvp(ctx, ctypes.byref(args), ctypes.byref(h), ctypes.c_void_p(stream)),
          "sog_direct_hvp")


def realspace_hvp(ctx, *, atom_begin, atom_count, positions, charges, amp, bw2, norm_factor, remove_self,
                  charge_neutral_lambda, dir_q, dir_r, dir_amp, dir_bw2, out_q, out_r, out_amp, out_bw2,
                  stream=None, **_unused):
    """sog_realspace_hvp on a direct-solver context (non-periodic frames)."""
    _require_cuda(positions)
    nf = len(atom_begin)
    ab, ac = _host_i64(atom_begin), _host_i64(atom_count)
    args = RealspaceArgs()
    args.nframes = nf
    args.atom_begin = ctypes.cast(ab, _c_i64p)
    args.atom_count = ctypes.cast(ac, _c_i64p)
    args.nchannels = charges.shape[1]
    args.positions, args.charges = _ptr(positions), _ptr(charges)
    args.n_gauss = amp.numel()
    args.amp, args.bw2 = _ptr(amp), _ptr(bw2)
    args.norm_factor = float(norm_factor)
    args.remove_self = int(remove_self)
    args.charge_neutral_lambda = float(charge_neutral_lambda or 0.0)
    h = _hvp_args(dir_q, dir_r, dir_amp, dir_bw2, out_q, out_r, out_amp, out_bw2)
    if stream is None:
        stream = torch.cuda.current_stream(positions.device).cuda_stream
    check(load().sog_realspace_hvp(ctx, ctypes.byref(args), ctypes.byref(h), ctypes.c_void_p(stream)),
          "sog_realspace_hvp")
