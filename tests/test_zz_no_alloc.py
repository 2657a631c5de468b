"""sog_direct_forward_noalloc against sog_direct_forward, through the C ABI.

The no-allocation entry point keeps its scratch in a fixed file-scope device
array; it must give the same energies and derivatives as the allocating entry
point on the same inputs, on two calls in a row (the second call reuses the
scratch the first one left behind), and reject a call whose scratch would not
fit before launching anything.  Collected last so that it runs both alone and
after the other GPU tests.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from sog_b200 import _lib  # noqa: E402

pytestmark = pytest.mark.gpu

RTOL = 1e-12  # same kernels, same reduction order: agreement to rounding
ATOL = 1e-13


def _inputs(dev, seed=7):
    rng = np.random.default_rng(seed)
    counts = [37, 52]
    cells = np.stack([
        np.array([[11.0, 0.0, 0.0], [1.2, 12.5, 0.0], [-0.8, 0.9, 10.4]]),
        np.diag([13.0, 11.5, 12.2]),
    ])
    pos, q = [], []
    for f, n in enumerate(counts):
        frac = rng.random((n, 3))
        pos.append(frac @ cells[f])
        qq = rng.normal(size=(n, 2))
        q.append(qq - qq.mean(axis=0))
    amp = rng.uniform(0.2, 1.0, 6)
    bw2 = np.geomspace(0.8, 40.0, 6)
    t = lambda a: torch.tensor(np.ascontiguousarray(a), dtype=torch.float64, device=dev)
    return dict(counts=counts, begins=[0, counts[0]], nk=[[5, 6, 7], [6, 5, 5]],
                ksq=[(2 * np.pi / 1.6) ** 2, (2 * np.pi / 1.5) ** 2],
                pos=t(np.concatenate(pos)), q=t(np.concatenate(q)), cells=t(cells),
                amp=t(amp), bw2=t(bw2))


def _outputs(dev, n, nf, m):
    z = lambda *s: torch.zeros(*s, dtype=torch.float64, device=dev)
    return dict(energy=z(nf), forces=z(n, 3), potential=z(n, 2), grad_amp=z(nf, m),
                grad_bw2=z(nf, m), virial=z(nf, 3, 3))


def _args(inp, out, keep):
    nf = len(inp["counts"])
    a = _lib.DirectArgs()
    keep += [(ctypes.c_int64 * nf)(*inp["begins"]), (ctypes.c_int64 * nf)(*inp["counts"]),
             (ctypes.c_int32 * (3 * nf))(*[v for row in inp["nk"] for v in row]),
             (ctypes.c_double * nf)(*inp["ksq"])]
    a.nframes = nf
    a.atom_begin = ctypes.cast(keep[-4], _lib._c_i64p)
    a.atom_count = ctypes.cast(keep[-3], _lib._c_i64p)
    a.nk = ctypes.cast(keep[-2], _lib._c_i32p)
    a.k_sq_max = ctypes.cast(keep[-1], _lib._c_dp)
    a.nchannels = 2
    p = lambda x: ctypes.c_void_p(x.data_ptr())
    a.positions, a.charges, a.cells = p(inp["pos"]), p(inp["q"]), p(inp["cells"])
    a.n_gauss = inp["amp"].numel()
    a.amp, a.bw2 = p(inp["amp"]), p(inp["bw2"])
    a.norm_factor, a.self_coeff = 14.3996454784255, 1.0 / np.sqrt(np.pi)
    a.remove_self, a.k0_correction = 1, 1
    a.charge_neutral_lambda = 0.0
    for k in ("energy", "forces", "potential", "grad_amp", "grad_bw2", "virial"):
        setattr(a, k, p(out[k]))
    return a


def _noalloc(lib):
    fn = lib.sog_direct_forward_noalloc
    fn.argtypes = [ctypes.c_int, ctypes.POINTER(_lib.DirectArgs), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def test_noalloc_matches_direct_twice():
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _lib.load()
    inp = _inputs(dev)
    n, nf, m = inp["pos"].shape[0], 2, inp["amp"].numel()
    keep = []
    ref = _outputs(dev, n, nf, m)
    ctx = _lib.direct_ctx(0, _lib.DTYPE_F64)
    _lib.check(lib.sog_direct_forward(ctx, ctypes.byref(_args(inp, ref, keep)), _stream(dev)),
               "sog_direct_forward")
    fn = _noalloc(lib)
    for call in range(2):
        out = _outputs(dev, n, nf, m)
        _lib.check(fn(_lib.DTYPE_F64, ctypes.byref(_args(inp, out, keep)), _stream(dev)),
                   "sog_direct_forward_noalloc")
        torch.cuda.synchronize()
        for k in ref:
            assert torch.isfinite(out[k]).all(), (call, k)
            torch.testing.assert_close(out[k], ref[k], rtol=RTOL, atol=ATOL, msg=f"call {call}, {k}")
    assert float(ref["energy"].abs().min()) > 0.0


def test_noalloc_rejects_oversized_call():
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _lib.load()
    inp = _inputs(dev)
    inp["nk"] = [[60, 60, 60], [6, 5, 5]]  # 61*121*121 modes: far beyond the fixed scratch
    n, nf, m = inp["pos"].shape[0], 2, inp["amp"].numel()
    keep = []
    out = _outputs(dev, n, nf, m)
    before = lib.sog_launch_count()
    rc = _noalloc(lib)(_lib.DTYPE_F64, ctypes.byref(_args(inp, out, keep)), _stream(dev))
    assert rc == 1  # SOG_ERR_INVALID
    assert b"scratch" in lib.sog_last_error()
    assert lib.sog_launch_count() == before
    torch.cuda.synchronize()
    assert float(out["energy"].abs().max()) == 0.0
