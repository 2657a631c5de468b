"""sog_direct_forward_noalloc through the C ABI.

The no-allocation entry point is for callers that may not allocate memory
inside a force call (an MD engine that owns all device memory in its own
arena, or runs where cudaMalloc could block on queued work or fail mid-run).
It keeps its scratch in a fixed file-scope device array, so this file checks:

  * it gives the same energies and derivatives as the allocating entry point
    sog_direct_forward on the same inputs, on two calls in a row (the second
    call reuses the scratch the first one left behind), in fp64 and fp32,
    for ragged frames, for 64 frames of at most 32 atoms (the one-warp atom
    kernel) and for a mode box large enough for the block-tree reductions;
    every reduction of a call that fits the 8 MiB array takes one pass (its
    mode boxes stay far below the size that splits a reduction);
  * it matches reference-made fixtures of the direct k-sum (energies, forces,
    dE/dq) at the usual tolerances;
  * a call after the first one on a device allocates nothing: neither torch's
    allocator statistics nor the device's free memory change across it (the
    first call may load the module, and with it the array, into the context);
  * the optional caller-owned status word reports non-finite inputs;
  * a call with more than 64 frames, or whose scratch would not fit, is
    rejected before anything is launched.

Collected last so that a run that stops at the first failure has run every
other test first; it passes both alone and after the other GPU tests.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from sog_b200 import _lib  # noqa: E402
from tests._cases import direct_n_dl, direct_nk, load  # noqa: E402

pytestmark = pytest.mark.gpu

NORM = 14.3996454784255


def _tol(dtype):
    # same kernels and reduction order as the allocating entry point
    return (dict(rtol=1e-12, atol=1e-13) if dtype == torch.float64 else dict(rtol=1e-6, atol=1e-6))


def _inputs(dev, dtype=torch.float64, seed=7, counts=(37, 52), nk=((5, 6, 7), (6, 5, 5)), nch=2):
    rng = np.random.default_rng(seed)
    nf = len(counts)
    cells, pos, q = [], [], []
    for f, n in enumerate(counts):
        cell = np.diag(rng.uniform(9.0, 13.0, 3))
        cell[1, 0], cell[2, 0], cell[2, 1] = rng.uniform(-1.2, 1.2, 3)
        cells.append(cell)
        pos.append(rng.random((n, 3)) @ cell)
        qq = rng.normal(size=(n, nch))
        q.append(qq - qq.mean(axis=0))
    amp = rng.uniform(0.2, 1.0, 6)
    bw2 = np.geomspace(0.8, 40.0, 6)
    t = lambda a: torch.tensor(np.ascontiguousarray(a), dtype=dtype, device=dev)
    begins = list(np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(int))
    return dict(counts=list(counts), begins=begins, nk=[list(v) for v in nk],
                ksq=[(2 * np.pi / 1.5) ** 2] * nf, nch=nch, self_coeff=1.0 / np.sqrt(np.pi),
                remove_self=1, lam=0.0, pos=t(np.concatenate(pos)), q=t(np.concatenate(q)),
                cells=t(np.stack(cells)), amp=t(amp), bw2=t(bw2))


def _outputs(dev, n, nf, m, nch, dtype=torch.float64):
    z = lambda *s: torch.zeros(*s, dtype=dtype, device=dev)
    return dict(energy=z(nf), forces=z(n, 3), potential=z(n, nch), grad_amp=z(nf, m),
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
    a.nchannels = inp["nch"]
    p = lambda x: ctypes.c_void_p(x.data_ptr())
    a.positions, a.charges, a.cells = p(inp["pos"]), p(inp["q"]), p(inp["cells"])
    a.n_gauss = inp["amp"].numel()
    a.amp, a.bw2 = p(inp["amp"]), p(inp["bw2"])
    a.norm_factor, a.self_coeff = NORM, float(inp["self_coeff"])
    a.remove_self, a.k0_correction = int(inp["remove_self"]), 1
    a.charge_neutral_lambda = float(inp["lam"])
    for k in ("energy", "forces", "potential", "grad_amp", "grad_bw2", "virial"):
        setattr(a, k, p(out[k]) if k in out else None)
    return a


def _noalloc(lib):
    fn = lib.sog_direct_forward_noalloc
    fn.argtypes = [ctypes.c_int, ctypes.POINTER(_lib.DirectArgs), ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _dcode(dtype):
    return _lib.DTYPE_F64 if dtype == torch.float64 else _lib.DTYPE_F32


def _compare_with_direct(inp, dtype):
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _lib.load()
    n, nf, m, nch = inp["pos"].shape[0], len(inp["counts"]), inp["amp"].numel(), inp["nch"]
    keep = []
    ref = _outputs(dev, n, nf, m, nch, dtype)
    ctx = _lib.direct_ctx(0, _dcode(dtype))
    _lib.check(lib.sog_direct_forward(ctx, ctypes.byref(_args(inp, ref, keep)), _stream(dev)),
               "sog_direct_forward")
    fn = _noalloc(lib)
    status = torch.full((1,), 0xFFFF, dtype=torch.int32, device=dev)
    for call in range(2):
        out = _outputs(dev, n, nf, m, nch, dtype)
        _lib.check(fn(_dcode(dtype), ctypes.byref(_args(inp, out, keep)),
                      ctypes.c_void_p(status.data_ptr()), _stream(dev)),
                   "sog_direct_forward_noalloc")
        torch.cuda.synchronize()
        assert int(status.item()) == 0, call
        for k in ref:
            assert torch.isfinite(out[k]).all(), (call, k)
            torch.testing.assert_close(out[k], ref[k], **_tol(dtype), msg=f"call {call}, {k}")
    assert float(ref["energy"].abs().min()) > 0.0


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_noalloc_matches_direct_twice(dtype):
    _compare_with_direct(_inputs("cuda:0", dtype), dtype)


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_noalloc_matches_direct_64_tiny_frames(dtype):
    rng = np.random.default_rng(11)
    counts = [int(c) for c in rng.integers(2, 33, 64)]   # neutral frames of one atom have zero energy
    nk = [tuple(int(v) for v in rng.integers(2, 6, 3)) for _ in range(64)]
    _compare_with_direct(_inputs("cuda:0", dtype, seed=12, counts=counts, nk=nk, nch=1), dtype)


def test_noalloc_matches_direct_large_mode_box():
    # 21 x 41 x 41 modes per frame: 138 partial blocks, reduced by the block tree
    _compare_with_direct(_inputs("cuda:0", torch.float64, seed=5, counts=(90, 70),
                                 nk=((20, 20, 20), (18, 20, 19))), torch.float64)


@pytest.mark.parametrize("name", ["cfg1_direct", "direct_triclinic_2ch_rsi1", "direct_mixed_batch"])
def test_noalloc_matches_reference_fixture(name):
    """The direct k-sum fixtures made by running the reference (energy,
    autograd forces and dE/dq with per-frame weights)."""
    c = load(name)
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _lib.load()
    q = c["q"] if c["q"].ndim == 2 else c["q"][:, None]
    batch = c["batch"]
    order = np.argsort(batch, kind="stable")
    nf = int(batch.max()) + 1
    counts = [int((batch == f).sum()) for f in range(nf)]
    cells = c["cell"].reshape(-1, 3, 3)
    n_dl = direct_n_dl(c)
    t = lambda a: torch.tensor(np.ascontiguousarray(a), dtype=torch.float64, device=dev)
    inp = dict(counts=counts, begins=list(np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(int)),
               nk=[direct_nk(cl, n_dl) for cl in cells], ksq=[(2 * np.pi / n_dl) ** 2] * nf,
               nch=q.shape[1], self_coeff=float(c["self_coeff"]), remove_self=int(c["remove_self"]),
               lam=max(float(c["lam"]), 0.0), pos=t(c["r"][order]), q=t(q[order]), cells=t(cells),
               amp=t(c["amp"]), bw2=t(c["bw2"]))
    n, m = len(order), inp["amp"].numel()
    out = _outputs(dev, n, nf, m, inp["nch"])
    keep = []
    _lib.check(_noalloc(lib)(_lib.DTYPE_F64, ctypes.byref(_args(inp, out, keep)), None, _stream(dev)),
               "sog_direct_forward_noalloc")
    torch.cuda.synchronize()
    e = out["energy"].cpu().numpy()
    assert np.max(np.abs(e - c["energy"])) <= 1e-10 * np.max(np.abs(c["energy"]))
    w = c["grad_weights"][batch[order]]
    f = out["forces"].cpu().numpy() * w[:, None]
    assert np.abs(f - c["forces"][order]).max() < 1e-9
    gq = out["potential"].cpu().numpy() * w[:, None]
    assert np.abs(gq - c["grad_q"].reshape(q.shape)[order]).max() < 1e-9


def test_noalloc_allocates_nothing_after_the_first_call():
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _lib.load()
    fn = _noalloc(lib)
    inp = _inputs(dev)
    n, nf, m = inp["pos"].shape[0], 2, inp["amp"].numel()
    keep = []
    outs = [_outputs(dev, n, nf, m, 2) for _ in range(3)]
    args = [_args(inp, o, keep) for o in outs]
    _lib.check(fn(_lib.DTYPE_F64, ctypes.byref(args[0]), None, _stream(dev)), "first call")
    torch.cuda.synchronize()
    stats0 = torch.cuda.memory_stats(dev)
    free0, _ = torch.cuda.mem_get_info(dev)
    for a in args[1:]:
        _lib.check(fn(_lib.DTYPE_F64, ctypes.byref(a), None, _stream(dev)), "later call")
    torch.cuda.synchronize()
    stats1 = torch.cuda.memory_stats(dev)
    free1, _ = torch.cuda.mem_get_info(dev)
    for k in ("allocation.all.allocated", "reserved_bytes.all.current", "allocated_bytes.all.current"):
        assert stats1.get(k, 0) == stats0.get(k, 0), k
    assert free1 == free0
    torch.testing.assert_close(outs[2]["energy"], outs[0]["energy"], rtol=0, atol=0)


def test_noalloc_status_word_reports_nonfinite_input():
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _lib.load()
    inp = _inputs(dev)
    inp["pos"][5, 1] = float("nan")
    n, nf, m = inp["pos"].shape[0], 2, inp["amp"].numel()
    out = _outputs(dev, n, nf, m, 2)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    keep = []
    _lib.check(_noalloc(lib)(_lib.DTYPE_F64, ctypes.byref(_args(inp, out, keep)),
                             ctypes.c_void_p(status.data_ptr()), _stream(dev)),
               "sog_direct_forward_noalloc")
    torch.cuda.synchronize()
    assert int(status.item()) & 1  # SOG_STATUS_NONFINITE


@pytest.mark.parametrize("what", ["scratch", "frames"])
def test_noalloc_rejects_oversized_call(what):
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _lib.load()
    if what == "scratch":
        # 61 x 121 x 121 modes: far beyond the fixed scratch
        inp = _inputs(dev, nk=((60, 60, 60), (6, 5, 5)))
    else:
        inp = _inputs(dev, counts=[3] * 65, nk=[(2, 2, 2)] * 65, nch=1)
    n, nf, m = inp["pos"].shape[0], len(inp["counts"]), inp["amp"].numel()
    keep = []
    out = _outputs(dev, n, nf, m, inp["nch"])
    before = lib.sog_launch_count()
    rc = _noalloc(lib)(_lib.DTYPE_F64, ctypes.byref(_args(inp, out, keep)), None, _stream(dev))
    assert rc == 1  # SOG_ERR_INVALID
    assert (b"scratch" if what == "scratch" else b"64 frames") in lib.sog_last_error()
    assert lib.sog_launch_count() == before
    torch.cuda.synchronize()
    assert float(out["energy"].abs().max()) == 0.0
