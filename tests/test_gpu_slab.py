"""z-slab decomposition of one frame (``mesh_decomposition="slab"``) against
the single-device mesh path on the same inputs.

With one process the slab path runs every exchange as a local copy, which
checks the slab kernels (z-range spread, pack / unpack, y-slab Green table and
fused z pass, halo planes, slab gather and dE/dq) on one GPU.  With two or
more GPUs the same comparison runs over NCCL in child processes.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

E_RTOL = 1e-12
F_ATOL = 1e-11


def _system(n, L, seed, tric=False, nch=1):
    rng = np.random.default_rng(seed)
    if tric:
        cell = np.array([[L, 0.0, 0.0], [0.9, L * 1.05, 0.0], [-0.7, 1.1, L * 0.97]])
    else:
        cell = np.eye(3) * L
    r = rng.random((n, 3)) @ cell
    q = rng.normal(size=(n, nch))
    q -= q.mean(axis=0)
    return r, q, cell


def _gauss(decomp, order=6, n_dl=1.0, transport="peer"):
    from sog_b200 import Gaussian
    bw = 1.2 * 1.62 ** np.arange(8)
    amp = 1.0 / (bw * np.sqrt(2 * np.pi))
    return Gaussian(n_dl=n_dl, amp=torch.tensor(amp), bandwidth=torch.tensor(bw),
                    use_bspline_fft=True, bspline_order=order, trainable=False,
                    mesh_decomposition=decomp, slab_transport=transport)


def _solve(decomp, r, q, cell, dev, order=6, want_pot=False, transport="peer"):
    g = _gauss(decomp, order, transport=transport).to(dev)
    rt = torch.tensor(r, device=dev)
    qt = torch.tensor(q, device=dev, requires_grad=want_pot)
    ct = torch.tensor(cell[None], device=dev)
    out = g.compute_bundle(q=qt, r=rt, cell=ct, compute_force=True)
    pot = None
    if want_pot:
        (pot,) = torch.autograd.grad(out["energy"].sum(), qt)
    return out["energy"].detach(), out["forces"].detach(), pot


@pytest.mark.parametrize("tric,order,nch,transport", [(False, 6, 1, "peer"), (False, 6, 1, "exchange"),
                                                     (True, 4, 1, "exchange"), (False, 5, 2, "peer")])
def test_slab_one_rank_matches_mesh(tric, order, nch, transport):
    dev = torch.device("cuda:0")
    r, q, cell = _system(2500, 31.0, 11, tric, nch)
    e0, f0, p0 = _solve("none", r, q, cell, dev, order, want_pot=True)
    e1, f1, p1 = _solve("slab", r, q, cell, dev, order, want_pot=True, transport=transport)
    torch.testing.assert_close(e1, e0, rtol=E_RTOL, atol=0.0)
    torch.testing.assert_close(f1, f0, rtol=0.0, atol=F_ATOL)
    torch.testing.assert_close(p1, p0, rtol=0.0, atol=F_ATOL)
    assert float(f0.abs().max()) > 1e-3


def test_slab_rejects_parameter_gradients():
    dev = torch.device("cuda:0")
    r, q, cell = _system(300, 31.0, 3)
    from sog_b200 import Gaussian
    g = Gaussian(n_dl=1.0, use_bspline_fft=True, trainable=True, mesh_decomposition="slab").to(dev)
    out = None
    with pytest.raises(NotImplementedError):
        out = g.compute_bundle(q=torch.tensor(q, device=dev), r=torch.tensor(r, device=dev),
                               cell=torch.tensor(cell[None], device=dev), compute_force=True,
                               compute_virial=True)
    assert out is None


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _child(rank, world, port, tric, transport, res):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        r, q, cell = _system(3000, 31.0, 5, tric)
        e0, f0, p0 = _solve("none", r, q, cell, dev, 6, want_pot=True)
        e1, f1, p1 = _solve("slab", r, q, cell, dev, 6, want_pot=True, transport=transport)
        err = [float((e1 - e0).abs().max() / e0.abs().max()), float((f1 - f0).abs().max()),
               float((p1 - p0).abs().max())]
        res[rank] = err
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("tric,transport", [(False, "peer"), (False, "exchange"), (True, "exchange")])
def test_slab_two_ranks_nccl(tric, transport):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        res = man.dict()
        port = _free_port()
        procs = [ctx.Process(target=_child, args=(k, 2, port, tric, transport, res)) for k in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        for k in range(2):
            e_rel, f_abs, p_abs = res[k]
            assert e_rel <= E_RTOL and f_abs <= F_ATOL and p_abs <= F_ATOL, (k, res[k])
