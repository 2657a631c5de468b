"""Host side of the z-slab decomposition on CPU: the exchange callback of
``sog_b200.slab.SlabGroup`` over two ``gloo`` ranks (the contract in
include/sog_b200.h: all-to-all block order, halo direction, in-place sum,
failure reporting), and the one-process fallback."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")

from sog_b200 import _lib  # noqa: E402
from sog_b200.slab import SlabGroup  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        g = SlabGroup()
        assert (g.rank, g.size) == (rank, world)
        ws = g.workspace(4096, torch.device("cpu"))
        ws.zero_()
        blk = 16
        # all-to-all: block k of this rank holds 10*rank + k
        for k in range(world):
            ws[k * blk:(k + 1) * blk] = 10 * rank + k
        g.exchange(ws, _lib.EXCH_ALLTOALL, 0, 1024, blk)
        got = [int(ws[1024 + k * blk]) for k in range(world)]
        # halo: send 8 bytes of value 100+rank to rank-1, receive from rank+1
        ws[2048:2056] = 100 + rank
        g.exchange(ws, _lib.EXCH_HALO, 2048, 2560, 8)
        halo = int(ws[2560])
        # in-place sum of doubles
        d = ws[3072:3072 + 24].view(torch.float64)
        d[:] = torch.tensor([1.0, rank, 2.5 * rank], dtype=torch.float64)
        g.exchange(ws, _lib.EXCH_SUM_F64, 3072, 3072, 24)
        sums = ws[3072:3072 + 24].view(torch.float64).tolist()
        # all-gather: 8 bytes of value 50+rank from every rank, rank-major
        ws[3584:3592] = 50 + rank
        g.exchange(ws, _lib.EXCH_ALLGATHER, 3584, 3712, 8)
        gathered = [int(ws[3712 + 8 * k]) for k in range(world)]
        # the C callback reports a failure as status 1 and keeps the exception
        fn = g.callback(ws)
        bad = fn(None, 99, 0, 0, 8, None)
        pending = None
        try:
            g.raise_pending()
        except ValueError as exc:
            pending = str(exc)
        out[rank] = (got, halo, sums, bad, pending, gathered)
    finally:
        dist.destroy_process_group()


def test_exchange_two_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    world = 2
    with ctx.Manager() as man:
        out = man.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(k, world, port, out)) for k in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        for r in range(world):
            got, halo, sums, bad, pending, gathered = out[r]
            assert got == [10 * k + r for k in range(world)]       # rank k's block r, rank-major
            assert halo == 100 + (r + 1) % world                     # from rank r+1
            assert sums == [2.0, 1.0, 2.5]
            assert bad == 1 and "unknown exchange kind" in pending
            assert gathered == [50 + k for k in range(world)]


def test_exchange_one_process_is_local_copy():
    g = SlabGroup()
    assert (g.rank, g.size) == (0, 1) and g.transport == _lib.SLAB_PEER
    with pytest.raises(ValueError):
        SlabGroup(transport="smoke-signals")
    ws = g.workspace(256, torch.device("cpu"))
    ws[:64] = torch.arange(64, dtype=torch.uint8)
    g.exchange(ws, _lib.EXCH_ALLTOALL, 0, 128, 64)
    assert torch.equal(ws[128:192], ws[:64])
    ws[64:72] = 7
    g.exchange(ws, _lib.EXCH_HALO, 64, 200, 8)
    assert int(ws[200]) == 7
    before = ws.clone()
    g.exchange(ws, _lib.EXCH_SUM_F64, 0, 0, 16)
    assert torch.equal(ws, before)
    assert g.workspace(128, torch.device("cpu")) is ws       # reused while large enough
