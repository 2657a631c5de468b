"""Host side of sharding independent frames over data-parallel ranks
(``sog_b200.shard``) on CPU: the longest-processing-time partition and the
select / gather round trip over two ``gloo`` ranks, with a stand-in per-frame
computation in place of the solver."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from sog_b200.shard import FrameShards, frame_costs, lpt_partition  # noqa: E402


def test_lpt_partition_covers_every_frame_once_and_balances():
    rng = np.random.default_rng(3)
    costs = rng.uniform(1.0, 100.0, 97).tolist()
    for world in (1, 2, 3, 8):
        parts = lpt_partition(costs, world)
        flat = sorted(j for p in parts for j in p)
        assert flat == list(range(len(costs)))
        loads = [sum(costs[j] for j in p) for p in parts]
        # LPT bound: max load <= mean load + largest single cost
        assert max(loads) <= sum(costs) / world + max(costs) + 1e-9
        assert parts == lpt_partition(costs, world)  # deterministic
    assert lpt_partition([5.0, 1.0], 4)[2:] == [[], []]
    with pytest.raises(ValueError):
        lpt_partition([1.0], 0)


def test_frame_costs():
    c = frame_costs([100, 200], [4096, 32768], order=6)
    assert c[0] == pytest.approx(4096 * 12 + 216 * 100)
    assert c[1] > c[0]
    assert frame_costs([3, 5]) == [3.0, 5.0]


def _fake_solve(r, q, batch, nf):
    """Per-frame sum of q |r|^2 and per-atom q r (stands in for the solver)."""
    e = torch.zeros(nf, dtype=r.dtype)
    e.index_add_(0, batch, q[:, 0] * (r * r).sum(1))
    return e, q * r


def _batch_of(counts):
    return torch.repeat_interleave(torch.arange(len(counts)), torch.tensor(counts))


def test_frame_shards_one_rank_is_identity():
    counts = [4, 1, 7, 3]
    n = sum(counts)
    r = torch.randn(n, 3, dtype=torch.float64)
    q = torch.randn(n, 1, dtype=torch.float64)
    sh = FrameShards(counts, lpt_partition(frame_costs(counts), 1), 0, torch.device("cpu"))
    rl, ql, _, bl = sh.select(r, q, None)
    e, f = _fake_solve(rl, ql, bl, len(sh.frames))
    e0, f0 = _fake_solve(r, q, _batch_of(counts), len(counts))
    assert torch.equal(sh.gather_energy(e), e0)
    assert torch.equal(sh.gather_atoms(f), f0)


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
        gen = torch.Generator().manual_seed(5)
        counts = torch.randint(1, 40, (23,), generator=gen).tolist()
        n = sum(counts)
        r = torch.randn(n, 3, dtype=torch.float64, generator=gen)
        q = torch.randn(n, 1, dtype=torch.float64, generator=gen)
        cells = torch.randn(len(counts), 3, 3, dtype=torch.float64, generator=gen)
        sh = FrameShards(counts, lpt_partition(frame_costs(counts), world), rank, torch.device("cpu"))
        rl, ql, cl, bl = sh.select(r, q, cells)
        assert torch.equal(cl, cells[sh.frames])
        e, f = _fake_solve(rl, ql, bl, len(sh.frames))
        e_all = sh.gather_energy(e)
        f_all = sh.gather_atoms(f)
        e0, f0 = _fake_solve(r, q, _batch_of(counts), len(counts))
        out[rank] = (bool(torch.equal(e_all, e0)), bool(torch.equal(f_all, f0)), len(sh.frames))
    finally:
        dist.destroy_process_group()


def test_frame_shards_two_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        out = man.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(k, 2, port, out)) for k in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        for k in range(2):
            e_ok, f_ok, nfr = out[k]
            assert e_ok and f_ok, (k, out[k])
        assert out[0][2] + out[1][2] == 23 and min(out[0][2], out[1][2]) > 0
