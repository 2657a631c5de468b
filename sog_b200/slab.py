"""Ranks that share one large frame's mesh (z-slab decomposition).

``SlabGroup`` is the caller side of ``sog_mesh_slab_forward``: it owns the
device workspace the library exchanges through and implements the exchange
callback with ``torch.distributed`` collectives (NCCL between GPUs; any
backend that has ``all_to_all_single`` and point-to-point for host tensors).
With one process (no initialised process group, or a group of size 1) every
exchange is a local copy, so the slab path also runs on one GPU.

Exchange kinds (the contract of ``include/sog_b200.h``):

* ``EXCH_ALLTOALL``: block k of ``bytes`` at ``send_off + k*bytes`` goes to
  rank k; rank k's block lands at ``recv_off + k*bytes``;
* ``EXCH_HALO``: ``bytes`` at ``send_off`` go to rank r-1, rank r+1's land at
  ``recv_off`` (ranks mod size);
* ``EXCH_SUM_F64``: in-place sum over ranks of ``bytes/8`` doubles;
* ``EXCH_ALLGATHER``: ``bytes`` at ``send_off`` from every rank to
  ``recv_off + k*bytes``.

Transports: ``"peer"`` (default) lets the library's kernels store the
transposed spectra straight into the other GPUs' receive buffers (CUDA IPC,
one node); the callbacks then carry only the handle swap and small sums, the
latter also serving as stream-ordered barriers.  ``"exchange"`` packs the
blocks and moves them with ``all_to_all_single`` / point-to-point calls.

The reference solves the whole mesh on every rank (its plugin's FFT3d spans
the full grid, lmp/sog.cpp:1084-1087), so this class has no reference
counterpart.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import _lib


class SlabGroup:
    def __init__(self, group: Optional["dist.ProcessGroup"] = None, transport: str = "peer"):
        if transport not in ("peer", "exchange"):
            raise ValueError("`transport` should be 'peer' or 'exchange'.")
        self.transport = _lib.SLAB_PEER if transport == "peer" else _lib.SLAB_EXCHANGE
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.rank = dist.get_rank(group)
            self.size = dist.get_world_size(group)
        else:
            self.rank, self.size = 0, 1
        self._ws: dict = {}
        self._pending: Optional[BaseException] = None

    # ---- workspace ----
    def workspace(self, nbytes: int, device: torch.device) -> torch.Tensor:
        """A uint8 device buffer of at least ``nbytes`` (reused across calls)."""
        key = (device.type, device.index)
        ws = self._ws.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(int(nbytes), dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    # ---- exchanges ----
    def exchange(self, ws: torch.Tensor, kind: int, send_off: int, recv_off: int, nbytes: int) -> None:
        if kind == _lib.EXCH_ALLTOALL:
            total = nbytes * self.size
            send = ws[send_off:send_off + total]
            recv = ws[recv_off:recv_off + total]
            if self.size == 1:
                recv.copy_(send)
            else:
                dist.all_to_all_single(recv, send, group=self.group)
        elif kind == _lib.EXCH_HALO:
            send = ws[send_off:send_off + nbytes]
            recv = ws[recv_off:recv_off + nbytes]
            if self.size == 1:
                recv.copy_(send)
            else:
                prev = self._global((self.rank - 1) % self.size)
                nxt = self._global((self.rank + 1) % self.size)
                ops = [dist.P2POp(dist.isend, send, prev, self.group),
                       dist.P2POp(dist.irecv, recv, nxt, self.group)]
                for req in dist.batch_isend_irecv(ops):
                    req.wait()
        elif kind == _lib.EXCH_ALLGATHER:
            send = ws[send_off:send_off + nbytes]
            recv = ws[recv_off:recv_off + nbytes * self.size]
            if self.size == 1:
                recv.copy_(send)
            else:
                dist.all_gather_into_tensor(recv, send, group=self.group)
        elif kind == _lib.EXCH_SUM_F64:
            if nbytes % 8 or send_off % 8:
                raise ValueError("EXCH_SUM_F64 needs 8-byte aligned doubles")
            if self.size > 1:
                buf = ws[send_off:send_off + nbytes].view(torch.float64)
                dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group)
        else:
            raise ValueError(f"unknown exchange kind {kind}")

    def _global(self, group_rank: int) -> int:
        if self.group is None:
            return group_rank
        return dist.get_global_rank(self.group, group_rank)

    def callback(self, ws: torch.Tensor):
        """The C callback body: runs ``exchange`` and reports failure as a
        non-zero status (the exception is re-raised after the C call)."""
        def fn(ctx, kind, send_off, recv_off, nbytes, stream):
            del ctx, stream  # collectives run on torch's current stream, which the library uses
            try:
                self.exchange(ws, int(kind), int(send_off), int(recv_off), int(nbytes))
                return 0
            except BaseException as exc:  # noqa: BLE001 - reported through the C status
                self._pending = exc
                return 1
        return fn

    def raise_pending(self) -> None:
        exc, self._pending = self._pending, None
        if exc is not None:
            raise exc

    def sum_(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over the ranks (per-slab forces / dE/dq -> every atom)."""
        if self.size > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t
