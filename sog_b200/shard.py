"""Independent frames shared out over data-parallel ranks.

A batch of frames (molecules or boxes, each with its own cell and mesh) has
no exchange step: every rank solves a subset of the frames on its own GPU with
no collective on the data path, and only the per-frame results are put back
together at the end.

* ``frame_costs`` estimates a frame's solve time as N_g·log2(N_g) + p³·N_f
  (mesh transforms plus stencil updates); without a mesh (direct k-sum, real
  space) the atom count stands in.
* ``lpt_partition`` assigns frames by the longest-processing-time rule:
  largest cost first, each to the least-loaded rank (ties to the lower rank),
  so the result is deterministic and every rank computes the same plan
  without communicating.
* ``FrameShards`` is one rank's share of a batch: the index of its atoms in
  the caller's order, a local batch vector, its cells, and the gathers that
  rebuild the full per-frame energy vector (and per-atom forces) from every
  rank's share.

The reference solves every frame of a batch in one process (the per-frame
loop of compute_bundle, gaussian.py:550-820), so this module has no
reference counterpart.
"""
from __future__ import annotations

import heapq
import math
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def frame_costs(natoms: Sequence[int], grid_points: Optional[Sequence[int]] = None,
                order: int = 6) -> List[float]:
    """Estimated relative solve cost of each frame."""
    out = []
    for j, n in enumerate(natoms):
        if grid_points is None:
            out.append(float(n))
        else:
            ng = float(grid_points[j])
            out.append(ng * math.log2(max(ng, 2.0)) + float(order) ** 3 * float(n))
    return out


def lpt_partition(costs: Sequence[float], world: int) -> List[List[int]]:
    """Frames of each rank (ascending frame order within a rank)."""
    if world < 1:
        raise ValueError("`world` must be at least 1")
    order = sorted(range(len(costs)), key=lambda j: (-float(costs[j]), j))
    heap = [(0.0, r) for r in range(world)]
    heapq.heapify(heap)
    assign: List[List[int]] = [[] for _ in range(world)]
    for j in order:
        load, r = heapq.heappop(heap)
        assign[r].append(j)
        heapq.heappush(heap, (load + float(costs[j]), r))
    return [sorted(a) for a in assign]


class FrameShards:
    """One rank's share of a batch whose frames are contiguous atom ranges.

    ``counts[j]`` is the atom count of frame j (frames in output order, atoms
    of frame j at ``sum(counts[:j]) ...``); ``assign`` is the partition of
    every rank (``lpt_partition``)."""

    def __init__(self, counts: Sequence[int], assign: Sequence[Sequence[int]], rank: int,
                 device: torch.device):
        self.counts = [int(c) for c in counts]
        self.assign = [list(a) for a in assign]
        self.world = len(self.assign)
        self.rank = int(rank)
        self.device = device
        begins, acc = [], 0
        for c in self.counts:
            begins.append(acc)
            acc += c
        self.natoms = acc
        self.nframes = len(self.counts)
        mine = self.assign[self.rank]
        self.frames = mine
        idx = [torch.arange(begins[j], begins[j] + self.counts[j]) for j in mine]
        self.atom_index = (torch.cat(idx) if idx else torch.zeros(0, dtype=torch.long)).to(device)
        self.frame_index = torch.tensor(mine, dtype=torch.long, device=device)
        self.local_batch = torch.repeat_interleave(
            torch.arange(len(mine), device=device),
            torch.tensor([self.counts[j] for j in mine], dtype=torch.long, device=device))
        self.max_frames = max(len(a) for a in self.assign)
        self.max_atoms = max(sum(self.counts[j] for j in a) for a in self.assign)
        # where rank k's padded slots land in the full vectors
        fpos, apos = [], []
        for a in self.assign:
            fpos.append(list(a) + [-1] * (self.max_frames - len(a)))
            at = [i for j in a for i in range(begins[j], begins[j] + self.counts[j])]
            apos.append(at + [-1] * (self.max_atoms - len(at)))
        fflat = torch.tensor([p for row in fpos for p in row], dtype=torch.long)
        aflat = torch.tensor([p for row in apos for p in row], dtype=torch.long)
        self._fsel = (fflat >= 0).nonzero().flatten().to(device)
        self._fdst = fflat[fflat >= 0].to(device)
        self._asel = (aflat >= 0).nonzero().flatten().to(device)
        self._adst = aflat[aflat >= 0].to(device)

    def select(self, r: torch.Tensor, q: torch.Tensor, cell: Optional[torch.Tensor]
               ) -> Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor], torch.Tensor]:
        """This rank's positions, charges, cells and local batch vector."""
        rl = r.index_select(0, self.atom_index)
        ql = q.index_select(0, self.atom_index)
        cl = None if cell is None else cell.index_select(0, self.frame_index)
        return rl, ql, cl, self.local_batch

    def _gather(self, local: torch.Tensor, rows: int, sel: torch.Tensor, dst: torch.Tensor,
                total: int, group) -> torch.Tensor:
        pad = torch.zeros((rows,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        pad[:local.shape[0]] = local
        if self.world > 1:
            allp = torch.empty((self.world * rows,) + tuple(local.shape[1:]), dtype=local.dtype,
                               device=local.device)
            dist.all_gather_into_tensor(allp, pad, group=group)
        else:
            allp = pad
        out = torch.zeros((total,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        out.index_copy_(0, dst, allp.index_select(0, sel))
        return out

    def gather_energy(self, e_local: torch.Tensor, group=None) -> torch.Tensor:
        """Per-frame results of every rank -> the full [nframes, ...] tensor.
        Forward values only: the gathered tensor carries no autograd graph, so
        a loss is backpropagated on each rank's own local outputs (the
        gradient of a data-parallel sum of per-rank losses)."""
        return self._gather(e_local, self.max_frames, self._fsel, self._fdst, self.nframes, group)

    def gather_atoms(self, x_local: torch.Tensor, group=None) -> torch.Tensor:
        """Per-atom results (forces, dE/dq) of every rank -> [natoms, ...].
        Forward values only, as gather_energy."""
        return self._gather(x_local, self.max_atoms, self._asel, self._adst, self.natoms, group)
