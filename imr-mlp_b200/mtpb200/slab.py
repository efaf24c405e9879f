"""Slab decomposition of one periodic box over the ranks of a process group.

The box's atoms are grouped into slabs along the first lattice direction
(fractional coordinate of the wrapped position), one slab per rank, and kept
in slab order.  Rank r evaluates the site terms of its own atoms only: its
library context sees the whole box in a *rotated* order that starts with its
slab (so its centres are the first n_r atoms, mtpb_set_center_count), with
neighbours drawn from every atom of the periodic box.  One EFS step is then

  1. all-gather of the owned positions (the exchange of the halo: NVLink moves
     the whole box, ~25 MB for 1M atoms, in tens of microseconds);
  2. EFS of the owned centres, giving partial forces for every atom (the
     reverse ghost contributions of a LAMMPS newton-on step,
     LAMMPS/USER-MLIP/pair_MLIP_gpu_direct.cpp:457);
  3. reduce-scatter (sum) of the partial forces, all-reduce of the energy and
     virial.

No kernel reads another GPU's memory; all transfers are collectives into
local buffers.  The functions take torch tensors and a torch.distributed
process group (nccl on GPUs, gloo on the CPU in the tests).
"""
from __future__ import annotations

from typing import Sequence

import numpy as np


class SlabLayout:
    """Slab order of a box: `order[k]` is the input index of the atom at slab
    position k; rank r owns slab positions starts[r] .. starts[r+1]."""

    def __init__(self, cell: np.ndarray, positions: np.ndarray, nranks: int):
        cell = np.asarray(cell, dtype=np.float64).reshape(3, 3)
        frac = np.asarray(positions, dtype=np.float64) @ np.linalg.inv(cell)
        fx = frac[:, 0] - np.floor(frac[:, 0])
        slab = np.minimum((fx * nranks).astype(np.int64), nranks - 1)
        self.nranks = nranks
        self.order = np.argsort(slab, kind="stable")
        self.counts = np.bincount(slab, minlength=nranks).astype(np.int64)
        self.starts = np.concatenate([[0], np.cumsum(self.counts)]).astype(np.int64)
        self.natoms = int(self.starts[-1])

    def rotation(self, rank: int) -> np.ndarray:
        """Slab positions in rank `rank`'s local order (its own slab first)."""
        s = int(self.starts[rank])
        return np.concatenate([np.arange(s, self.natoms), np.arange(0, s)])

    def to_local(self, x, rank: int):
        """Slab-ordered array -> rank-local order (torch or numpy)."""
        s = int(self.starts[rank])
        return _cat([x[s:], x[:s]])

    def to_slab(self, x, rank: int):
        """Rank-local array -> slab order."""
        s = int(self.starts[rank])
        n = self.natoms
        return _cat([x[n - s:], x[:n - s]])


def _cat(parts: Sequence):
    if isinstance(parts[0], np.ndarray):
        return np.concatenate(parts)
    import torch
    return torch.cat(list(parts))


class SlabExchange:
    """The collectives of one EFS step on a slab layout."""

    def __init__(self, layout: SlabLayout, rank: int, dist, device):
        import torch
        self.L = layout
        self.rank = rank
        self.dist = dist
        self.maxc = int(layout.counts.max())
        self.nccl = dist.get_backend() == "nccl"
        ws = layout.nranks
        self.gbuf = torch.zeros((ws, self.maxc, 3), dtype=torch.float64, device=device)
        self.sendbuf = torch.zeros((self.maxc, 3), dtype=torch.float64, device=device)
        self.fbuf = torch.zeros((ws, self.maxc, 3), dtype=torch.float64, device=device)
        self.fout = torch.zeros((self.maxc, 3), dtype=torch.float64, device=device)

    def gather_positions(self, own):
        """own: (n_rank, 3) positions of this rank's slab -> (N, 3) slab order."""
        n = own.shape[0]
        self.sendbuf[:n].copy_(own)
        if self.nccl:
            self.dist.all_gather_into_tensor(self.gbuf, self.sendbuf)
        else:
            parts = list(self.gbuf.unbind(0))
            self.dist.all_gather(parts, self.sendbuf)
            for r, p in enumerate(parts):
                self.gbuf[r].copy_(p)
        c = self.L.counts
        return _cat([self.gbuf[r, :int(c[r])] for r in range(self.L.nranks)])

    def reduce_forces(self, partial):
        """partial: (N, 3) slab-ordered partial forces -> (n_rank, 3) sums."""
        c, st = self.L.counts, self.L.starts
        for r in range(self.L.nranks):
            self.fbuf[r, :int(c[r])].copy_(partial[int(st[r]):int(st[r + 1])])
        if self.nccl:
            self.dist.reduce_scatter_tensor(self.fout, self.fbuf)
            return self.fout[:int(c[self.rank])]
        self.dist.all_reduce(self.fbuf)
        return self.fbuf[self.rank, :int(c[self.rank])]

    def reduce_totals(self, t):
        """Sum of per-rank energy / virial totals (in place)."""
        self.dist.all_reduce(t)
        return t
