"""Configuration sharding of the batched EFS and training workloads.

Independent structures are assigned whole to ranks (the reference trainer
splits its training set over MPI ranks the same way,
train/train_mtp.cpp:3061-3085).  Each rank evaluates its shard with its own
library context; the batched EFS needs no data-path collective, and the
trainer sums one contiguous device vector [loss, 7 metrics, gradient] over
the ranks with a single all-reduce, each rank having normalised by the
global structure count (mtpb_loss_grad's norm_count)."""
from __future__ import annotations

from typing import Dict, List, Sequence

import numpy as np


def shard_lpt(sizes: Sequence[float], nranks: int) -> np.ndarray:
    """Greedy longest-processing-time assignment of items to ranks by size
    (structures by atom count: edge counts are proportional to atom counts
    within a configuration).  Returns owner[i]; ties go to the lower rank."""
    order = np.argsort(-np.asarray(sizes, dtype=np.float64), kind="stable")
    load = np.zeros(nranks)
    owner = np.zeros(len(sizes), dtype=np.int64)
    for i in order:
        r = int(np.argmin(load))
        owner[i] = r
        load[r] += sizes[i]
    return owner


def shard_of(structures: List[Dict[str, np.ndarray]], owner: np.ndarray, rank: int):
    """The structures of one rank, in input order, and their input indices."""
    idx = [i for i, o in enumerate(owner) if o == rank]
    return [structures[i] for i in idx], idx


def allreduce_loss_grad(dist, out, group=None):
    """Sums [loss, metrics[7], grad[...]] over the ranks in place (one
    all-reduce of a few KB: the only collective of a training evaluation)."""
    dist.all_reduce(out, group=group)
    return out
