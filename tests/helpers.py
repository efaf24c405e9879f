"""Shared test helpers (neighbour-list digests and comparisons)."""
import hashlib

import numpy as np


def canonical_digest(off, nbr, rij) -> str:
    """sha256 over per-atom lists sorted by (neighbour, rx, ry, rz)."""
    h = hashlib.sha256()
    for i in range(len(off) - 1):
        a, b = off[i], off[i + 1]
        order = np.lexsort((rij[a:b, 2], rij[a:b, 1], rij[a:b, 0], nbr[a:b]))
        h.update(np.ascontiguousarray(nbr[a:b][order]).astype(np.int64).tobytes())
        h.update(np.ascontiguousarray(rij[a:b][order]).astype(np.float64).tobytes())
    return h.hexdigest()


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float64).view(np.int64)


def canonical(off, nbr, rij):
    order = np.empty(len(nbr), dtype=np.int64)
    for i in range(len(off) - 1):
        a, b = off[i], off[i + 1]
        order[a:b] = a + np.lexsort((rij[a:b, 2], rij[a:b, 1], rij[a:b, 0], nbr[a:b]))
    return nbr[order], rij[order], order


def same_lists(off_a, nbr_a, rij_a, off_b, nbr_b, rij_b) -> bool:
    if not np.array_equal(off_a, off_b):
        return False
    na, ra, _ = canonical(off_a, nbr_a, rij_a)
    nb, rb, _ = canonical(off_b, nbr_b, rij_b)
    return np.array_equal(na, nb) and np.array_equal(bits(ra), bits(rb))
