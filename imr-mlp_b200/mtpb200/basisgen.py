"""Generator of moment-tensor-potential bases of a given level.

No level-24 basis ships with the reference (its generator, mtmbasis, needs
the full reference build), so this module builds one from the published
definition of the MTP basis (Shapeev, Multiscale Model. Simul. 14 (2016)):

* moment tensors M_{mu,nu} = sum_j f_mu(r_j) rhat_j^{(x) nu} have level
  2 + 4 mu + nu; a basis function is a scalar contraction of moment tensors,
  or a product of such scalars, whose levels sum to at most the maximum
  level (mtmbasis/mtm.h:642-651 states the same weighted rule, 2/1/2 ... for
  mu/nu/dim, i.e. lev = 2 + 4 mu + nu per tensor);
* a symmetric tensor is stored by its components A_abc (a x-, b y- and
  c z-indices), the basic moments alpha_index_basic = {mu, a, b, c};
* contractions are written as product rules {l1, l2, c, id} with integer
  multiplicities, m[id] += c * m[l1] * m[l2]:
  - full contraction of two rank-nu tensors:
        A : B = sum_{|g| = nu} mult(g) A_g B_g,   mult = nu!/(a! b! c!);
  - contraction of three tensors A (rank n1), B (n2), D (n3) with k index
    pairs between A and B: the integer-weighted intermediate
        T_g = sum_{a + b = g, |l| = k} mult(a) mult(b) mult(l) A_{a+l} B_{b+l}
    (|a| = n1 - k, |b| = n2 - k) gives C : D = sum_g T_g D_g;
  - products of scalar basis functions (two or three factors).

The result has the layout of the reference's templates (basic moments first,
rules in dependency order, alpha_moment_mapping listing the scalars).  It is a
synthetic stand-in: it shares the level rule, the tensor shapes and the rule
form of the shipped templates, not their exact rule lists.
"""
from __future__ import annotations

import itertools
from math import factorial
from typing import Dict, List, Tuple

import numpy as np

from .mtpfile import MTPModel


def _mult(g: Tuple[int, int, int]) -> int:
    a, b, c = g
    return factorial(a + b + c) // (factorial(a) * factorial(b) * factorial(c))


def _comps(n: int) -> List[Tuple[int, int, int]]:
    return [(a, b, n - a - b) for a in range(n, -1, -1) for b in range(n - a, -1, -1)]


def tensor_level(mu: int, nu: int) -> int:
    return 2 + 4 * mu + nu


class _Builder:
    def __init__(self):
        self.basic: List[Tuple[int, int, int, int]] = []
        self.basic_id: Dict[Tuple[int, int, int, int], int] = {}
        self.rules: List[Tuple[int, int, int, int]] = []
        self.n_derived = 0
        self.derived_keys: Dict[object, int] = {}
        self.pending: List[Tuple[object, Dict[Tuple[int, int], int]]] = []

    def comp(self, mu, g):
        key = (mu,) + tuple(g)
        if key not in self.basic_id:
            self.basic_id[key] = len(self.basic)
            self.basic.append(key)
        return ("b", self.basic_id[key])

    def derived(self, key, terms: Dict[Tuple[object, object], int]):
        """Registers moment `key` = sum c * x * y over terms {(x, y): c}."""
        if key in self.derived_keys:
            return ("d", self.derived_keys[key])
        idx = self.n_derived
        self.n_derived += 1
        self.derived_keys[key] = idx
        self.pending.append((idx, {k: v for k, v in terms.items() if v != 0}))
        return ("d", idx)


def generate(level: int, species_count: int = 1, min_dist: float = 2.0, max_dist: float = 5.0,
             rb_size: int = 8, triples: bool = True, products: int = 3) -> MTPModel:
    """Basis of all contractions of up to three moment tensors and products of
    up to `products` scalars with level <= `level`."""
    mu_max = (level - 2) // 4
    tensors = [(mu, nu) for mu in range(mu_max + 1) for nu in range(level + 1)
               if tensor_level(mu, nu) <= level]
    B = _Builder()
    scalars: List[Tuple[int, Tuple[str, int]]] = []   # (level, moment ref)
    # single tensors of rank 0
    for mu, nu in tensors:
        if nu == 0:
            scalars.append((tensor_level(mu, 0), B.comp(mu, (0, 0, 0))))
    # full contractions of two tensors (rank 0 pairs are products, below)
    for (m1, n1), (m2, n2) in itertools.combinations_with_replacement(tensors, 2):
        if n1 != n2 or n1 == 0 or tensor_level(m1, n1) + tensor_level(m2, n2) > level:
            continue
        terms = {}
        for g in _comps(n1):
            x, y = B.comp(m1, g), B.comp(m2, g)
            terms[(x, y)] = terms.get((x, y), 0) + _mult(g)
        lev = tensor_level(m1, n1) + tensor_level(m2, n2)
        scalars.append((lev, B.derived(("pair", m1, m2, n1), terms)))
    # connected contractions of three tensors of nonzero rank
    if triples:
        for t3 in itertools.combinations_with_replacement(tensors, 3):
            (m1, n1), (m2, n2), (m3, n3) = t3
            if min(n1, n2, n3) == 0 or sum(tensor_level(*t) for t in t3) > level:
                continue
            if (n1 + n2 + n3) % 2 or n1 > n2 + n3 or n2 > n1 + n3 or n3 > n1 + n2:
                continue
            k = (n1 + n2 - n3) // 2   # index pairs between the first two tensors
            r = n3
            tkey = ("T", m1, n1, m2, n2, k)
            terms = {}
            for al in _comps(n1 - k):
                for be in _comps(n2 - k):
                    for la in _comps(k):
                        ga = tuple(al[i] + la[i] for i in range(3))
                        gb = tuple(be[i] + la[i] for i in range(3))
                        g = tuple(al[i] + be[i] for i in range(3))
                        w = _mult(al) * _mult(be) * _mult(la)
                        key = (g, B.comp(m1, ga), B.comp(m2, gb))
                        terms[key] = terms.get(key, 0) + w
            # intermediate components T_g
            comps = {}
            for g in _comps(r):
                tg = {(x, y): c for (gg, x, y), c in terms.items() if gg == g}
                if tg:
                    comps[g] = B.derived(tkey + (g,), tg)
            sterms = {}
            for g, ref in comps.items():
                sterms[(ref, B.comp(m3, g))] = 1
            lev = sum(tensor_level(*t) for t in t3)
            scalars.append((lev, B.derived(("triple",) + t3, sterms)))
    # products of scalars (two or three connected factors)
    base = list(scalars)
    pair_of = {}
    if products >= 2:
        for i, j in itertools.combinations_with_replacement(range(len(base)), 2):
            (l1, s1), (l2, s2) = base[i], base[j]
            if l1 + l2 <= level:
                ref = B.derived(("prod", s1, s2), {(s1, s2): 1})
                pair_of[(i, j)] = (l1 + l2, ref)
                scalars.append((l1 + l2, ref))
    if products >= 3:
        for i, j, k in itertools.combinations_with_replacement(range(len(base)), 3):
            lev = base[i][0] + base[j][0] + base[k][0]
            if lev <= level and (i, j) in pair_of:
                pref = pair_of[(i, j)][1]
                ref = B.derived(("prod3", i, j, k), {(pref, base[k][1]): 1})
                scalars.append((lev, ref))
    return _to_model(B, scalars, species_count, min_dist, max_dist, rb_size, mu_max)


def _to_model(B: _Builder, scalars, K, rmin, rmax, R, mu_max) -> MTPModel:
    order = sorted(range(len(B.basic)),
                   key=lambda i: (B.basic[i][0], sum(B.basic[i][1:]), -B.basic[i][1],
                                  -B.basic[i][2]))
    new_basic = {old: new for new, old in enumerate(order)}
    nb = len(order)

    def mid(ref):
        kind, i = ref
        return new_basic[i] if kind == "b" else nb + i

    times = []
    for idx, terms in B.pending:
        for (x, y), c in terms.items():
            times.append((mid(x), mid(y), int(c), nb + idx))
    mapping, seen = [], set()
    for _, ref in scalars:
        m = mid(ref)
        if m not in seen:
            seen.add(m)
            mapping.append(m)
    basic = np.array([B.basic[i] for i in order], dtype=np.int32).reshape(-1, 4)
    M = nb + B.n_derived
    mu = mu_max + 1
    S = len(mapping)
    return MTPModel(
        species_count=K, min_dist=np.array([rmin]),
        max_dist=np.array([rmax]), rb_size=R, radial_func_count=mu,
        alpha_moments_count=M, alpha_index_basic=basic,
        alpha_index_times=np.array(times, dtype=np.int32).reshape(-1, 4),
        alpha_moment_mapping=np.array(mapping, dtype=np.int32),
        radial_coeffs=np.zeros(K * K * mu * R), species_coeffs=np.zeros(K),
        moment_coeffs=np.zeros(S), scaling=0.01)
