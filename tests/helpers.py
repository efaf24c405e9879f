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


# Radial families exercised by the parity tests: every family, every
# configurable cutoff and shift, the one-minus-Chebyshev polynomials, lambda = 0
# branches, and a lower bound that excludes the first neighbour shell.
RADIAL_CASES = {
    "chebycos": dict(name="RBChebyCos"),
    "poly4": dict(name="RBChebyshevPoly4", b=-0.5),
    "poly5": dict(name="RBChebyshevPoly5", b=-1.0 / 3.0),
    "poly5_min26": dict(name="RBChebyshevPoly5", b=0.25, min_dist=2.6),
    "cfg_cosine_linear": dict(name="RBChebyshevConfigurable", cutoff_type="cosine"),
    "cfg_poly5_exp": dict(name="RBChebyshevConfigurable", cutoff_type="poly5", b=0.2,
                          shift_type="exponential", shift_lambda=1.5),
    "cfg_smooth7_tanh_flip": dict(name="RBChebyshevConfigurable", cutoff_type="smoothstep7",
                                  r1=3.0, r2=4.0, shift_type="exponential_tanh",
                                  shift_lambda=1.2, shift_scale_lambda=0.7,
                                  one_minus_chebyshev=True),
    "cfg_nquad_i2": dict(name="RBChebyshevConfigurable", cutoff_type="normalized_quadratic",
                         shift_type="i2"),
    "cfg_cosleft_expleft": dict(name="RBChebyshevConfigurable", cutoff_type="cosine_left",
                                shift_type="exponential_left", shift_lambda=0.8),
    "cfg_cosunscaled_exp0": dict(name="RBChebyshevConfigurable", cutoff_type="cosine_unscaled",
                                 shift_type="exponential", shift_lambda=0.0),
    "cfg_cossq_flip": dict(name="RBChebyshevConfigurable", cutoff_type="cosine_squared",
                           one_minus_chebyshev=True),
    "cfg_sinsq_tanh0": dict(name="RBChebyshevConfigurable", cutoff_type="sine_squared",
                            shift_type="exponential_tanh", shift_lambda=0.0,
                            shift_scale_lambda=0.5),
    "cfg_poly3": dict(name="RBChebyshevConfigurable", cutoff_type="poly3", b=0.1),
    "cfg_poly4_expleft0": dict(name="RBChebyshevConfigurable", cutoff_type="poly4", b=-0.2,
                               shift_type="exponential_left", shift_lambda=0.0),
    "cfg_smooth5_i2": dict(name="RBChebyshevConfigurable", cutoff_type="smoothstep5",
                           shift_type="i2"),
    "cfg_quad_tanh_noscale": dict(name="RBChebyshevConfigurable", cutoff_type="quadratic",
                                  shift_type="exponential_tanh", shift_lambda=0.9,
                                  shift_scale_lambda=0.0),
}


def with_radial_family(model, case):
    """The model with every pair's radial basis replaced by RADIAL_CASES[case]
    (an optional min_dist in the case moves the lower bound)."""
    import dataclasses
    from mtpb200.mtpfile import RadialFamily
    spec = dict(RADIAL_CASES[case])
    lo = spec.pop("min_dist", None)
    fam = RadialFamily(**spec)
    n = model.species_count ** 2 if model.radial_basis_split else 1
    mins = np.array(model.min_dist, dtype=np.float64)
    if lo is not None:
        mins[:] = lo
    return dataclasses.replace(model, radial_family=[fam] * n, min_dist=mins)


def with_polyb(model, name, reference=None, split=False):
    """The model with every pair's radial basis replaced by RBPolyB or
    RBPolyBCos (`name`); with `reference` the orthogonalisation matrices are the
    ones the compiled reference loader computes for the same text (the
    parity pin), else numpy's (mtpfile.polyb_data).  `split` writes one basis
    per ordered pair."""
    import dataclasses
    from mtpb200 import format_mtp
    from mtpb200.mtpfile import RadialFamily, polyb_data
    K = model.species_count
    n = K * K if split else 1
    mins = np.full(n, float(model.min_dist[0]))
    maxs = np.full(n, float(model.max_dist[0]))
    fams = []
    for p in range(n):
        pm, pn = polyb_data(mins[p], maxs[p], model.rb_size)
        fams.append(RadialFamily(name=name, poly_matrix=pm, poly_norm=pn))
    m = dataclasses.replace(model, radial_family=fams, radial_basis_split=split,
                            min_dist=mins, max_dist=maxs)
    if reference is not None:
        data = reference.polyb(format_mtp(m), K)
        for p in range(n):
            assert data[p] is not None, "the reference loader has no RBPolyB data"
            fams[p].poly_matrix, fams[p].poly_norm = data[p]
    return m
