"""The level-24 stand-in basis generator (mtpb200.basisgen): calibration
against the shipped level-16/20 templates, rotational invariance of the
generated bases through the C oracle, and a level-24 plan that the graph
planner accepts.  Needs no GPU."""
import ctypes as C

import numpy as np
import pytest

from conftest import load_model
from mtpb200 import basisgen, configs


def _basic_set(m):
    return {tuple(r) for r in m.alpha_index_basic.tolist()}


@pytest.mark.parametrize("level,template", [(16, "l16_k2.mtp"), (20, "l20_k2.mtp")])
def test_generator_matches_shipped_template_sizes(level, template):
    g = basisgen.generate(level)
    t = load_model(template)
    assert _basic_set(g) == _basic_set(t)
    for a, b in ((g.alpha_index_times_count, t.alpha_index_times_count),
                 (g.alpha_moments_count, t.alpha_moments_count),
                 (g.alpha_scalar_moments, t.alpha_scalar_moments)):
        assert abs(a - b) <= 0.25 * b, (a, b)


def test_generated_rules_are_topological_with_integer_multiplicities():
    m = basisgen.generate(24)
    T = m.alpha_index_times
    assert T.dtype == np.int32 and np.all(T[:, 2] >= 1)
    nb = m.alpha_index_basic_count
    done = set(range(nb))
    first = {}
    for i, (a, b, c, t) in enumerate(T.tolist()):
        assert a in done and b in done, i
        first.setdefault(t, i)
        done.add(t)   # every rule of a target comes before its first use
    assert set(m.alpha_moment_mapping.tolist()) <= done
    assert m.alpha_index_basic[:, 0].max() == 5 and (m.alpha_index_basic[:, 1:].sum(1)).max() == 10


def _rotation(seed):
    q, _ = np.linalg.qr(np.random.default_rng(seed).normal(size=(3, 3)))
    return q * np.sign(np.linalg.det(q))


@pytest.mark.parametrize("level", [16, 24])
def test_generated_basis_is_rotation_invariant(oracle, level):
    m = configs.seeded_coefficients(basisgen.generate(level, species_count=2), 5)
    st = configs.config4_structures(1, seed=17)[0]
    R = _rotation(3)
    es = []
    for cell, pos in ((st["cell"], st["positions"]), (st["cell"] @ R.T, st["positions"] @ R.T)):
        nl = oracle.neighbors(cell, st["pbc"], pos, m.cutoff)
        e, _, f, _ = oracle.efs(m, st["types"], nl)
        es.append(e)
    assert abs(es[0] - es[1]) <= 1e-10 * max(1.0, abs(es[0]))


def test_level24_plan_needs_global_rows():
    import mtpb200
    from mtpb200 import _ModelKeep, _lib
    m = configs.level24_model()
    lib = mtpb200.library()
    keep = _ModelKeep(m)
    ints = [C.c_int() for _ in range(6)]
    nrec = C.c_long()
    sob = np.zeros(m.alpha_index_basic_count, np.int32)
    phases = np.zeros(64, np.int32)
    rc = lib.mtpb_graph_program(C.byref(keep.view), C.byref(ints[0]),
                                sob.ctypes.data_as(_lib._ip), C.byref(ints[1]), C.byref(ints[2]),
                                C.byref(ints[3]), C.byref(ints[4]), C.byref(ints[5]),
                                phases.ctypes.data_as(_lib._ip), C.byref(nrec), None)
    assert rc == 0, lib.mtpb_last_error()
    nslot, nrows = ints[0].value, ints[1].value
    assert nslot == 581
    assert nrows * 8 * 8 > 200 * 1024   # beyond shared memory even at 8 atoms per block
