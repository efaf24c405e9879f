"""Moment graphs larger than shared memory: the graph kernels keep their
rows in an L2-resident global slice per persistent block.  The mode is
checked bit for bit against the shared-memory mode (MTPB_DAG_GLOBAL_ROWS=1 on
a level-20 model) and, on the generated level-24 stand-in, against the C
oracle for EFS and the training gradient."""
import os

import numpy as np
import pytest

from conftest import load_model
from mtpb200 import configs

pytestmark = pytest.mark.gpu

TOL_E_ATOM = 1e-10
TOL_F = 1e-9
TOL_W = 1e-9
WEIGHTS = (1.0, 0.01, 0.001, 1.0, 0.0, 1.0)


def _run(model, sts, labels, force_global):
    from mtpb200 import MTPGpuDirect, StructureBatch
    old = os.environ.get("MTPB_DAG_GLOBAL_ROWS")
    os.environ["MTPB_DAG_GLOBAL_ROWS"] = "1" if force_global else "0"
    try:
        with MTPGpuDirect(model, 0) as gpu:
            efs = gpu.efs(StructureBatch.from_structures(sts), site_energy=True)
            grad = gpu.loss_grad(*labels, WEIGHTS)
    finally:
        if old is None:
            del os.environ["MTPB_DAG_GLOBAL_ROWS"]
        else:
            os.environ["MTPB_DAG_GLOBAL_ROWS"] = old
    return efs, grad


def _labels(sts, seed):
    rng = np.random.default_rng(seed)
    n = sum(len(s["types"]) for s in sts)
    return (rng.normal(0, 1, len(sts)), rng.normal(0, 0.1, (n, 3)),
            rng.normal(0, 0.5, (len(sts), 9)))


def test_global_rows_bitwise_equal_to_shared_rows():
    m = load_model("l20_k3.mtp")
    sts = configs.config2(3, seed=81)
    lab = _labels(sts, 1)
    (e0, g0), (e1, g1) = _run(m, sts, lab, False), _run(m, sts, lab, True)
    for a, b in zip(e0, e1):
        assert np.array_equal(a, b)
    assert g0[0] == g1[0] and np.array_equal(g0[2], g1[2])


def test_level24_stand_in_against_oracle(oracle):
    from oracle import concat_lists
    m = configs.level24_model()
    sts = configs.config4_structures(3, seed=82)
    lab = _labels(sts, 2)
    (e, f, s, se), (loss, metrics, grad) = _run(m, sts, lab, False)
    offs, _, _, _, types = configs.batch(sts)
    lists = [oracle.neighbors(x["cell"], x["pbc"], x["positions"], m.cutoff) for x in sts]
    for k, (x, nl) in enumerate(zip(sts, lists)):
        re, rse, rf, rs = oracle.efs(m, x["types"], nl)
        a0, a1 = offs[k], offs[k + 1]
        assert abs(e[k] - re) / (a1 - a0) < TOL_E_ATOM
        assert np.max(np.abs(se[a0:a1] - rse)) < TOL_E_ATOM
        assert np.max(np.abs(f[a0:a1] - rf)) < TOL_F
        assert np.max(np.abs(s[k] - rs)) < TOL_W
    rl, rm, rg = oracle.loss_grad(m, offs, types, concat_lists(lists, offs), *lab, WEIGHTS)
    assert abs(loss - rl) <= 1e-10 * max(1.0, abs(rl))
    assert np.max(np.abs(grad - rg)) <= 1e-9 * max(1.0, np.max(np.abs(rg)))


def test_config5_interface_against_oracle(oracle):
    """Level-24 stand-in with K=3, R=10, rmin 0.8, r_cut 6 on one
    Ru(0001)/water interface (configuration 5)."""
    from mtpb200 import MTPGpuDirect, StructureBatch
    m = configs.level24_model(species_count=3, rmin=0.8, rmax=6.0, rb_size=10, seed=55)
    st = configs.ru_water_interface(7)
    with MTPGpuDirect(m, 0) as gpu:
        e, f, s, se = gpu.efs(StructureBatch.from_structures([st]), site_energy=True)
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], m.cutoff)
    re, rse, rf, rs = oracle.efs(m, st["types"], nl)
    n = len(st["types"])
    assert abs(e[0] - re) / n < TOL_E_ATOM
    assert np.max(np.abs(se - rse)) < TOL_E_ATOM
    assert np.max(np.abs(f - rf)) < TOL_F
    assert np.max(np.abs(s[0] - rs)) < TOL_W
