"""mtpb_set_center_count on the GPU: a box split into slabs, each evaluated
by its own context on a rotated view (own slab first, neighbours from the
whole box), partial forces summed in slab order, equals the one-context
result and the oracle.  Two ranks are emulated on one GPU, one after the
other; the collectives themselves are covered by tests/test_slab.py."""
import numpy as np
import pytest

from mtpb200 import configs
from mtpb200.slab import SlabLayout

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nranks", [2, 3])
def test_center_count_slabs_sum_to_full_box(oracle, model_l16, nranks):
    from mtpb200 import MTPGpuDirect, StructureBatch
    st = configs.ni3al_l12(5, 3.52, 0.08, seed=9)
    L = SlabLayout(st["cell"], st["positions"], nranks)
    pos = st["positions"][L.order]
    types = st["types"][L.order].astype(np.int32)
    cell = st["cell"].reshape(1, 9)
    off = np.array([0, L.natoms], np.int32)
    f_sum = np.zeros((L.natoms, 3))
    e_sum, w_sum = 0.0, np.zeros((3, 3))
    with MTPGpuDirect(model_l16, 0) as gpu:
        for r in range(nranks):
            gpu.set_center_count(int(L.counts[r]))
            b = StructureBatch(off, cell, None, L.to_local(pos, r), L.to_local(types, r))
            e, f, s, se = gpu.efs(b, site_energy=True)
            assert se.shape[0] == L.counts[r]
            f_sum += L.to_slab(f, r)
            e_sum += e[0]
            w_sum += s[0]
        gpu.set_center_count(0)
        e1, f1, s1, _ = gpu.efs(StructureBatch(off, cell, None, pos, types))
    nl = oracle.neighbors(st["cell"], st["pbc"], pos, model_l16.cutoff)
    re, _, rf, rw = oracle.efs(model_l16, types, nl)
    n = L.natoms
    for ee, ff, ww in ((e_sum, f_sum, w_sum), (e1[0], f1, s1[0])):
        assert abs(ee - re) / n < 1e-10
        assert np.max(np.abs(ff - rf)) < 1e-9
        assert np.max(np.abs(ww - rw)) < 1e-9
