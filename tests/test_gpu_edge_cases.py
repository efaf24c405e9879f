"""Empty and ragged inputs on the GPU against the oracle: batches with
empty structures, an isolated atom (no neighbour within the cutoff), a
single-atom cell (neighbours are its own images), mixed sizes, and a CSR
request without centres."""
import ctypes as C

import numpy as np
import pytest

from mtpb200 import configs

pytestmark = pytest.mark.gpu


def _cubic(a, pos, types):
    return {"cell": np.eye(3) * a, "pbc": np.ones(3, np.int32),
            "positions": np.asarray(pos, dtype=np.float64).reshape(-1, 3),
            "types": np.asarray(types, dtype=np.int32)}


def _check_batch(oracle, model, sts):
    from mtpb200 import MTPGpuDirect, StructureBatch
    b = StructureBatch.from_structures(sts)
    with MTPGpuDirect(model, 0) as gpu:
        e, f, s, se = gpu.efs(b, site_energy=True)
    offs = b.atom_offsets
    for k, x in enumerate(sts):
        a0, a1 = offs[k], offs[k + 1]
        if a1 == a0:
            assert e[k] == 0.0 and np.all(s[k] == 0.0)
            continue
        nl = oracle.neighbors(x["cell"], x["pbc"], x["positions"], model.cutoff)
        re, rse, rf, rs = oracle.efs(model, x["types"], nl)
        assert abs(e[k] - re) / (a1 - a0) < 1e-10
        assert np.max(np.abs(se[a0:a1] - rse)) < 1e-10
        assert np.max(np.abs(f[a0:a1] - rf)) < 1e-9
        assert np.max(np.abs(s[k] - rs)) < 1e-9


def test_empty_isolated_and_single_atom_structures(oracle, model_l16):
    sts = [
        _cubic(20.0, np.zeros((0, 3)), []),                       # empty
        _cubic(20.0, [[1.0, 2.0, 3.0]], [1]),                     # isolated atom
        _cubic(3.0, [[0.2, 0.1, 0.3]], [0]),                      # own images only
        configs.config1(),                                        # 256 atoms
        _cubic(20.0, np.zeros((0, 3)), []),                       # empty again
        _cubic(12.0, [[0, 0, 0], [2.5, 0, 0], [9.0, 9.0, 9.0]], [0, 1, 1]),   # pair + loner
    ]
    _check_batch(oracle, model_l16, sts)


def test_only_empty_structures(model_l16):
    from mtpb200 import MTPGpuDirect, StructureBatch
    sts = [_cubic(10.0, np.zeros((0, 3)), []) for _ in range(3)]
    with MTPGpuDirect(model_l16, 0) as gpu:
        e, f, s, se = gpu.efs(StructureBatch.from_structures(sts))
        assert gpu.neighbor_count() == 0
    assert np.all(e == 0.0) and np.all(s == 0.0)


def test_ragged_batch_level20(oracle, model_l20_k3):
    sts = configs.config2(5, seed=23)
    sts.insert(2, _cubic(15.0, [[1, 1, 1]], [2]))
    _check_batch(oracle, model_l20_k3, sts)


def test_csr_without_centres(model_l16):
    from mtpb200 import MTPGpuDirect
    with MTPGpuDirect(model_l16, 0) as gpu:
        out = gpu.compute_batch(np.zeros(1, np.int32), np.zeros(0, np.int32),
                                np.zeros(4, np.int32), np.zeros((4, 3)), center_count=0)
    assert out["energy"] == 0.0
    assert np.all(out["force"] == 0.0) and np.all(out["virial"] == 0.0)


@pytest.mark.parametrize("cutoff", [8.0, 11.0])
def test_high_degree_lists(oracle, model_l16, cutoff):
    """Long cutoffs on the 256-atom box: about 200 and 530 neighbours per atom,
    so the in-edge lists take the 256-entry register sort and the single-lane
    fallback of the neighbour builder; lists, energies and forces still match
    the oracle."""
    import dataclasses
    from helpers import same_lists
    from mtpb200 import MTPGpuDirect, StructureBatch
    m = dataclasses.replace(model_l16, max_dist=np.array([cutoff]))
    st = configs.config1()
    with MTPGpuDirect(m, 0) as gpu:
        gpu.build_neighbors(StructureBatch.from_structures([st]))
        off, nbr, rij, _ = gpu.get_neighbors()
        e, f, s, _ = gpu.compute()
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], cutoff)
    assert same_lists(off, nbr, rij, nl.offsets, nl.nbr, nl.rij)
    assert np.diff(off).max() > (256 if cutoff > 10 else 128)
    re, _, rf, rs = oracle.efs(m, st["types"], nl)
    assert abs(e[0] - re) < 1e-12 * max(1.0, abs(re))
    assert np.max(np.abs(f - rf)) < 1e-9 * max(1.0, np.max(np.abs(rf)))
    assert np.max(np.abs(s[0] - rs)) < 1e-9 * max(1.0, np.max(np.abs(rs)))
