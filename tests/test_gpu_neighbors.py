"""GPU neighbour builder: per-atom neighbour sets bit-exact with the
reference builder (golden fixtures) and the oracle restatement."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, load_model
from helpers import bits, canonical_digest, same_lists
from mtpb200 import configs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu16(model_l16):
    from mtpb200 import MTPGpuDirect
    g = MTPGpuDirect(model_l16, 0)
    yield g
    g.close()


def _build(gpu, structures):
    from mtpb200 import StructureBatch
    b = StructureBatch.from_structures(structures)
    gpu.build_neighbors(b)
    return b, gpu.get_neighbors()


def test_config1_matches_reference_golden(gpu16):
    g = np.load(os.path.join(GOLDEN, "golden_config1_l16.npz"))
    st = {"cell": g["cell"], "pbc": np.ones(3, np.int32), "positions": g["positions"],
          "types": g["types"]}
    _, (off, nbr, rij, sh) = _build(gpu16, [st])
    assert np.array_equal(np.diff(off), g["counts"])
    assert canonical_digest(off, nbr, rij) == str(g["digest"])


def test_strained_alloys_match_reference_golden(model_l20_k3):
    from mtpb200 import MTPGpuDirect
    g = np.load(os.path.join(GOLDEN, "golden_config2_l20.npz"))
    n = int(g["count"])
    sts = [{"cell": g[f"s{k}_cell"], "pbc": np.ones(3, np.int32),
            "positions": g[f"s{k}_positions"], "types": g[f"s{k}_types"]} for k in range(n)]
    with MTPGpuDirect(model_l20_k3, 0) as gpu:
        b, (off, nbr, rij, _) = _build(gpu, sts)
    for k in range(n):
        a0, a1 = b.atom_offsets[k], b.atom_offsets[k + 1]
        o = off[a0:a1 + 1] - off[a0]
        e0, e1 = off[a0], off[a1]
        assert same_lists(o, nbr[e0:e1] - a0, rij[e0:e1], g[f"s{k}_offsets"], g[f"s{k}_nbr"],
                          g[f"s{k}_rij"])


def test_small_cells_match_reference_golden():
    """Thin cell (many images), skewed cell, single atom."""
    from mtpb200 import MTPGpuDirect
    m = load_model("many_body_k3.mtp")
    g = np.load(os.path.join(GOLDEN, "golden_small_cells.npz"))
    n = int(g["count"])
    sts = [{"cell": g[f"s{k}_cell"], "pbc": np.ones(3, np.int32),
            "positions": g[f"s{k}_positions"], "types": g[f"s{k}_types"]} for k in range(n)]
    with MTPGpuDirect(m, 0) as gpu:
        b, (off, nbr, rij, _) = _build(gpu, sts)
    for k in range(n):
        a0, a1 = b.atom_offsets[k], b.atom_offsets[k + 1]
        o = off[a0:a1 + 1] - off[a0]
        e0, e1 = off[a0], off[a1]
        assert same_lists(o, nbr[e0:e1] - a0, rij[e0:e1], g[f"s{k}_offsets"], g[f"s{k}_nbr"],
                          g[f"s{k}_rij"])


@pytest.mark.parametrize("seed", [5, 6])
def test_batched_strained_match_oracle(gpu16, oracle, seed):
    sts = configs.config2(24, seed=seed)
    for s in sts:
        s["types"] = np.minimum(s["types"], 1).astype(np.int32)
    b, (off, nbr, rij, _) = _build(gpu16, sts)
    for k, st in enumerate(sts):
        nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], gpu16.cutoff)
        a0, a1 = b.atom_offsets[k], b.atom_offsets[k + 1]
        e0, e1 = off[a0], off[a1]
        assert same_lists(off[a0:a1 + 1] - e0, nbr[e0:e1] - a0, rij[e0:e1], nl.offsets, nl.nbr,
                          nl.rij)


def test_edge_cases_empty_structures(gpu16):
    """Empty structures inside a batch and an empty batch."""
    sts = [configs.config1()]
    empty = {"cell": np.eye(3) * 10, "pbc": np.ones(3, np.int32),
             "positions": np.zeros((0, 3)), "types": np.zeros(0, np.int32)}
    b, (off, nbr, rij, _) = _build(gpu16, [empty] + sts + [empty])
    assert off[-1] == gpu16.neighbor_count() > 0
    e, f, s, _ = gpu16.compute()
    assert e.shape == (3,) and e[0] == 0.0 and e[2] == 0.0


def test_list_symmetry_full_size_property(gpu16):
    """(i -> j, r) has (j -> i, -r) bit for bit on a 108k-atom box."""
    st = configs.ni3al_l12(30, 3.52, 0.08, seed=9)
    st["types"] = st["types"].astype(np.int32)
    _, (off, nbr, rij, sh) = _build(gpu16, [st])
    n = len(off) - 1
    centers = np.repeat(np.arange(n), np.diff(off))
    key_f = np.stack([centers, nbr, *bits(rij).T], 1)
    key_b = np.stack([nbr, centers, *bits(-rij).T], 1)
    sf = key_f[np.lexsort(key_f.T[::-1])]
    sb = key_b[np.lexsort(key_b.T[::-1])]
    assert np.array_equal(sf, sb)
    assert np.all(np.sum(rij * rij, 1) < gpu16.cutoff ** 2)
