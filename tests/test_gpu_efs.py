"""EFS parity of the CUDA path against the oracle and the reference golden
outputs.

Tolerances are the north-star bar: energy per atom 1e-10 eV, forces 1e-9
eV/Angstrom, virial 1e-9 eV (absolute), checked here with margin."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, load_model
from mtpb200 import configs

pytestmark = pytest.mark.gpu

TOL_E_ATOM = 1e-10
TOL_F = 1e-9
TOL_W = 1e-9


def _efs(model, structures, site_energy=True):
    from mtpb200 import MTPGpuDirect, StructureBatch
    b = StructureBatch.from_structures(structures)
    with MTPGpuDirect(model, 0) as gpu:
        out = gpu.efs(b, site_energy=site_energy)
        nl = gpu.get_neighbors()
        mom = gpu.site_moments()
        d = gpu.edge_derivatives(int(nl[0][-1]))
    return b, out, nl, mom, d


def _oracle_batch(oracle, model, structures, offs):
    from oracle import concat_lists
    lists = [oracle.neighbors(s["cell"], s["pbc"], s["positions"], model.cutoff)
             for s in structures]
    return concat_lists(lists, offs)


def test_config1_level16_against_reference_golden(model_l16):
    g = np.load(os.path.join(GOLDEN, "golden_config1_l16.npz"))
    st = {"cell": g["cell"], "pbc": np.ones(3, np.int32), "positions": g["positions"],
          "types": g["types"]}
    b, (e, f, s, se), _, _, _ = _efs(model_l16, [st])
    n = len(g["types"])
    assert abs(e[0] - float(g["energy"])) / n < TOL_E_ATOM
    assert np.max(np.abs(se - g["site_energy"])) < TOL_E_ATOM
    assert np.max(np.abs(f - g["forces"])) < TOL_F
    w = s[0]
    sym = np.array([w[0, 0], w[1, 1], w[2, 2], 0.5 * (w[0, 1] + w[1, 0]),
                    0.5 * (w[0, 2] + w[2, 0]), 0.5 * (w[1, 2] + w[2, 1])])
    assert np.max(np.abs(sym - g["virial6"])) < TOL_W


def test_config2_level20_three_species_against_golden(model_l20_k3):
    g = np.load(os.path.join(GOLDEN, "golden_config2_l20.npz"))
    n = int(g["count"])
    sts = [{"cell": g[f"s{k}_cell"], "pbc": np.ones(3, np.int32),
            "positions": g[f"s{k}_positions"], "types": g[f"s{k}_types"]} for k in range(n)]
    b, (e, f, s, se), _, _, _ = _efs(model_l20_k3, sts)
    for k in range(n):
        a0, a1 = b.atom_offsets[k], b.atom_offsets[k + 1]
        assert abs(e[k] - float(g[f"s{k}_energy"])) / (a1 - a0) < TOL_E_ATOM
        assert np.max(np.abs(f[a0:a1] - g[f"s{k}_forces"])) < TOL_F


def test_small_cells_split_basis_against_golden():
    m = load_model("many_body_k3.mtp")
    g = np.load(os.path.join(GOLDEN, "golden_small_cells.npz"))
    n = int(g["count"])
    sts = [{"cell": g[f"s{k}_cell"], "pbc": np.ones(3, np.int32),
            "positions": g[f"s{k}_positions"], "types": g[f"s{k}_types"]} for k in range(n)]
    b, (e, f, s, se), _, _, _ = _efs(m, sts)
    for k in range(n):
        a0, a1 = b.atom_offsets[k], b.atom_offsets[k + 1]
        assert abs(e[k] - float(g[f"s{k}_energy"])) < TOL_E_ATOM * (a1 - a0)
        assert np.max(np.abs(f[a0:a1] - g[f"s{k}_forces"]), initial=0) < TOL_F


def test_moments_adjoints_and_edge_derivatives_vs_oracle(oracle, model_l20_k3):
    """Intermediate quantities: basic moments, dE/db, dE_i/dr_ij."""
    sts = configs.config2(6, seed=17)
    offs = configs.batch(sts)[0]
    b, (e, f, s, se), (off, nbr, rij, _), (mom, adj), d = _efs(model_l20_k3, sts)
    nl = _oracle_batch(oracle, model_l20_k3, sts, offs)
    bo, ao = oracle.site_moments(model_l20_k3, b.types, nl)
    assert np.max(np.abs(mom - bo)) < 1e-12 * max(1.0, np.max(np.abs(bo)))
    assert np.max(np.abs(adj - ao)) < 1e-11 * max(1.0, np.max(np.abs(ao)))
    # edge derivatives: match edges by (centre, neighbour, r) after sorting
    from helpers import canonical
    seo, dref = oracle.site_derivatives(model_l20_k3, b.types, nl)
    _, _, og = canonical(off, nbr, rij)
    _, _, oo = canonical(nl.offsets, nl.nbr, nl.rij)
    assert np.max(np.abs(d[og] - dref[oo])) < TOL_F
    assert np.max(np.abs(se - seo)) < TOL_E_ATOM


@pytest.mark.parametrize("seed", [1, 2])
def test_batched_level20_vs_oracle(oracle, model_l20_k3, seed):
    sts = configs.config2(32, seed=100 + seed)
    offs = configs.batch(sts)[0]
    b, (e, f, s, se), _, _, _ = _efs(model_l20_k3, sts)
    nl = _oracle_batch(oracle, model_l20_k3, sts, offs)
    eo, fo, so = oracle.efs_batch(model_l20_k3, offs, b.types, nl)
    nat = np.diff(offs)
    assert np.max(np.abs(e - eo) / nat) < TOL_E_ATOM
    assert np.max(np.abs(f - fo)) < TOL_F
    assert np.max(np.abs(s - so)) < TOL_W


def test_level16_config1_forces_finite_difference(model_l16):
    """Forces are -dE/dx of the GPU energy (central differences)."""
    from mtpb200 import MTPGpuDirect, StructureBatch
    st = configs.config1()
    h = 1e-5
    with MTPGpuDirect(model_l16, 0) as gpu:
        e0, f0, _, _ = gpu.efs(StructureBatch.from_structures([st]))
        for (i, dd) in [(0, 0), (17, 1), (200, 2)]:
            p1 = {**st, "positions": st["positions"].copy()}
            p2 = {**st, "positions": st["positions"].copy()}
            p1["positions"][i, dd] += h
            p2["positions"][i, dd] -= h
            ep = gpu.efs(StructureBatch.from_structures([p1]))[0][0]
            em = gpu.efs(StructureBatch.from_structures([p2]))[0][0]
            assert abs(-(ep - em) / (2 * h) - f0[i, dd]) < 1e-8
    assert np.max(np.abs(f0.sum(0))) < 1e-11


def test_update_coefficients_changes_results(oracle, model_l16):
    from mtpb200 import MTPGpuDirect, StructureBatch
    st = configs.config1()
    m2 = configs.seeded_coefficients(model_l16, 99)
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], model_l16.cutoff)
    eo, _, fo, _ = oracle.efs(m2, st["types"], nl)
    with MTPGpuDirect(model_l16, 0) as gpu:
        gpu.efs(StructureBatch.from_structures([st]))
        gpu.set_coefficients(m2.coefficients())
        e, f, _, _ = gpu.efs(StructureBatch.from_structures([st]))
    assert abs(e[0] - eo) / 256 < TOL_E_ATOM
    assert np.max(np.abs(f - fo)) < TOL_F


def test_deterministic_repeat(model_l20):
    """Two runs give bit-identical outputs (no atomics on the data path)."""
    from mtpb200 import MTPGpuDirect, StructureBatch
    st = configs.ni3al_l12(8, 3.52, 0.08, seed=3)
    b = StructureBatch.from_structures([st])
    with MTPGpuDirect(model_l20, 0) as gpu:
        r1 = gpu.efs(b, site_energy=True)
        r2 = gpu.efs(b, site_energy=True)
    for a, c in zip(r1, r2):
        assert np.array_equal(a, c)


def test_neighbor_reuse_with_skin_matches_fresh_build(oracle, model_l16):
    """MD-style reuse: build with a skin, move atoms by less than skin/2 and
    recompute with the stored periodic images (reuse_topology semantics)."""
    from mtpb200 import MTPGpuDirect, StructureBatch
    st = configs.config1()
    rng = np.random.default_rng(12)
    moved = {**st, "positions": st["positions"] + rng.uniform(-0.2, 0.2, st["positions"].shape)}
    b0 = StructureBatch.from_structures([st])
    b1 = StructureBatch.from_structures([moved])
    out = {"energy": np.zeros(1), "forces": np.zeros((256, 3)), "stress": np.zeros((1, 9))}
    with MTPGpuDirect(model_l16, 0) as gpu:
        gpu.set_skin(0.5)
        gpu.efs_structures(b0, reuse_neighbors=False, out=out)
        gpu.efs_structures(b1, reuse_neighbors=True, out=out)
        assert gpu.last_launch_count() < 12      # refresh, not a rebuild
    nl = oracle.neighbors(moved["cell"], moved["pbc"], moved["positions"], model_l16.cutoff)
    eo, _, fo, so = oracle.efs(model_l16, moved["types"], nl)
    assert abs(out["energy"][0] - eo) / 256 < TOL_E_ATOM
    assert np.max(np.abs(out["forces"] - fo)) < TOL_F
    assert np.max(np.abs(out["stress"][0] - so.reshape(9))) < TOL_W


def test_neighbor_reuse_unchanged_positions_bit_identical(model_l20):
    from mtpb200 import MTPGpuDirect, StructureBatch
    st = configs.ni3al_l12(6, 3.52, 0.08, seed=4)
    b = StructureBatch.from_structures([st])
    N = b.n_atoms
    o1 = {"energy": np.zeros(1), "forces": np.zeros((N, 3)), "stress": np.zeros((1, 9))}
    o2 = {k: np.zeros_like(v) for k, v in o1.items()}
    with MTPGpuDirect(model_l20, 0) as gpu:
        gpu.efs_structures(b, reuse_neighbors=False, out=o1)
        gpu.efs_structures(b, reuse_neighbors=True, out=o2)
    for k in o1:
        assert np.array_equal(o1[k], o2[k])


def test_energy_only_call_skips_the_reverse_pass(model_l20_k3):
    """An output without forces and stress returns the same energies with
    fewer launches, and no edge derivatives."""
    from mtpb200 import MTPBError, MTPGpuDirect, StructureBatch
    sts = configs.config2(3, seed=77)
    b = StructureBatch.from_structures(sts)
    with MTPGpuDirect(model_l20_k3, 0) as gpu:
        e, f, s, se = gpu.efs(b, site_energy=True)
        full = gpu.last_launch_count()
        out = dict(energy=np.zeros(len(sts)), site_energy=np.zeros(b.n_atoms))
        gpu.efs_structures(b, reuse_neighbors=False, out=out)
        assert gpu.last_launch_count() < full
        assert np.array_equal(out["energy"], e) and np.array_equal(out["site_energy"], se)
        with pytest.raises(MTPBError):
            gpu.edge_derivatives(10)
