"""The CPU oracle pinned against the reference's own code and the golden
fixtures (CPU only)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, load_model
from helpers import RADIAL_CASES, with_radial_family
from mtpb200 import configs, format_mtp
from oracle import concat_lists


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float64).view(np.int64)


def _same_lists(a, b):
    a, b = a.canonical(), b.canonical()
    return (np.array_equal(a.offsets, b.offsets) and np.array_equal(a.nbr, b.nbr)
            and np.array_equal(_bits(a.rij), _bits(b.rij)))


def test_oracle_neighbors_match_reference_config1(oracle, reference):
    st = configs.config1()
    a = oracle.neighbors(st["cell"], st["pbc"], st["positions"], 5.0)
    b = reference.neighbors(st["cell"], st["pbc"], st["positions"], 5.0)
    assert a.n_edges == b.n_edges > 0
    assert _same_lists(a, b)


@pytest.mark.parametrize("seed", [3, 4])
def test_oracle_neighbors_match_reference_strained(oracle, reference, seed):
    for st in configs.config2(6, seed=seed):
        a = oracle.neighbors(st["cell"], st["pbc"], st["positions"], 5.0)
        b = reference.neighbors(st["cell"], st["pbc"], st["positions"], 5.0)
        assert _same_lists(a, b)


def test_oracle_neighbors_symmetric(oracle):
    """Every (i -> j, r) has (j -> i, -r) exactly (neighborhood.cpp:121,130)."""
    st = configs.config2(1, seed=8)[0]
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], 5.0)
    centers = np.repeat(np.arange(len(nl.offsets) - 1), np.diff(nl.offsets))
    fwd = set(zip(centers, nl.nbr, *(_bits(nl.rij).T)))
    back = set(zip(nl.nbr, centers, *(_bits(-nl.rij).T)))
    assert fwd == back


def test_oracle_neighbors_golden_config1(oracle):
    g = np.load(os.path.join(GOLDEN, "golden_config1_l16.npz"))
    from helpers import canonical_digest
    nl = oracle.neighbors(g["cell"], np.ones(3, np.int32), g["positions"], 5.0)
    assert np.array_equal(np.diff(nl.offsets), g["counts"])
    assert canonical_digest(nl.offsets, nl.nbr, nl.rij) == str(g["digest"])


def test_oracle_efs_golden_config1(oracle, model_l16):
    g = np.load(os.path.join(GOLDEN, "golden_config1_l16.npz"))
    nl = oracle.neighbors(g["cell"], np.ones(3, np.int32), g["positions"], model_l16.cutoff)
    e, se, f, s = oracle.efs(model_l16, g["types"], nl)
    assert abs(e - float(g["energy"])) < 1e-12 * max(1.0, abs(e))
    assert np.max(np.abs(se - g["site_energy"])) < 1e-13
    assert np.max(np.abs(f - g["forces"])) < 1e-13
    sym = [s[0, 0], s[1, 1], s[2, 2], 0.5 * (s[0, 1] + s[1, 0]), 0.5 * (s[0, 2] + s[2, 0]),
           0.5 * (s[1, 2] + s[2, 1])]
    assert np.max(np.abs(np.array(sym) - g["virial6"])) < 1e-12


def test_oracle_golden_config2_level20(oracle, model_l20_k3):
    g = np.load(os.path.join(GOLDEN, "golden_config2_l20.npz"))
    for k in range(int(g["count"])):
        nl = oracle.neighbors(g[f"s{k}_cell"], np.ones(3, np.int32), g[f"s{k}_positions"],
                              model_l20_k3.cutoff)
        from oracle import NeighborList
        ref = NeighborList(g[f"s{k}_offsets"], g[f"s{k}_nbr"], g[f"s{k}_rij"])
        assert _same_lists(nl, ref)
        e, se, f, s = oracle.efs(model_l20_k3, g[f"s{k}_types"], nl)
        assert abs(e - float(g[f"s{k}_energy"])) < 1e-11
        assert np.max(np.abs(f - g[f"s{k}_forces"])) < 1e-11


def test_oracle_golden_small_cells(oracle):
    m = load_model("many_body_k3.mtp")
    g = np.load(os.path.join(GOLDEN, "golden_small_cells.npz"))
    from oracle import NeighborList
    for k in range(int(g["count"])):
        nl = oracle.neighbors(g[f"s{k}_cell"], np.ones(3, np.int32), g[f"s{k}_positions"],
                              m.cutoff)
        ref = NeighborList(g[f"s{k}_offsets"], g[f"s{k}_nbr"], g[f"s{k}_rij"])
        assert _same_lists(nl, ref)
        e, se, f, s = oracle.efs(m, g[f"s{k}_types"], nl)
        assert abs(e - float(g[f"s{k}_energy"])) < 1e-12
        assert np.max(np.abs(f - g[f"s{k}_forces"]), initial=0) < 1e-12


def test_oracle_efs_matches_mlipcore(oracle, reference, model_l16):
    st = configs.config2(1, seed=31)[0]
    types = np.where(st["types"] > 1, 1, st["types"]).astype(np.int32)
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], model_l16.cutoff)
    e, se, f, s = oracle.efs(model_l16, types, nl)
    e2, se2, f2, _ = reference.mlip_efs(format_mtp(model_l16), types, nl,
                                        oracle.wrap(st["cell"], st["pbc"], st["positions"]))
    assert abs(e - e2) < 1e-12 * max(1, abs(e))
    assert np.max(np.abs(f - f2)) < 1e-12


def test_oracle_forces_finite_difference(oracle):
    """Forces are -dE/dx (central differences, ut_mtp_cuda.cpp:1170-1280 recipe)."""
    m = load_model("pair_k1.mtp")
    cell = np.eye(3) * 12.0
    pos = np.array([[0.0, 0.0, 0.0], [1.1, 0.2, -0.1], [-0.4, 1.3, 0.3], [0.2, -0.6, 1.4]]) + 5.0
    types = np.zeros(4, np.int32)

    def energy(p):
        nl = oracle.neighbors(cell, np.ones(3, np.int32), p, m.cutoff)
        return oracle.efs(m, types, nl)[0]

    nl = oracle.neighbors(cell, np.ones(3, np.int32), pos, m.cutoff)
    _, _, f, _ = oracle.efs(m, types, nl)
    h = 1e-6
    for i in range(4):
        for d in range(3):
            p1, p2 = pos.copy(), pos.copy()
            p1[i, d] += h
            p2[i, d] -= h
            fd = -(energy(p1) - energy(p2)) / (2 * h)
            assert abs(fd - f[i, d]) < 2e-7
    assert np.max(np.abs(f.sum(axis=0))) < 1e-11


def _grad_fixture():
    g = np.load(os.path.join(GOLDEN, "golden_grad_l16.npz"))
    return g


def test_oracle_gradient_golden(oracle, model_l16):
    g = _grad_fixture()
    offs = g["atom_offsets"]
    cells = g["cells"]
    lists = [oracle.neighbors(cells[s], np.ones(3, np.int32), g["positions"][offs[s]:offs[s + 1]],
                              model_l16.cutoff) for s in range(len(offs) - 1)]
    nl = concat_lists(lists, offs)
    loss, metrics, grad = oracle.loss_grad(model_l16, offs, g["types"], nl, g["target_energy"],
                                           g["target_forces"], g["target_stress"])
    assert abs(loss - float(g["loss"])) < 1e-12 * max(1, abs(loss))
    assert np.max(np.abs(grad - g["grad"])) < 1e-12 * max(1, np.max(np.abs(grad)))


@pytest.mark.slow
def test_oracle_gradient_finite_difference(oracle):
    """dL/dc against central differences, step 1e-6*max(1,|c|)
    (unitest/ut_mtp_cpu_training.cpp:46-55 recipe)."""
    m = load_model("many_body_k3.mtp")
    st = configs.config2(1, seed=44)[0]
    types = st["types"]
    offs = np.array([0, len(types)], np.int32)
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], m.cutoff)
    rng = np.random.default_rng(3)
    te = np.array([rng.normal()])
    tf = rng.normal(0, 0.05, (len(types), 3))
    ts = rng.normal(0, 0.2, 9)
    c0 = m.coefficients()
    loss, _, grad = oracle.loss_grad(m, offs, types, nl, te, tf, ts)
    for k in range(len(c0)):
        h = 1e-6 * max(1.0, abs(c0[k]))
        cp, cm = c0.copy(), c0.copy()
        cp[k] += h
        cm[k] -= h
        lp = oracle.loss_grad(m.with_coefficients(cp), offs, types, nl, te, tf, ts)[0]
        lm = oracle.loss_grad(m.with_coefficients(cm), offs, types, nl, te, tf, ts)[0]
        fd = (lp - lm) / (2 * h)
        assert abs(fd - grad[k]) <= 3e-5 * max(1e-3, abs(fd)) + 3e-9, (k, fd, grad[k])


@pytest.mark.parametrize("case", ["level24_k2", "config5_k3_r10"])
def test_oracle_efs_matches_mlipcore_generated_level24(oracle, reference, case):
    """The C restatement against the compiled reference MLIPCore on the
    generated level-24 stand-ins (configs 4 and 5 models)."""
    if case == "level24_k2":
        m = configs.level24_model()
        st = configs.config4_structures(1, seed=33)[0]
    else:
        m = configs.level24_model(species_count=3, rmin=0.8, rmax=6.0, rb_size=10, seed=55)
        st = configs.ru_water_interface(3)
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], m.cutoff)
    e, se, f, s = oracle.efs(m, st["types"], nl)
    e2, se2, f2, _ = reference.mlip_efs(format_mtp(m), st["types"], nl,
                                        oracle.wrap(st["cell"], st["pbc"], st["positions"]))
    assert abs(e - e2) < 1e-12 * max(1, abs(e))
    assert np.max(np.abs(f - f2)) < 1e-11 * max(1.0, np.max(np.abs(f)))


@pytest.mark.parametrize("case", sorted(RADIAL_CASES))
def test_oracle_radial_families_match_mlipcore(oracle, reference, model_l16, case):
    """Every radial family (and configurable cutoff / shift) of the C
    restatement, which follows basis/basis.cpp, cutoff.cpp and xtrans.cpp,
    against the compiled reference MLIPCore reading the same .mtp text
    (runtime/mtp/radial_basis.h)."""
    m = with_radial_family(model_l16, case)
    st = configs.config1()
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], m.cutoff)
    e, se, f, s = oracle.efs(m, st["types"], nl)
    e2, se2, f2, _ = reference.mlip_efs(format_mtp(m), st["types"], nl,
                                        oracle.wrap(st["cell"], st["pbc"], st["positions"]))
    assert abs(e - e2) < 1e-11 * max(1, abs(e)), (e, e2)
    assert np.max(np.abs(f - f2)) < 1e-10 * max(1.0, np.max(np.abs(f)))
    assert np.max(np.abs(se - se2)) < 1e-11 * max(1.0, np.max(np.abs(se)))


@pytest.mark.parametrize("case", sorted(RADIAL_CASES))
def test_mtp_radial_family_round_trip(case, model_l16):
    from mtpb200 import parse_mtp
    m = with_radial_family(model_l16, case)
    m2 = parse_mtp(format_mtp(m))
    assert m2.radial_family == m.radial_family
    assert np.array_equal(m2.min_dist, m.min_dist)


@pytest.mark.parametrize("name,split", [("RBPolyB", False), ("RBPolyBCos", False),
                                        ("RBPolyB", True)])
def test_oracle_polyb_matches_mlipcore(oracle, reference, model_l16, name, split):
    """RBPolyB / RBPolyBCos of the C restatement (the reference loader's
    orthogonalisation matrix, evaluate_polynomial's order) against the
    compiled reference MLIPCore reading the same .mtp text."""
    from helpers import with_polyb
    m = with_polyb(model_l16, name, reference, split=split)
    st = configs.config1()
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], m.cutoff)
    e, se, f, s = oracle.efs(m, st["types"], nl)
    e2, se2, f2, _ = reference.mlip_efs(format_mtp(m), st["types"], nl,
                                        oracle.wrap(st["cell"], st["pbc"], st["positions"]))
    assert abs(e - e2) < 1e-12 * max(1, abs(e)), (e, e2)
    assert np.max(np.abs(f - f2)) < 1e-11 * max(1.0, np.max(np.abs(f)))
    assert np.max(np.abs(se - se2)) < 1e-12 * max(1.0, np.max(np.abs(se)))
    assert np.max(np.abs(f)) > 0


def test_polyb_numpy_matrix_is_an_approximation(oracle, reference, model_l16):
    """mtpfile.polyb_data (numpy's eigensolver) against the reference loader's
    matrix (Eigen's): the overlap matrix's condition number is 1.3e13 at R = 8,
    so the two matrices differ at about 1e-4 of their largest entry and the
    energies they give by ~1e-8 eV/atom, far above the parity tolerance.  This
    is why the library takes the matrix as model data (the C++ binding passes
    the reference loader's own)."""
    from helpers import with_polyb
    approx = with_polyb(model_l16, "RBPolyB")
    ref = with_polyb(model_l16, "RBPolyB", reference)
    M1 = np.asarray(approx.radial_family[0].poly_matrix)
    M2 = np.asarray(ref.radial_family[0].poly_matrix)
    assert np.allclose(approx.radial_family[0].poly_norm, ref.radial_family[0].poly_norm,
                       rtol=1e-14, atol=0)
    assert np.max(np.abs(M1 - M2)) < 1e-3 * np.max(np.abs(M2))
    st = configs.config1()
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], model_l16.cutoff)
    e1 = oracle.efs(approx, st["types"], nl)[0]
    e2 = oracle.efs(ref, st["types"], nl)[0]
    assert abs(e1 - e2) / len(st["types"]) < 1e-6
