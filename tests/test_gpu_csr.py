"""Caller-supplied neighbour lists: the CSR batch request and the LAMMPS
pair-style request, against a closed-form known answer and the reference's
MLIPCore::compute."""
import numpy as np
import pytest

from conftest import load_model
from mtpb200 import configs

pytestmark = pytest.mark.gpu

# 4-atom cluster of the reference known-answer test (unitest/ut_mtp_cuda.cpp:46-135)
X4 = np.array([[0.0, 0.0, 0.0], [1.1, 0.2, -0.1], [-0.4, 1.3, 0.3], [0.2, -0.6, 1.4]])


def closed_form_energy(x, c0=0.7, c1=-0.2, species=0.3, m0=1.2, m1=-0.4, rmax=5.0):
    total = 0.0
    for i in range(len(x)):
        b0 = b1 = 0.0
        for j in range(len(x)):
            if i == j:
                continue
            rv = x[j] - x[i]
            r = np.sqrt(rv @ rv)
            ksi = (2.0 * r - rmax) / rmax
            rb0 = (r - rmax) ** 2
            rad = c0 * rb0 + c1 * ksi * rb0
            b0 += rad
            b1 += rad * rv[0] / r
        total += species + m0 * b0 + m1 * b1 * b1
    return total


def full_lists(n):
    off = np.arange(0, n * (n - 1) + 1, n - 1, dtype=np.int32)
    nbr = np.array([j for i in range(n) for j in range(n) if j != i], np.int32)
    return off, nbr


def test_known_answer_small_system_csr():
    from mtpb200 import MTPGpuDirect
    m = load_model("pair_k1.mtp")
    off, nbr = full_lists(4)
    with MTPGpuDirect(m, 0) as gpu:
        out = gpu.compute_batch(off, nbr | 0x40000000, np.zeros(4, np.int32), X4,
                                neighbor_mask=0x3FFFFFFF, site_virial=True)
        # forces against central differences of the closed form
        h = 1e-6
        for i in range(4):
            for d in range(3):
                xp, xm = X4.copy(), X4.copy()
                xp[i, d] += h
                xm[i, d] -= h
                fd = -(closed_form_energy(xp) - closed_form_energy(xm)) / (2 * h)
                assert abs(fd - out["force"][i, d]) < 2e-7
    ref = closed_form_energy(X4)
    assert abs(out["energy"] - ref) <= 1e-11 * abs(ref)
    assert abs(out["site_energy"].sum() - out["energy"]) < 1e-12
    assert np.max(np.abs(out["force"].sum(0))) < 1e-11
    # virial xx/xy against strain finite differences of the closed form
    eps = 1e-6
    for (a, b, q) in [(0, 0, 0), (0, 1, 3)]:
        F = np.eye(3)
        F[a, b] += eps
        ep = closed_form_energy(X4 @ F.T)
        F[a, b] -= 2 * eps
        em = closed_form_energy(X4 @ F.T)
        w = -(ep - em) / (2 * eps)
        gv = out["virial"][q]
        if q == 3:   # symmetric component vs one-sided strain derivative
            F = np.eye(3)
            F[b, a] += eps
            ep2 = closed_form_energy(X4 @ F.T)
            F[b, a] -= 2 * eps
            em2 = closed_form_energy(X4 @ F.T)
            w = 0.5 * (w - (ep2 - em2) / (2 * eps))
        assert abs(gv - w) < 5e-7
    assert np.max(np.abs(out["site_virial"].sum(0) - out["virial"])) < 1e-12


def _ghost_problem(oracle, model, st):
    """Full lists with explicit ghost atoms, as LAMMPS supplies them."""
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], model.cutoff)
    n = len(st["types"])
    E = nl.n_edges
    x0 = oracle.wrap(st["cell"], st["pbc"], st["positions"])
    centers = np.repeat(np.arange(n), np.diff(nl.offsets))
    x = np.concatenate([x0, x0[centers] + nl.rij])
    types = np.concatenate([st["types"], st["types"][nl.nbr]]).astype(np.int32)
    nbr = (n + np.arange(E)).astype(np.int32)
    return nl, x, types, nbr


def test_csr_with_ghosts_matches_mlipcore(oracle, reference, model_l16):
    from mtpb200 import MTPGpuDirect, format_mtp
    st = configs.config1()
    nl, x, types, nbr = _ghost_problem(oracle, model_l16, st)
    n = len(st["types"])
    e_ref, se_ref, f_ref, vir_ref = reference.mlip_efs(format_mtp(model_l16), st["types"], nl,
                                                       x[:n])
    with MTPGpuDirect(model_l16, 0) as gpu:
        out = gpu.compute_batch(nl.offsets, nbr, types, x, center_count=n, site_virial=True)
    f = out["force"][:n].copy()
    np.add.at(f, nl.nbr, out["force"][n:])
    assert abs(out["energy"] - e_ref) / n < 1e-10
    assert np.max(np.abs(out["site_energy"] - se_ref)) < 1e-10
    assert np.max(np.abs(f - f_ref)) < 1e-9
    assert np.max(np.abs(out["site_virial"] - vir_ref)) < 1e-9


def test_lammps_request_matches_csr(oracle, model_l16):
    """ilist order, masked neighbour bits, type map, accumulation into f."""
    from mtpb200 import MTPGpuDirect
    st = configs.config1()
    nl, x, types, nbr = _ghost_problem(oracle, model_l16, st)
    n = len(st["types"])
    NT = len(types)
    rng = np.random.default_rng(0)
    ilist = rng.permutation(n).astype(np.int32)
    numneigh = np.zeros(NT, np.int32)
    numneigh[:n] = np.diff(nl.offsets)
    first = [nbr[nl.offsets[i]:nl.offsets[i + 1]] | 0x40000000 if i < n else np.zeros(0, np.int32)
             for i in range(NT)]
    lmp_type = types + 1                       # LAMMPS types are 1-based
    tmap = np.array([-1, 0, 1], np.int32)
    f = np.full((NT, 3), 0.25)
    en = np.array([1.0])
    vir = np.zeros(6)
    sv = np.zeros((NT, 6))
    with MTPGpuDirect(model_l16, 0) as gpu:
        ref = gpu.compute_batch(nl.offsets, nbr, types, x, center_count=n, site_virial=True)
        gpu.compute_lammps(ilist, numneigh, first, lmp_type, tmap, x, f, energy=en,
                           site_virial=sv, virial=vir)
    assert np.max(np.abs((f - 0.25) - ref["force"])) < 1e-12
    assert abs(en[0] - 1.0 - ref["energy"]) < 1e-10
    assert np.max(np.abs(vir - ref["virial"])) < 1e-10
    assert np.max(np.abs(sv - ref["site_virial"])) < 1e-12


def test_skipped_types_like_mlipcore(oracle, reference, model_l16):
    """Atoms whose type maps to -1 are neither centres nor neighbours."""
    from mtpb200 import MTPGpuDirect
    st = configs.config1()
    nl, x, types, nbr = _ghost_problem(oracle, model_l16, st)
    n = len(st["types"])
    t2 = types.copy()
    t2[::7] = -1
    with MTPGpuDirect(model_l16, 0) as gpu:
        out = gpu.compute_batch(nl.offsets, nbr, t2, x, center_count=n)
    # same result as removing those atoms from the lists
    keep_edges = t2[nbr] >= 0
    cen = np.repeat(np.arange(n), np.diff(nl.offsets))
    keep = keep_edges & (t2[cen] >= 0)
    off2 = np.zeros(n + 1, np.int32)
    np.add.at(off2, cen[keep] + 1, 1)
    off2 = np.cumsum(off2).astype(np.int32)
    with MTPGpuDirect(model_l16, 0) as gpu:
        out2 = gpu.compute_batch(off2, nbr[keep], np.where(t2 < 0, 0, t2), x, center_count=n)
    mask = t2[:n] >= 0
    assert abs(out["energy"] - (out2["site_energy"][mask]).sum()) < 1e-10
    assert np.all(out["site_energy"][~mask] == 0)
