"""The reference-side binding MTPB200Direct (imr-mlp_b200/bindings/
mtpb_direct.hpp), compiled against the reference's own headers with its
runtime/mtp/mlip.cpp (oracle/_ref/librefdirect.so): a model loaded by
MLIPCore::setup_from_text goes to the GPU through initialize_from_mlip, and
compute_batch (MTPGpuBatchRequest) and compute_lammps (MTPGpuComputeRequest)
must reproduce MLIPCore::compute (runtime/mtp/mlip.cpp:906-1193) on the same
explicit-ghost problem, for plain, split and non-Chebyshev radial bases.

Tolerances (absolute): energy per atom and site energies 1e-10 eV, forces
1e-9 eV/A, per-atom virials 1e-9 eV."""
import numpy as np
import pytest

from conftest import load_model
from helpers import with_radial_family
from mtpb200 import configs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def binding_available():
    from oracle import ReferenceBinding
    if not ReferenceBinding.available():
        pytest.skip("oracle/_ref/librefdirect.so not built (reference checkout absent)")


def _ghost_problem(oracle, model, st):
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], model.cutoff)
    n = len(st["types"])
    x0 = oracle.wrap(st["cell"], st["pbc"], st["positions"])
    centers = np.repeat(np.arange(n), np.diff(nl.offsets))
    x = np.concatenate([x0, x0[centers] + nl.rij])
    types = np.concatenate([st["types"], st["types"][nl.nbr]]).astype(np.int32)
    nbr = (n + np.arange(nl.n_edges)).astype(np.int32)
    return nl, x, types, nbr


MODELS = [("l16_k2.mtp", None), ("l20_k3.mtp", None), ("many_body_k3.mtp", None),
          ("l16_k2.mtp", "chebycos"), ("l16_k2.mtp", "poly5"),
          ("l16_k2.mtp", "cfg_smooth7_tanh_flip")]


@pytest.mark.parametrize("name,case", MODELS)
def test_binding_compute_batch_matches_mlipcore(oracle, reference, binding_available, name,
                                                case):
    from oracle import ReferenceBinding
    from mtpb200 import format_mtp
    model = load_model(name)
    if case:
        model = with_radial_family(model, case)
    st = configs.config1()
    nl, x, types, nbr = _ghost_problem(oracle, model, st)
    n = len(st["types"])
    text = format_mtp(model)
    e_ref, se_ref, f_ref, vir_ref = reference.mlip_efs(text, st["types"], nl, x[:n])
    with ReferenceBinding(text, model.species_count, 0) as b:
        out = b.compute_batch(n, nl.offsets, nbr, types, x)
        out_v = b.compute_batch(n, nl.offsets, nl.nbr, types[:n], x[:n], vectors=nl.rij)
    f = out["force"][:n].copy()
    np.add.at(f, nl.nbr, out["force"][n:])
    assert abs(out["energy"] - e_ref) / n < 1e-10
    assert np.max(np.abs(out["site_energy"] - se_ref)) < 1e-10
    assert np.max(np.abs(f - f_ref)) < 1e-9
    assert np.max(np.abs(out["site_virial"] - vir_ref)) < 1e-9
    assert np.max(np.abs(out["virial"] - vir_ref.sum(0))) < 1e-9 * n
    # the periodic form with explicit vectors (the trainer's batch request)
    assert abs(out_v["energy"] - e_ref) / n < 1e-10
    assert np.max(np.abs(out_v["force"] - f_ref)) < 1e-9


def test_binding_compute_lammps_matches_batch(oracle, reference, binding_available, model_l16):
    from oracle import ReferenceBinding
    from mtpb200 import format_mtp
    st = configs.config1()
    nl, x, types, nbr = _ghost_problem(oracle, model_l16, st)
    n = len(st["types"])
    nt = len(types)
    rng = np.random.default_rng(5)
    ilist = rng.permutation(n).astype(np.int32)
    numneigh = np.zeros(nt, np.int32)
    numneigh[:n] = np.diff(nl.offsets)
    first_off = np.zeros(nt, np.int32)
    first_off[:n] = nl.offsets[:-1]
    flat = nbr | 0x40000000           # a special-bond flag above the index mask
    text = format_mtp(model_l16)
    e_ref, se_ref, f_ref, vir_ref = reference.mlip_efs(text, st["types"], nl, x[:n])
    force = np.full((nt, 3), 0.5)
    sv = np.zeros((nt, 6))
    with ReferenceBinding(text, model_l16.species_count, 0) as b:
        e, se, gv = b.compute_lammps(ilist, types, x, numneigh, first_off, flat, 0x3FFFFFFF,
                                     force, sv)
    f = force[:n] - 0.5
    np.add.at(f, nl.nbr, force[n:] - 0.5)
    assert abs(e - e_ref) / n < 1e-10
    assert np.max(np.abs(se[:n] - se_ref)) < 1e-10
    assert np.max(np.abs(f - f_ref)) < 1e-9
    assert np.max(np.abs(sv - vir_ref)) < 1e-9



@pytest.mark.parametrize("name", ["RBPolyB", "RBPolyBCos"])
def test_binding_polyb_matches_mlipcore(oracle, reference, binding_available, model_l16, name):
    """A PolyB model loaded by MLIPCore goes through the binding with the
    loader's own orthogonalisation matrix."""
    from helpers import with_polyb
    from oracle import ReferenceBinding
    from mtpb200 import format_mtp
    model = with_polyb(model_l16, name)      # the text only; the loader makes the matrix
    st = configs.config1()
    nl, x, types, nbr = _ghost_problem(oracle, model, st)
    n = len(st["types"])
    text = format_mtp(model)
    e_ref, se_ref, f_ref, vir_ref = reference.mlip_efs(text, st["types"], nl, x[:n])
    with ReferenceBinding(text, model.species_count, 0) as b:
        out = b.compute_batch(n, nl.offsets, nbr, types, x)
    f = out["force"][:n].copy()
    np.add.at(f, nl.nbr, out["force"][n:])
    assert abs(out["energy"] - e_ref) / n < 1e-10
    assert np.max(np.abs(out["site_energy"] - se_ref)) < 1e-10
    assert np.max(np.abs(f - f_ref)) < 1e-9
    assert np.max(np.abs(out["site_virial"] - vir_ref)) < 1e-9
