"""Lists with a skin on the GPU: MD-style reuse over a batch of structures.

With a skin the neighbour list also holds pairs between r_c and r_c + skin.
Every compute then runs the active-edge pass: it tests each listed edge
against the pair cutoff with the staging arithmetic, compacts the active
edges (vector, neighbour, species pair) for the moment kernels, zeroes the
derivatives of the inactive ones and, on a reuse step, first recomputes
every edge vector from the moved positions and the stored periodic images.
Checked here against the oracle on the moved positions (energies, forces,
virials), on a ragged three-species batch with a level-20 model, over several
reuse steps, for energy-only calls, and for the per-edge derivatives (zero on
the edges beyond the cutoff, equal on the others to a list built without the
skin)."""
import numpy as np
import pytest

from mtpb200 import configs

pytestmark = pytest.mark.gpu

TOL_E_ATOM = 1e-10
TOL_F = 1e-9
TOL_W = 1e-9


def _moved(sts, seed, amp):
    rng = np.random.default_rng(seed)
    return [{**s, "positions": s["positions"] + rng.uniform(-amp, amp, s["positions"].shape)}
            for s in sts]


def _check_against_oracle(oracle, model, sts, out, offs):
    for k, s in enumerate(sts):
        a, b = offs[k], offs[k + 1]
        nl = oracle.neighbors(s["cell"], s["pbc"], s["positions"], model.cutoff)
        eo, _, fo, so = oracle.efs(model, s["types"], nl)
        assert abs(out["energy"][k] - eo) / (b - a) < TOL_E_ATOM
        assert np.max(np.abs(out["forces"][a:b] - fo)) < TOL_F
        assert np.max(np.abs(out["stress"][k] - so.reshape(9))) < TOL_W


def test_reuse_steps_with_skin_batch_level20(oracle, model_l20_k3):
    from mtpb200 import MTPGpuDirect, StructureBatch
    sts = configs.config2(5, seed=81)
    b0 = StructureBatch.from_structures(sts)
    N, S = b0.n_atoms, len(sts)
    out = {"energy": np.zeros(S), "forces": np.zeros((N, 3)), "stress": np.zeros((S, 9))}
    with MTPGpuDirect(model_l20_k3, 0) as gpu:
        gpu.set_skin(0.6)
        gpu.efs_structures(b0, reuse_neighbors=False, out=out)
        _check_against_oracle(oracle, model_l20_k3, sts, out, b0.atom_offsets)
        for step, amp in enumerate((0.12, 0.08, 0.14)):   # all within skin / 2
            moved = _moved(sts, 90 + step, amp)
            b = StructureBatch.from_structures(moved)
            gpu.efs_structures(b, reuse_neighbors=True, out=out)
            _check_against_oracle(oracle, model_l20_k3, moved, out, b.atom_offsets)
        # an energy-only reuse call gives the same energies
        e_full = out["energy"].copy()
        only = {"energy": np.zeros(S)}
        gpu.efs_structures(b, reuse_neighbors=True, out=only)
        assert np.max(np.abs(only["energy"] - e_full)) / N < TOL_E_ATOM


def test_edge_derivatives_with_skin(oracle, model_l16):
    """Edges between r_c and r_c + skin carry zero derivatives; the others
    carry those of a list built without the skin (matched by pair and
    displacement)."""
    from mtpb200 import MTPGpuDirect, StructureBatch
    st = configs.config1()
    moved = _moved([st], 7, 0.2)[0]
    b0 = StructureBatch.from_structures([st])
    b1 = StructureBatch.from_structures([moved])
    n = b0.n_atoms
    out = {"energy": np.zeros(1), "forces": np.zeros((n, 3)), "stress": np.zeros((1, 9))}

    def edges(gpu):
        import ctypes as C
        E = gpu.neighbor_count()
        offs = np.zeros(n + 1, np.int32)
        nbr = np.zeros(max(E, 1), np.int32)
        shift = np.zeros(max(E, 1), np.int32)
        r = np.zeros((max(E, 1), 3))
        assert gpu.lib.mtpb_get_neighbors(gpu.ctx, offs.ctypes.data_as(C.POINTER(C.c_int)),
                                          nbr.ctypes.data_as(C.POINTER(C.c_int)),
                                          r.ctypes.data_as(C.POINTER(C.c_double)),
                                          shift.ctypes.data_as(C.POINTER(C.c_int))) == 0
        d = gpu.edge_derivatives(E)
        centre = np.repeat(np.arange(n), np.diff(offs))
        # keyed by pair and displacement (a refreshed list keeps the build's
        # periodic images, whose shift codes a fresh build may number apart)
        return {(int(i), int(j)) + tuple(np.round(rr, 6)): (rr, dd) for i, j, rr, dd in
                zip(centre, nbr[:E], r[:E], d)}

    with MTPGpuDirect(model_l16, 0) as gpu:
        gpu.set_skin(0.5)
        gpu.efs_structures(b0, reuse_neighbors=False, out=out)
        gpu.efs_structures(b1, reuse_neighbors=True, out=out)
        skin = edges(gpu)
    with MTPGpuDirect(model_l16, 0) as gpu:
        gpu.efs_structures(b1, reuse_neighbors=False, out=out)
        plain = edges(gpu)
    rc = model_l16.cutoff
    n_beyond = 0
    for key, (r, d) in skin.items():
        if np.linalg.norm(r) > rc:
            n_beyond += 1
            assert np.all(d == 0.0)
        else:
            assert key in plain
            assert np.max(np.abs(d - plain[key][1])) < TOL_F
    assert n_beyond > 0
    assert len(skin) - n_beyond == len(plain)
