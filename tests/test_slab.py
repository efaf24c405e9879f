"""Host logic of the slab decomposition with a ghost-atom halo exchange
(mtpb200.slab) on the CPU: 2 and 3 gloo ranks, and every rank of a
decomposition in one process (LocalRanks).  Each rank evaluates the site
terms of its owned atoms with the C oracle on its local structure (owned
atoms plus the ghost layers in the stretched periodic cell); the reverse
exchange returns the ghost forces to their owners.  Forces (by global atom
id), energy and virial must equal the single-process oracle on the whole box
after a rebuild, after reuse steps that only exchange positions, and after a
rebuild at which atoms migrate between slabs.  Needs no GPU."""
import os
import socket

import numpy as np
import pytest

from mtpb200 import configs

SKIN = 0.5
REPS = 6          # 21.1 A box: slabs of 10.6 / 7.0 A at 2 / 3 ranks, halo 5.5 A


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _box():
    return configs.ni3al_l12(REPS, 3.52, 0.08, seed=5)


def _moves(n, seed=17):
    """Per-atom displacements by global id: none for the first build, two
    small ones (below skin/2) for the reuse steps, then 0.9 A along x (plus
    noise) for the second rebuild, so that the atoms next to every slab face
    cross it and migrate."""
    rng = np.random.default_rng(seed)
    small = rng.uniform(-0.12, 0.12, (2, n, 3))
    big = np.zeros((n, 3))
    big[:, 0] = 0.9
    big += rng.uniform(-0.1, 0.1, (n, 3))
    return [np.zeros((n, 3)), small[0], small[1], big]


STEPS = [(True, 0), (False, 1), (False, 2), (True, 3)]   # (rebuild, displacement index)


def _partial_efs(oracle, model, cell, pos, types, ncenter):
    """Site terms of centres [0, ncenter) of a local structure: energy,
    forces on every local atom, virial."""
    nl = oracle.neighbors(cell, np.ones(3, np.int32), pos, model.cutoff)
    se, d = oracle.site_derivatives(model, types, nl)
    f = np.zeros((len(types), 3))
    w = np.zeros((3, 3))
    for i in range(ncenter):
        for e in range(nl.offsets[i], nl.offsets[i + 1]):
            f[i] += d[e]
            f[nl.nbr[e]] -= d[e]
            w -= np.outer(d[e], nl.rij[e])
    return float(se[:ncenter].sum()), f, w


def _reference(oracle, model, st, disp):
    pos = st["positions"] + disp
    nl = oracle.neighbors(st["cell"], st["pbc"], pos, model.cutoff)
    e, _, f, w = oracle.efs(model, st["types"], nl)
    return e, f, w.reshape(3, 3)


def test_local_ranks_match_single_process(oracle, model_l16):
    """All ranks in one process (LocalRanks) for 2 and 3 ranks."""
    torch = pytest.importorskip("torch")
    from mtpb200.slab import LocalRanks, SlabDomain
    st = _box()
    n = len(st["types"])
    moves = _moves(n)
    for nranks in (2, 3):
        ds = [SlabDomain(st["cell"], nranks, r, model_l16.cutoff + SKIN) for r in range(nranks)]
        for d in ds:
            d.assign(st["positions"], st["types"])
        assert sum(d.n_own for d in ds) == n
        lr = LocalRanks(ds)
        migrated = 0
        prev = 0
        for rebuild, k in STEPS:
            for d in ds:   # positions move continuously (the domain wraps them)
                ids = d.ids.numpy()
                d.pos = d.pos + torch.as_tensor(moves[k][ids] - moves[prev][ids])
            prev = k
            if rebuild:
                lr.rebuild()
                migrated += sum(d.migrated for d in ds)
            xs = lr.positions()
            parts = [_partial_efs(oracle, model_l16, d.local_cell, x.numpy(),
                                  d.local_types().numpy(), d.n_own) for d, x in zip(ds, xs)]
            fo = lr.forces([torch.from_numpy(p[1]) for p in parts])
            f = np.zeros((n, 3))
            seen = np.zeros(n, np.int64)
            for d, ff in zip(ds, fo):
                f[d.ids.numpy()] = ff.numpy()
                seen[d.ids.numpy()] += 1
            assert np.all(seen == 1)
            e_ref, f_ref, w_ref = _reference(oracle, model_l16, st, moves[k])
            assert abs(sum(p[0] for p in parts) - e_ref) / n < 1e-10
            assert np.max(np.abs(f - f_ref)) < 1e-9
            assert np.max(np.abs(sum(p[2] for p in parts) - w_ref)) < 1e-9
            # the halo is two layers, far less than the box
            assert all(d.n_ghost < n for d in ds)
        assert migrated > 0   # the last rebuild moved atoms between slabs


def _rank_main(rank, ws, port, result_dir):
    import sys
    import torch
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path.insert(0, os.path.join(root, "imr-mlp_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    from oracle import Oracle
    from mtpb200 import read_mtp
    from mtpb200.slab import DistributedSlab, SlabDomain
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        O = Oracle()
        model = read_mtp(os.path.join(root, "tests", "golden", "models", "l16_k2.mtp"))
        st = _box()
        n = len(st["types"])
        moves = _moves(n)
        d = SlabDomain(st["cell"], ws, rank, model.cutoff + SKIN)
        d.assign(st["positions"], st["types"])
        ds = DistributedSlab(d, dist)
        res = {}
        prev = 0
        for s, (rebuild, k) in enumerate(STEPS):
            ids = d.ids.numpy()
            d.pos = d.pos + torch.as_tensor(moves[k][ids] - moves[prev][ids])
            prev = k
            if rebuild:
                ds.rebuild()
            x = ds.positions()
            e, f, w = _partial_efs(O, model, d.local_cell, x.numpy(),
                                   d.local_types().numpy(), d.n_own)
            fo = ds.forces(torch.from_numpy(f))
            tot = ds.totals(torch.tensor([e] + list(w.reshape(9)), dtype=torch.float64))
            res[f"ids{s}"] = d.ids.numpy()
            res[f"f{s}"] = fo.numpy()
            res[f"tot{s}"] = tot.numpy()
            res[f"mig{s}"] = np.array([d.migrated if rebuild else 0])
        np.savez(os.path.join(result_dir, f"rank{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ws", [2, 3])
def test_gloo_ranks_match_single_process(oracle, model_l16, tmp_path, ws):
    pytest.importorskip("torch")
    import torch.multiprocessing as mp
    port = _free_port()
    mp.spawn(_rank_main, args=(ws, port, str(tmp_path)), nprocs=ws, join=True)
    st = _box()
    n = len(st["types"])
    moves = _moves(n)
    migrated = 0
    for s, (_, k) in enumerate(STEPS):
        e_ref, f_ref, w_ref = _reference(oracle, model_l16, st, moves[k])
        f = np.zeros((n, 3))
        seen = np.zeros(n, np.int64)
        for r in range(ws):
            d = np.load(os.path.join(tmp_path, f"rank{r}.npz"))
            f[d[f"ids{s}"]] = d[f"f{s}"]
            seen[d[f"ids{s}"]] += 1
            assert abs(d[f"tot{s}"][0] - e_ref) / n < 1e-10
            assert np.max(np.abs(d[f"tot{s}"][1:] - w_ref.reshape(9))) < 1e-9
            migrated += int(d[f"mig{s}"][0])
        assert np.all(seen == 1)
        assert np.max(np.abs(f - f_ref)) < 1e-9
    assert migrated > 0


def test_domain_geometry_and_limits():
    from mtpb200.slab import SlabDomain, interplanar_spacing
    st = _box()
    L = interplanar_spacing(st["cell"])
    assert abs(L - 3.52 * REPS) < 1e-9
    d = SlabDomain(st["cell"], 3, 1, 5.5)
    assert abs(d.h * L - 5.5) < 1e-12
    # the stretched direction holds slab + two halos + a gap wider than the halo
    assert d.extent * L > (d.width + 2 * d.h) * L + 5.5
    with pytest.raises(ValueError):
        SlabDomain(st["cell"], 4, 0, 5.5)     # 5.3 A slabs, thinner than the halo
    with pytest.raises(ValueError):
        SlabDomain(st["cell"], 1, 0, 5.5)
