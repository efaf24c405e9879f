"""Host logic of the slab decomposition (mtpb200.slab) on two gloo ranks on
the CPU: each rank evaluates the site terms of its own slab with the C oracle
on its rotated view of the whole box, then the collectives of SlabExchange
assemble forces, energy and virial, which must equal the single-process
oracle result.  Needs no GPU."""
import os
import socket

import numpy as np
import pytest

from mtpb200 import configs
from mtpb200.slab import SlabLayout

WS = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _box():
    st = configs.ni3al_l12(3, 3.52, 0.08, seed=5)
    return st


def _partial_efs(oracle, model, st, pos, types, ncenter):
    """Site terms of centres [0, ncenter) of a box given in local order."""
    nl = oracle.neighbors(st["cell"], st["pbc"], pos, model.cutoff)
    se, d = oracle.site_derivatives(model, types, nl)
    n = len(types)
    f = np.zeros((n, 3))
    w = np.zeros((3, 3))
    for i in range(ncenter):
        for e in range(nl.offsets[i], nl.offsets[i + 1]):
            f[i] += d[e]
            f[nl.nbr[e]] -= d[e]
            w -= np.outer(d[e], nl.rij[e])
    return se[:ncenter].sum(), f, w


def _rank_main(rank, port, result_dir):
    import sys
    import torch
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path.insert(0, os.path.join(root, "imr-mlp_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    from oracle import Oracle
    from mtpb200 import read_mtp
    from mtpb200.slab import SlabExchange, SlabLayout
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WS)
    try:
        O = Oracle()
        model = read_mtp(os.path.join(root, "tests", "golden", "models", "l16_k2.mtp"))
        st = _box()
        L = SlabLayout(st["cell"], st["positions"], WS)
        pos_slab = st["positions"][L.order]
        types_slab = st["types"][L.order]
        own = torch.from_numpy(pos_slab[L.starts[rank]:L.starts[rank + 1]].copy())
        X = SlabExchange(L, rank, dist, torch.device("cpu"))
        full = X.gather_positions(own).numpy()
        assert np.array_equal(full, pos_slab)
        pos_loc = L.to_local(full, rank)
        types_loc = L.to_local(types_slab, rank)
        e, f_loc, w = _partial_efs(O, model, st, pos_loc, types_loc, int(L.counts[rank]))
        f_own = X.reduce_forces(torch.from_numpy(L.to_slab(f_loc, rank).copy())).numpy()
        tot = X.reduce_totals(torch.tensor([e] + list(w.reshape(9)), dtype=torch.float64))
        np.savez(os.path.join(result_dir, f"rank{rank}.npz"), f_own=f_own, tot=tot.numpy())
    finally:
        dist.destroy_process_group()


def test_layout_rotation_roundtrip():
    st = _box()
    L = SlabLayout(st["cell"], st["positions"], 3)
    assert L.counts.sum() == len(st["types"]) and np.all(L.counts > 0)
    x = np.arange(L.natoms * 3, dtype=np.float64).reshape(-1, 3)
    for r in range(3):
        loc = L.to_local(x, r)
        assert np.array_equal(loc[:L.counts[r]], x[L.starts[r]:L.starts[r + 1]])
        assert np.array_equal(L.to_slab(loc, r), x)
        assert np.array_equal(loc, x[L.rotation(r)])


def test_two_gloo_ranks_match_single_process(oracle, model_l16, tmp_path):
    torch = pytest.importorskip("torch")
    import torch.multiprocessing as mp
    port = _free_port()
    mp.spawn(_rank_main, args=(port, str(tmp_path)), nprocs=WS, join=True)
    st = _box()
    L = SlabLayout(st["cell"], st["positions"], WS)
    pos_slab = st["positions"][L.order]
    types_slab = st["types"][L.order]
    nl = oracle.neighbors(st["cell"], st["pbc"], pos_slab, model_l16.cutoff)
    e, _, f, w = oracle.efs(model_l16, types_slab, nl)
    for r in range(WS):
        d = np.load(os.path.join(tmp_path, f"rank{r}.npz"))
        assert np.max(np.abs(d["f_own"] - f[L.starts[r]:L.starts[r + 1]])) < 1e-11
        assert abs(d["tot"][0] - e) < 1e-10 * len(types_slab)
        assert np.max(np.abs(d["tot"][1:] - w.reshape(9))) < 1e-9
