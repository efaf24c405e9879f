"""The halo slab decomposition on the GPU: every rank of a 2- and 3-rank
decomposition runs in this process on one GPU, each with its own library
context evaluating only its owned atoms (mtpb_set_center_count) over its
local structure (owned atoms plus ghost layers, stretched periodic cell),
with neighbour lists built with a skin and reused between rebuilds.  The
exchanges are handed over in process (LocalRanks); tests/test_slab.py runs
the same exchanges over gloo ranks.  Forces by global atom id, energy and
virial equal the single-process oracle after a rebuild, after reuse steps
and after a rebuild with migration."""
import numpy as np
import pytest

from mtpb200 import configs

pytestmark = pytest.mark.gpu

SKIN = 0.5


def _moves(n, seed=19):
    rng = np.random.default_rng(seed)
    small = rng.uniform(-0.12, 0.12, (2, n, 3))
    big = np.zeros((n, 3))
    big[:, 0] = 0.9
    big += rng.uniform(-0.1, 0.1, (n, 3))
    return [np.zeros((n, 3)), small[0], small[1], big]


STEPS = [(True, 0), (False, 1), (False, 2), (True, 3), (False, 2)]


@pytest.mark.parametrize("nranks", [2, 3])
def test_halo_slabs_match_oracle(oracle, model_l16, nranks):
    torch = pytest.importorskip("torch")
    from mtpb200 import MTPGpuDirect
    from mtpb200.slab import LocalRanks, SlabDomain
    dev = torch.device("cuda", 0)
    st = configs.ni3al_l12(6, 3.52, 0.08, seed=9)
    n = len(st["types"])
    moves = _moves(n)
    ds = [SlabDomain(st["cell"], nranks, r, model_l16.cutoff + SKIN, device=dev)
          for r in range(nranks)]
    for d in ds:
        d.assign(st["positions"], st["types"])
    lr = LocalRanks(ds)
    gpus = [MTPGpuDirect(model_l16, 0) for _ in range(nranks)]
    try:
        for g in gpus:
            g.set_skin(SKIN)
        prev = 0
        for rebuild, k in STEPS:
            for d in ds:
                ids = d.ids.cpu().numpy()
                d.pos = d.pos + torch.as_tensor(moves[k][ids] - moves[prev][ids], device=dev)
            prev = k
            if rebuild:
                lr.rebuild()
            xs = lr.positions()
            forces, e_tot, w_tot = [], 0.0, np.zeros(9)
            for d, g, x in zip(ds, gpus, xs):
                nl = x.shape[0]
                if rebuild:
                    g.set_center_count(d.n_own)
                offs = torch.tensor([0, nl], dtype=torch.int32, device=dev)
                cell = torch.as_tensor(d.local_cell.reshape(1, 9), device=dev)
                pbc = torch.ones((1, 3), dtype=torch.int32, device=dev)
                e = torch.zeros(1, dtype=torch.float64, device=dev)
                f = torch.zeros((nl, 3), dtype=torch.float64, device=dev)
                s = torch.zeros((1, 9), dtype=torch.float64, device=dev)
                g.efs_device(offs, cell, pbc, x.contiguous(), d.local_types().contiguous(), e, f,
                             s, reuse_neighbors=not rebuild)
                torch.cuda.synchronize()
                forces.append(f)
                e_tot += float(e.item())
                w_tot += s.cpu().numpy().reshape(9)
            fo = lr.forces(forces)
            f_all = np.zeros((n, 3))
            seen = np.zeros(n, np.int64)
            for d, ff in zip(ds, fo):
                ids = d.ids.cpu().numpy()
                f_all[ids] = ff.cpu().numpy()
                seen[ids] += 1
            assert np.all(seen == 1)
            pos = st["positions"] + moves[k]
            nl = oracle.neighbors(st["cell"], st["pbc"], pos, model_l16.cutoff)
            re, _, rf, rw = oracle.efs(model_l16, st["types"], nl)
            assert abs(e_tot - re) / n < 1e-10
            assert np.max(np.abs(f_all - rf)) < 1e-9
            assert np.max(np.abs(w_tot - rw.reshape(9))) < 1e-9
        assert sum(d.rebuilds for d in ds) == 2 * nranks
    finally:
        for g in gpus:
            g.close()
