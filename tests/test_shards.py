"""Configuration sharding (mtpb200.shards) on two gloo ranks on the CPU: the
training step (each rank's loss and gradient on its LPT shard, normalised by
the global structure count, then one all-reduce of [loss, metrics, gradient])
and the batched EFS (each rank's shard, energies by structure, one
all-reduce of the energy total) equal the single-process oracle.  The
reference splits its training set over MPI ranks the same way
(train/train_mtp.cpp:3061-3085).  Needs no GPU."""
import os
import socket

import numpy as np
import pytest

from mtpb200 import configs

WS = 2
WEIGHTS = (1.0, 0.01, 0.001, 1.0, 0.0, 1.0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    sts = configs.config2(7, seed=71)
    for s in sts:
        s["types"] = np.minimum(s["types"], 1).astype(np.int32)
    rng = np.random.default_rng(72)
    n = sum(len(s["types"]) for s in sts)
    te = rng.normal(0, 1, len(sts))
    tf = rng.normal(0, 0.1, (n, 3))
    ts = rng.normal(0, 0.5, (len(sts), 9))
    return sts, te, tf, ts


def _slices(sts, idx, te, tf, ts):
    offs = np.concatenate([[0], np.cumsum([len(s["types"]) for s in sts])])
    f = np.concatenate([tf[offs[i]:offs[i + 1]] for i in idx]) if idx else np.zeros((0, 3))
    return te[idx], f, ts[idx]


def _lists(oracle, model, structures):
    from oracle import concat_lists
    offs, _, _, _, types = configs.batch(structures)
    nl = concat_lists([oracle.neighbors(s["cell"], s["pbc"], s["positions"], model.cutoff)
                       for s in structures], offs)
    return offs, types, nl


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
    from mtpb200.shards import allreduce_loss_grad, shard_lpt, shard_of
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WS)
    try:
        O = Oracle()
        model = read_mtp(os.path.join(root, "tests", "golden", "models", "l16_k2.mtp"))
        sts, te, tf, ts = _problem()
        owner = shard_lpt([len(s["types"]) for s in sts], WS)
        mine, idx = shard_of(sts, owner, rank)
        offs, types, nl = _lists(O, model, mine)
        lte, ltf, lts = _slices(sts, idx, te, tf, ts)
        # the oracle normalises by its own structure count: rescale to the
        # global count, as mtpb_loss_grad's norm_count does on the device
        loss, metrics, grad = O.loss_grad(model, offs, types, nl, lte, ltf, lts, WEIGHTS)
        scale = len(mine) / len(sts)
        out = torch.tensor(np.concatenate([[loss * scale], metrics, grad * scale]))
        allreduce_loss_grad(dist, out)
        # batched EFS of the shard; energies scattered by structure index
        e, f, s = O.efs_batch(model, offs, types, nl)
        energies = torch.zeros(len(sts), dtype=torch.float64)
        energies[idx] = torch.from_numpy(e)
        dist.all_reduce(energies)
        np.savez(os.path.join(result_dir, f"rank{rank}.npz"), out=out.numpy(),
                 energies=energies.numpy(), owner=owner, n_mine=len(mine))
    finally:
        dist.destroy_process_group()


def test_lpt_balances_and_covers():
    from mtpb200.shards import shard_lpt
    sizes = [256, 32, 108, 256, 108, 32, 32, 256]
    owner = shard_lpt(sizes, 3)
    loads = np.bincount(owner, weights=sizes, minlength=3)
    assert sorted(loads) == [352, 364, 364]
    assert set(owner) == {0, 1, 2}
    assert np.array_equal(shard_lpt(sizes, 3), owner)   # deterministic


def test_two_gloo_ranks_match_single_process(oracle, model_l16, tmp_path):
    pytest.importorskip("torch")
    import torch.multiprocessing as mp
    port = _free_port()
    mp.spawn(_rank_main, args=(port, str(tmp_path)), nprocs=WS, join=True)
    sts, te, tf, ts = _problem()
    offs, types, nl = _lists(oracle, model_l16, sts)
    loss, metrics, grad = oracle.loss_grad(model_l16, offs, types, nl, te, tf, ts, WEIGHTS)
    e, _, _ = oracle.efs_batch(model_l16, offs, types, nl)
    ref = np.concatenate([[loss], metrics, grad])
    outs = [np.load(os.path.join(tmp_path, f"rank{r}.npz")) for r in range(WS)]
    assert all(o["n_mine"] > 0 for o in outs)
    for o in outs:
        got = o["out"]
        band = 1e-9 * np.abs(ref) + 1e-12 * np.max(np.abs(ref))
        assert np.all(np.abs(got - ref) <= band)
        assert np.max(np.abs(o["energies"] - e)) < 1e-10 * max(len(t["types"]) for t in sts)
