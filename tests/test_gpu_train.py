"""Loss and coefficient gradient on the GPU (mtpb_loss_grad) against the C
restatement of Trainer_MTP::AddLossGard + PotMTP::AccumulateEFSCombinationGard
(oracle_loss_grad), the committed gradient fixture and central differences of
the GPU loss itself.

Tolerances: loss and metrics 1e-10 relative; every gradient component within
1e-9 of its own magnitude plus an absolute floor of 1e-12 times the largest
component (the device sums a factorised form of the reference's Jacobian
contraction in a different order, so components that cancel to near zero
carry the rounding of the largest terms)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, load_model
from mtpb200 import configs

pytestmark = pytest.mark.gpu

TOL_LOSS = 1e-10
TOL_GRAD = 1e-9
GRAD_FLOOR = 1e-12
WEIGHTS = (1.0, 0.01, 0.001, 1.0, 0.0, 1.0)


def _batch(structures):
    from mtpb200 import StructureBatch
    return StructureBatch.from_structures(structures)


def _oracle_grad(oracle, model, structures, te, tf, ts, weights=WEIGHTS):
    from oracle import concat_lists
    offs, _, _, _, types = configs.batch(structures)
    lists = [oracle.neighbors(s["cell"], s["pbc"], s["positions"], model.cutoff)
             for s in structures]
    nl = concat_lists(lists, offs)
    return oracle.loss_grad(model, offs, types, nl, te, tf, ts, weights)


def _labels(structures, seed):
    rng = np.random.default_rng(seed)
    n = sum(len(s["types"]) for s in structures)
    return (rng.normal(0, 1, len(structures)), rng.normal(0, 0.1, (n, 3)),
            rng.normal(0, 0.5, (len(structures), 9)))


def _gpu_grad(model, structures, te, tf, ts, weights=WEIGHTS, norm_count=0):
    from mtpb200 import MTPGpuDirect
    with MTPGpuDirect(model, 0) as gpu:
        gpu.build_neighbors(_batch(structures))
        return gpu.loss_grad(te, tf, ts, weights, norm_count)


def _close(got, ref):
    loss, metrics, grad = got
    rloss, rmetrics, rgrad = ref
    assert abs(loss - rloss) <= TOL_LOSS * max(1.0, abs(rloss))
    assert np.all(np.abs(metrics - rmetrics) <= TOL_LOSS * np.maximum(1.0, np.abs(rmetrics)))
    err = np.abs(grad - rgrad)
    band = TOL_GRAD * np.abs(rgrad) + GRAD_FLOOR * np.max(np.abs(rgrad))
    worst = int(np.argmax(err / np.maximum(band, 1e-300)))
    assert np.all(err <= band), (worst, float(err[worst]), float(rgrad[worst]),
                                 float(np.max(np.abs(rgrad))))


def _mixed(n, seed, K):
    sts = configs.config2(n, seed=seed)
    for s in sts:
        s["types"] = np.minimum(s["types"], K - 1).astype(np.int32)
    return sts


def test_gradient_matches_golden_fixture(model_l16):
    g = np.load(os.path.join(GOLDEN, "golden_grad_l16.npz"))
    offs = g["atom_offsets"]
    sts = [dict(cell=g["cells"][s].reshape(3, 3), pbc=np.ones(3, np.int32),
                positions=g["positions"][offs[s]:offs[s + 1]],
                types=g["types"][offs[s]:offs[s + 1]]) for s in range(len(offs) - 1)]
    # the fixture was made with the weights (1, 0.01, 0.0001; powers 1, 0, 1)
    got = _gpu_grad(model_l16, sts, g["target_energy"], g["target_forces"], g["target_stress"],
                    (1.0, 0.01, 0.0001, 1.0, 0.0, 1.0))
    _close(got, (float(g["loss"]), g["metrics"], g["grad"]))


@pytest.mark.parametrize("name,K", [("l16_k2.mtp", 2), ("l20_k3.mtp", 3),
                                    ("many_body_k3.mtp", 3), ("pair_k1.mtp", 1)])
def test_gradient_matches_oracle(oracle, name, K):
    m = load_model(name)
    sts = _mixed(3, 61, m.species_count)
    te, tf, ts = _labels(sts, 7)
    _close(_gpu_grad(m, sts, te, tf, ts), _oracle_grad(oracle, m, sts, te, tf, ts))


@pytest.mark.parametrize("weights", [(1.0, 0.0, 0.0, 1.0, 0.0, 1.0),
                                     (0.0, 1.0, 0.0, 1.0, 0.0, 1.0),
                                     (0.0, 0.0, 1.0, 1.0, 0.0, 1.0),
                                     (2.0, 0.03, 0.5, 2.0, 1.0, 0.5)])
def test_gradient_weight_variants(oracle, model_l16, weights):
    sts = _mixed(2, 62, 2)
    te, tf, ts = _labels(sts, 8)
    _close(_gpu_grad(model_l16, sts, te, tf, ts, weights),
           _oracle_grad(oracle, model_l16, sts, te, tf, ts, weights))


def test_gradient_missing_labels(oracle, model_l16):
    """A NULL label array drops that term for every structure."""
    sts = _mixed(2, 63, 2)
    te, tf, ts = _labels(sts, 9)
    _close(_gpu_grad(model_l16, sts, te, None, ts), _oracle_grad(oracle, model_l16, sts, te,
                                                                 None, ts))
    _close(_gpu_grad(model_l16, sts, None, tf, None), _oracle_grad(oracle, model_l16, sts, None,
                                                                   tf, None))


def test_gradient_norm_count_and_determinism(model_l16):
    sts = _mixed(3, 64, 2)
    te, tf, ts = _labels(sts, 10)
    from mtpb200 import MTPGpuDirect
    with MTPGpuDirect(model_l16, 0) as gpu:
        gpu.build_neighbors(_batch(sts))
        a = gpu.loss_grad(te, tf, ts, WEIGHTS)
        b = gpu.loss_grad(te, tf, ts, WEIGHTS)
        c = gpu.loss_grad(te, tf, ts, WEIGHTS, norm_count=12)
    assert a[0] == b[0] and np.array_equal(a[2], b[2]) and np.array_equal(a[1], b[1])
    assert np.allclose(c[2] * 12, a[2] * 3, rtol=1e-14, atol=0)
    assert np.array_equal(c[1], a[1])   # metrics are not normalised


def test_gradient_follows_coefficients_and_positions(oracle, model_l16):
    """The gradient program follows mtpb_update_coefficients, and the pair
    buckets follow a position update through the reuse path (list built
    with a skin, so the moved atoms stay inside it)."""
    from mtpb200 import MTPGpuDirect
    sts = _mixed(2, 65, 2)
    te, tf, ts = _labels(sts, 11)
    m2 = configs.seeded_coefficients(model_l16, 99)
    with MTPGpuDirect(model_l16, 0) as gpu:
        batch = _batch(sts)
        gpu.set_skin(0.5)
        gpu.build_neighbors(batch)
        gpu.loss_grad(te, tf, ts, WEIGHTS)
        gpu.set_coefficients(m2.coefficients())
        _close(gpu.loss_grad(te, tf, ts, WEIGHTS), _oracle_grad(oracle, m2, sts, te, tf, ts))
        rng = np.random.default_rng(3)
        moved = [dict(s, positions=s["positions"] + rng.normal(0, 0.01, s["positions"].shape))
                 for s in sts]
        out = dict(energy=np.zeros(len(sts)), forces=np.zeros((batch.n_atoms, 3)),
                   stress=np.zeros((len(sts), 9)))
        gpu.efs_structures(_batch(moved), reuse_neighbors=True, out=out)
        _close(gpu.loss_grad(te, tf, ts, WEIGHTS), _oracle_grad(oracle, m2, moved, te, tf, ts))


def test_gradient_central_differences(model_l16):
    """Directional derivatives of the GPU loss along radial, species and
    moment directions against the GPU gradient (central differences,
    step 1e-6 relative; unitest/ut_mtp_cpu_training.cpp:46-55 recipe)."""
    from mtpb200 import MTPGpuDirect
    sts = _mixed(2, 66, 2)
    te, tf, ts = _labels(sts, 12)
    m = model_l16
    c0 = m.coefficients()
    r = m.radial_coeffs_count
    K = m.species_count
    rng = np.random.default_rng(13)
    with MTPGpuDirect(m, 0) as gpu:
        gpu.build_neighbors(_batch(sts))
        _, _, g = gpu.loss_grad(te, tf, ts, WEIGHTS)
        for lo, hi in ((0, r), (r, r + K), (r + K, len(c0))):
            v = np.zeros_like(c0)
            v[lo:hi] = rng.normal(0, 1, hi - lo)
            h = 1e-6 * max(1.0, np.max(np.abs(c0[lo:hi])))
            gpu.set_coefficients(c0 + h * v)
            lp = gpu.loss_grad(te, tf, ts, WEIGHTS)[0]
            gpu.set_coefficients(c0 - h * v)
            lm = gpu.loss_grad(te, tf, ts, WEIGHTS)[0]
            gpu.set_coefficients(c0)
            fd = (lp - lm) / (2 * h)
            an = float(g @ v)
            assert abs(fd - an) <= 3e-5 + 3e-6 * abs(an), (lo, fd, an)


def test_level24_gradient_matches_oracle(oracle):
    """The config-4 workload's path: the generated level-24 graph (beyond
    shared memory: L2-resident dual-graph rows, 64 streams, split items), the
    two-pass edge kernel and the three-part launches, on three config-4
    structures, against the restated trainer."""
    m = configs.level24_model()
    sts = configs.config4_structures(3, seed=64)
    te, tf, ts = _labels(sts, 8)
    _close(_gpu_grad(m, sts, te, tf, ts), _oracle_grad(oracle, m, sts, te, tf, ts))


def test_nonfinite_label_is_reported(model_l16):
    """A NaN label makes the loss and gradient non-finite: host-memory calls
    return MTPB_ERR_NONFINITE (the reference's training_finite_kernel check,
    mtp_gpu_direct.cu:5395), device-memory calls leave the status to
    mtpb_check_training_values; a finite call afterwards is clean again."""
    torch = pytest.importorskip("torch")
    from mtpb200 import MTPBError, MTPGpuDirect
    sts = _mixed(2, 67, 2)
    te, tf, ts = _labels(sts, 14)
    bad = te.copy()
    bad[1] = np.nan
    with MTPGpuDirect(model_l16, 0) as gpu:
        gpu.build_neighbors(_batch(sts))
        with pytest.raises(MTPBError) as ei:
            gpu.loss_grad(bad, tf, ts, WEIGHTS)
        assert ei.value.status == 6 and "non-finite" in str(ei.value)
        gpu.loss_grad(te, tf, ts, WEIGHTS)
        assert gpu.check_training_values() == -1
        dev = torch.device("cuda", 0)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)   # noqa: E731
        loss = torch.zeros(1, dtype=torch.float64, device=dev)
        metrics = torch.zeros(7, dtype=torch.float64, device=dev)
        grad = torch.zeros(model_l16.coeff_count, dtype=torch.float64, device=dev)
        tf_bad = tf.copy()
        tf_bad[3, 1] = np.inf
        gpu.loss_grad_device(t(te), t(tf_bad), t(ts), loss, metrics, grad, WEIGHTS)
        with pytest.raises(MTPBError) as ei:
            gpu.check_training_values()
        assert ei.value.status == 6
        gpu.loss_grad_device(t(te), t(tf), t(ts), loss, metrics, grad, WEIGHTS)
        assert gpu.check_training_values() == -1
        assert torch.isfinite(grad).all()
