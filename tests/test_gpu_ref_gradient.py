"""Coefficient gradient pinned to the reference's own implementation.

The reference's PotMTP gradient (potentials/potential_mtp.cpp:3348-3550) does
not compile here, but its GPU trainer core does: MTPGpuDirect::compute_batch
-> prepare_loss -> accumulate_gradient (runtime/mtp/gpu-direct/
mtp_gpu_direct.cu:7980, 8261, 8651), built from the reference sources into
oracle/_ref/librefgpu.so and run in its deterministic FP64 mode.  The
reference holds that path to its CPU gradient within epsilon 4e-10 / margin
2e-8 (unitest/ut_mtp_cuda.cpp:1631-1769).

Compared here, on the same neighbour lists (the oracle's, equal bit for bit
to the reference Neighborhoods) and the same labels, with the trainer's
per-structure weights (train/train_mtp_gpu.cpp:252-292 with
Trainer_MTP::energy_weight etc., train/train_mtp.cpp:2552-2568):
  * mtpb_loss_grad (this library) against the reference, and
  * oracle_loss_grad (the CPU restatement) against the reference.

Tolerances: every gradient component within 1e-9 of its own magnitude plus an
absolute floor of 1e-12 x max|g| (components that cancel to near zero carry
rounding of the largest terms); metrics 1e-10 relative; forward energy per
atom 1e-10 eV, forces 1e-9 eV/A, site virials 1e-9 eV."""
import numpy as np
import pytest

from conftest import load_model
from mtpb200 import configs

pytestmark = pytest.mark.gpu

GRAD_REL = 1e-9
GRAD_FLOOR = 1e-12
TOL_METRIC = 1e-10
TOL_E_ATOM = 1e-10
TOL_F = 1e-9
TOL_W = 1e-9
CONFIG4_WEIGHTS = (1.0, 0.01, 0.001, 1.0, 0.0, 1.0)


@pytest.fixture(scope="module")
def refgpu_available():
    from oracle import ReferenceGpu
    if not ReferenceGpu.available():
        pytest.skip("oracle/_ref/librefgpu.so not built (reference checkout absent)")


def grad_errors(got, ref):
    """(max relative error over components, worst ratio of error to the
    allowed band)."""
    scale = float(np.max(np.abs(ref)))
    err = np.abs(got - ref)
    band = GRAD_REL * np.abs(ref) + GRAD_FLOOR * scale
    rel = err / np.maximum(np.abs(ref), 1e-300)
    return float(np.max(rel[np.abs(ref) > 1e-6 * scale])), float(np.max(err / band))


def assert_grad_close(got, ref, what):
    rel, worst = grad_errors(got, ref)
    print(f"{what}: max rel err (|g| > 1e-6 max) {rel:.3e}, worst err/band {worst:.3e}")
    assert worst <= 1.0, (what, rel, worst)


def _labels(structures, seed):
    rng = np.random.default_rng(seed)
    n = sum(len(s["types"]) for s in structures)
    return (rng.normal(0, 1, len(structures)), rng.normal(0, 0.1, (n, 3)),
            rng.normal(0, 0.5, (len(structures), 9)))


def _reference_weights(structures, weights):
    """Per-structure energy/stress and per-atom force weights as the GPU
    trainer fills them (w / N^power, atom fitness 1)."""
    we, wf, ws, pe, pf, ps = weights
    n = np.array([len(s["types"]) for s in structures], dtype=np.float64)
    return we / n ** pe, np.repeat(wf / n ** pf, n.astype(np.int64)), ws / n ** ps


def _compare(oracle, model, structures, weights, seed):
    from oracle import ReferenceGpu, concat_lists
    from mtpb200 import MTPGpuDirect, StructureBatch, format_mtp
    te, tf, ts = _labels(structures, seed)
    offs, _, _, _, types = configs.batch(structures)
    lists = [oracle.neighbors(s["cell"], s["pbc"], s["positions"], model.cutoff)
             for s in structures]
    nl = concat_lists(lists, offs)
    x = np.concatenate([oracle.wrap(s["cell"], s["pbc"], s["positions"]) for s in structures])
    ew, fw, sw = _reference_weights(structures, weights)
    S = len(structures)
    with ReferenceGpu(format_mtp(model), model.species_count, 0) as ref:
        rmetrics, rgrad, rf, rse, rsv = ref.loss_grad(offs, nl, types, x, te, ew, tf, fw, ts, sw)
    assert len(rgrad) == model.coeff_count
    with MTPGpuDirect(model, 0) as gpu:
        gpu.build_neighbors(StructureBatch.from_structures(structures))
        loss, metrics, grad = gpu.loss_grad(te, tf, ts, weights)
        e, f, _, se = gpu.efs(StructureBatch.from_structures(structures), site_energy=True)
    oloss, ometrics, ograd = oracle.loss_grad(model, offs, types, nl, te, tf, ts, weights)
    # forward pass of the reference GPU core against this library
    n_atoms = len(types)
    for s in range(S):
        a, b = offs[s], offs[s + 1]
        assert abs(rse[a:b].sum() - e[s]) / (b - a) < TOL_E_ATOM
    assert np.max(np.abs(rse - se)) < TOL_E_ATOM
    assert np.max(np.abs(rf - f)) < TOL_F
    # loss metrics (un-normalised) and the normalised loss
    assert np.all(np.abs(metrics - rmetrics) <= TOL_METRIC * np.maximum(1.0, np.abs(rmetrics)))
    assert abs(loss - rmetrics[0] / S) <= TOL_METRIC * max(1.0, abs(loss))
    assert np.all(np.abs(ometrics - rmetrics) <= TOL_METRIC * np.maximum(1.0, np.abs(rmetrics)))
    # the gradient: this library and the restatement against the reference
    assert_grad_close(grad, rgrad / S, "mtpb_loss_grad")
    assert_grad_close(ograd, rgrad / S, "oracle")
    assert n_atoms == offs[-1]


def test_gradient_level20_config4_structures(oracle, refgpu_available, model_l20):
    sts = configs.config4_structures(12, seed=4)
    _compare(oracle, model_l20, sts, CONFIG4_WEIGHTS, 21)


def test_gradient_level24_config4_structures(oracle, refgpu_available):
    model = configs.level24_model(2)
    sts = configs.config4_structures(6, seed=44)
    _compare(oracle, model, sts, CONFIG4_WEIGHTS, 22)


def test_gradient_split_radial_k3(oracle, refgpu_available):
    model = load_model("many_body_k3.mtp")
    sts = configs.config2(4, seed=65)
    _compare(oracle, model, sts, CONFIG4_WEIGHTS, 23)


@pytest.mark.parametrize("weights", [(2.0, 0.03, 0.5, 2.0, 1.0, 0.5),
                                     (0.0, 1.0, 0.0, 1.0, 0.0, 1.0)])
def test_gradient_weight_powers_level16(oracle, refgpu_available, model_l16, weights):
    sts = configs.config2(4, seed=66)
    for s in sts:
        s["types"] = np.minimum(s["types"], 1).astype(np.int32)
    _compare(oracle, model_l16, sts, weights, 24)

