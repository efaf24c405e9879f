"""Radial basis families on the GPU (RBChebyCos, RBChebyshevPoly4/5, every
cutoff / shift of RBChebyshevConfigurable, RBPolyB and RBPolyBCos) against the
C restatement, which
is pinned to the compiled reference MLIPCore in test_oracle.py: EFS of a
level-16 model on the config-1 box and of a split level-20 model on strained
alloys, and the loss gradient (the radial-coefficient gradient uses the
basis values and derivatives of the same families).

Tolerances as for the Chebyshev basis: energies 1e-10 per atom, forces and
virials 1e-9, gradients 1e-9 of their largest entry."""
import dataclasses

import numpy as np
import pytest

from conftest import load_model
from helpers import RADIAL_CASES, with_radial_family
from mtpb200 import configs
from mtpb200.mtpfile import RadialFamily

pytestmark = pytest.mark.gpu


def _check_efs(oracle, model, sts):
    from mtpb200 import MTPGpuDirect, StructureBatch
    b = StructureBatch.from_structures(sts)
    with MTPGpuDirect(model, 0) as gpu:
        e, f, s, se = gpu.efs(b, site_energy=True)
    offs = b.atom_offsets
    for k, x in enumerate(sts):
        a0, a1 = offs[k], offs[k + 1]
        nl = oracle.neighbors(x["cell"], x["pbc"], x["positions"], model.cutoff)
        re, rse, rf, rs = oracle.efs(model, x["types"], nl)
        assert abs(e[k] - re) / (a1 - a0) < 1e-10, (e[k], re)
        assert np.max(np.abs(se[a0:a1] - rse)) < 1e-10
        assert np.max(np.abs(f[a0:a1] - rf)) < 1e-9
        assert np.max(np.abs(s[k] - rs)) < 1e-9


@pytest.mark.parametrize("case", sorted(RADIAL_CASES))
def test_radial_family_efs_level16(oracle, model_l16, case):
    _check_efs(oracle, with_radial_family(model_l16, case), [configs.config1()])


def test_split_mixed_families_level20(oracle, model_l20_k3):
    """A split level-20 basis with a different family on every species pair."""
    m = model_l20_k3
    K = m.species_count
    names = sorted(RADIAL_CASES)
    fams, mins = [], np.array(m.min_dist, dtype=np.float64)
    if not m.radial_basis_split:
        m = dataclasses.replace(m, radial_basis_split=True,
                                min_dist=np.full(K * K, m.min_dist[0]),
                                max_dist=np.full(K * K, m.max_dist[0]))
        mins = np.array(m.min_dist, dtype=np.float64)
    for p in range(K * K):
        spec = dict(RADIAL_CASES[names[(3 * p) % len(names)]])
        lo = spec.pop("min_dist", None)
        if lo is not None:
            mins[p] = lo
        fams.append(RadialFamily(**spec))
    m = dataclasses.replace(m, radial_family=fams, min_dist=mins)
    _check_efs(oracle, m, configs.config2(3, seed=81))


@pytest.mark.parametrize("case", ["chebycos", "poly5_min26", "cfg_smooth7_tanh_flip",
                                  "cfg_cosleft_expleft"])
def test_radial_family_gradient(oracle, model_l16, case):
    from test_gpu_train import _close, _gpu_grad, _labels, _mixed, _oracle_grad
    m = with_radial_family(model_l16, case)
    sts = _mixed(2, 83, m.species_count)
    te, tf, ts = _labels(sts, 9)
    _close(_gpu_grad(m, sts, te, tf, ts), _oracle_grad(oracle, m, sts, te, tf, ts))



@pytest.mark.parametrize("name,split", [("RBPolyB", False), ("RBPolyBCos", False),
                                        ("RBPolyB", True)])
def test_polyb_efs_and_gradient(oracle, reference, model_l16, name, split):
    """RBPolyB / RBPolyBCos with the reference loader's orthogonalisation
    matrix: the device evaluates powers of (max - r) with the matrix and
    normalisations folded into the coefficients, and maps the radial gradient
    back through them."""
    from helpers import with_polyb
    from test_gpu_train import _close, _gpu_grad, _labels, _mixed, _oracle_grad
    m = with_polyb(model_l16, name, reference, split=split)
    _check_efs(oracle, m, [configs.config1()])
    sts = _mixed(2, 84, m.species_count)
    te, tf, ts = _labels(sts, 10)
    _close(_gpu_grad(m, sts, te, tf, ts), _oracle_grad(oracle, m, sts, te, tf, ts))
