"""Generates the committed parity fixtures under tests/golden/.

Run in a checkout that has the reference source tree and the compiled
reference oracle (``make -C oracle``):

    python tests/golden/make_fixtures.py --reference /path/to/reference

Outputs
-------
models/*.mtp
    Benchmark and test models: the coefficient-free Shapeev basis templates
    shipped with the reference (unitest/test-data/mtp-basis-corpus/shapeev-16
    and shapeev-20) with the benchmark header edits (species count, radial
    interval and size, explicit ``scaling``) and seeded U(-0.1, 0.1)
    coefficients; plus two small hand-made models (a many-body split-basis
    model and a single-channel model) written from scratch here.
golden_*.npz
    Outputs of the reference's own CPU code (oracle/_ref: ``Neighborhoods``
    with -DBOXED_NEBH and ``MLIPCore::compute``) on seeded structures, plus
    one gradient fixture from the C restatement (pinned by finite
    differences in tests/test_oracle.py, because the reference's gradient code
    needs libraries absent here).
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "imr-mlp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

from mtpb200 import configs, mtpfile  # noqa: E402
from mtpb200.mtpfile import MTPModel  # noqa: E402
from helpers import canonical_digest  # noqa: E402

SEEDS = {"l16_k2": 11, "l20_k3": 12, "l20_k2": 13}


def many_body_model(species: int = 3) -> MTPModel:
    """Small split-basis model: scalar density, squared vector moment and
    squared density, asymmetric per-pair radii and coefficients."""
    K = species
    mins = np.full(K * K, 0.5)
    maxs = np.array([4.0 + 0.4 * (i + j) for i in range(K) for j in range(K)])
    radial = np.zeros(K * K * 2)
    for i in range(K):
        for j in range(K):
            radial[(i * K + j) * 2:(i * K + j) * 2 + 2] = [0.03 * (i + 1) / (j + 1),
                                                             0.01 * (i - j + 1)]
    basic = np.array([[0, 0, 0, 0], [0, 1, 0, 0], [0, 0, 1, 0], [0, 0, 0, 1]], np.int32)
    times = np.array([[1, 1, 1, 4], [2, 2, 1, 4], [3, 3, 1, 4], [0, 0, 1, 5]], np.int32)
    return MTPModel(species_count=K, radial_func_count=1, rb_size=2, min_dist=mins,
                    max_dist=maxs, alpha_moments_count=6, alpha_index_basic=basic,
                    alpha_index_times=times, alpha_moment_mapping=np.array([0, 4, 5], np.int32),
                    radial_coeffs=radial, species_coeffs=-0.2 * (np.arange(K) + 1),
                    moment_coeffs=np.array([-0.15, 0.004, 0.005]), scaling=1.0,
                    radial_basis_split=True, potential_name="many_body")


def pair_model() -> MTPModel:
    """Single channel, density and one vector moment: E_i = s + c0 b0 + c1 b1^2."""
    basic = np.array([[0, 0, 0, 0], [0, 1, 0, 0]], np.int32)
    times = np.array([[1, 1, 1, 2]], np.int32)
    return MTPModel(species_count=1, radial_func_count=1, rb_size=2, min_dist=np.array([0.0]),
                    max_dist=np.array([5.0]), alpha_moments_count=3, alpha_index_basic=basic,
                    alpha_index_times=times, alpha_moment_mapping=np.array([0, 2], np.int32),
                    radial_coeffs=np.array([0.7, -0.2]), species_coeffs=np.array([0.3]),
                    moment_coeffs=np.array([1.2, -0.4]), scaling=1.0, potential_name="pair")


def small_cells(seed: int = 21):
    """Edge-case geometries: a cell thinner than the cutoff, a skewed cell
    and a single atom."""
    rng = np.random.default_rng(seed)
    out = []
    cell = np.array([[2.6, 0.0, 0.0], [1.3, 2.25, 0.0], [1.3, 0.75, 2.12]])
    pos = np.array([[0.0, 0.0, 0.0], [1.3, 0.75, 1.06]]) + rng.normal(0, 0.05, (2, 3))
    out.append({"cell": cell, "pbc": np.ones(3, np.int32), "positions": pos,
                "types": np.array([0, 1], np.int32)})
    cell = np.array([[6.0, 0.4, -0.3], [0.9, 5.5, 0.2], [-0.5, 0.7, 7.1]])
    frac = rng.uniform(0, 1, (12, 3))
    out.append({"cell": cell, "pbc": np.ones(3, np.int32), "positions": frac @ cell + 0.3,
                "types": rng.integers(0, 2, 12).astype(np.int32)})
    out.append({"cell": np.eye(3) * 3.1, "pbc": np.ones(3, np.int32),
                "positions": np.array([[0.2, -0.1, 3.3]]), "types": np.array([1], np.int32)})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("IMRMLP_REFERENCE", "/root/reference"),
                    help="reference checkout (default: $IMRMLP_REFERENCE)")
    args = ap.parse_args()
    from oracle import Oracle, Reference
    O, R = Oracle(), Reference()
    corpus = os.path.join(args.reference, "unitest", "test-data", "mtp-basis-corpus")
    os.makedirs(os.path.join(HERE, "models"), exist_ok=True)
    t16 = mtpfile.read_mtp(os.path.join(corpus, "shapeev-16.mtp"))
    t20 = mtpfile.read_mtp(os.path.join(corpus, "shapeev-20.mtp"))
    models = {
        "l16_k2": configs.seeded_coefficients(configs.with_species(t16, 2, 2.0, 5.0, 8),
                                              SEEDS["l16_k2"]),
        "l20_k3": configs.seeded_coefficients(configs.with_species(t20, 3, 2.0, 5.0, 8),
                                              SEEDS["l20_k3"]),
        "l20_k2": configs.seeded_coefficients(configs.with_species(t20, 2, 2.0, 5.0, 8),
                                              SEEDS["l20_k2"]),
        "many_body_k3": many_body_model(3),
        "pair_k1": pair_model(),
    }
    for name, m in models.items():
        m = MTPModel(**{**m.__dict__, "scaling": m.scaling if name in ("many_body_k3", "pair_k1")
                        else 0.01, "potential_name": name})
        mtpfile.write_mtp(m, os.path.join(HERE, "models", name + ".mtp"))
        models[name] = mtpfile.read_mtp(os.path.join(HERE, "models", name + ".mtp"))

    def ref_efs(model, st):
        nl = R.neighbors(st["cell"], st["pbc"], st["positions"], model.cutoff)
        wrapped = O.wrap(st["cell"], st["pbc"], st["positions"])
        e, se, f, vir = R.mlip_efs(mtpfile.format_mtp(model), st["types"], nl, wrapped)
        n = len(st["types"])
        gv = vir.sum(axis=0)
        return nl, e, se, f, gv

    # config 1: Ni3Al 256 atoms, level 16
    st = configs.config1()
    nl, e, se, f, gv = ref_efs(models["l16_k2"], st)
    np.savez_compressed(os.path.join(HERE, "golden_config1_l16.npz"),
                        cell=st["cell"], positions=st["positions"], types=st["types"],
                        counts=np.diff(nl.offsets).astype(np.int32),
                        digest=np.array(canonical_digest(nl.offsets, nl.nbr, nl.rij)),
                        energy=e, site_energy=se, forces=f, virial6=gv)
    # strained ternary alloys, level 20 (full lists stored)
    sts = configs.config2(3, seed=77)
    payload = {}
    for k, st in enumerate(sts):
        nl, e, se, f, gv = ref_efs(models["l20_k3"], st)
        payload.update({f"s{k}_cell": st["cell"], f"s{k}_positions": st["positions"],
                        f"s{k}_types": st["types"], f"s{k}_offsets": nl.offsets,
                        f"s{k}_nbr": nl.nbr, f"s{k}_rij": nl.rij, f"s{k}_energy": e,
                        f"s{k}_site_energy": se, f"s{k}_forces": f, f"s{k}_virial6": gv})
    np.savez_compressed(os.path.join(HERE, "golden_config2_l20.npz"), count=len(sts), **payload)
    # small / thin / skewed cells with the split-basis many-body model
    payload = {}
    cells = small_cells()
    for k, st in enumerate(cells):
        m = models["many_body_k3"]
        nl, e, se, f, gv = ref_efs(m, st)
        payload.update({f"s{k}_cell": st["cell"], f"s{k}_positions": st["positions"],
                        f"s{k}_types": st["types"], f"s{k}_offsets": nl.offsets,
                        f"s{k}_nbr": nl.nbr, f"s{k}_rij": nl.rij, f"s{k}_energy": e,
                        f"s{k}_site_energy": se, f"s{k}_forces": f, f"s{k}_virial6": gv})
    np.savez_compressed(os.path.join(HERE, "golden_small_cells.npz"), count=len(cells), **payload)
    # gradient regression fixture (C restatement; FD-pinned by the tests)
    sts = configs.config2(2, seed=91)
    offs, cells_, pbc, pos, types = configs.batch(sts)
    m = models["l16_k2"]
    lists = [O.neighbors(s["cell"], s["pbc"], s["positions"], m.cutoff) for s in sts]
    from oracle import concat_lists
    nl = concat_lists(lists, offs)
    rng = np.random.default_rng(5)
    te = rng.normal(0, 1, len(sts))
    tf = rng.normal(0, 0.1, (len(types), 3))
    ts = rng.normal(0, 0.5, (len(sts), 9))
    tsel = np.where(types > 1, 1, types).astype(np.int32)
    loss, metrics, grad = O.loss_grad(m, offs, tsel, nl, te, tf, ts)
    np.savez_compressed(os.path.join(HERE, "golden_grad_l16.npz"), atom_offsets=offs, cells=cells_,
                        positions=pos, types=tsel, target_energy=te, target_forces=tf,
                        target_stress=ts, loss=loss, metrics=metrics, grad=grad)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
