"""Seeded synthetic structures and model coefficients for the benchmark
configurations (no dataset is involved; every input is generated).

Species indices: Ni = 0, Al = 1, Cr = 2 for the metallic configurations;
Ru = 0, O = 1, H = 2 for the interface configuration.

Structures are plain dictionaries of numpy arrays:
``cell`` (3x3, rows are lattice vectors, Angstrom), ``pbc`` (3 ints),
``positions`` (N x 3), ``types`` (N int32).
"""
from __future__ import annotations

import dataclasses
from typing import Dict, List

import numpy as np

from .mtpfile import MTPModel

FCC_BASIS = np.array([[0.0, 0.0, 0.0], [0.5, 0.5, 0.0], [0.5, 0.0, 0.5], [0.0, 0.5, 0.5]])
BCC_BASIS = np.array([[0.0, 0.0, 0.0], [0.5, 0.5, 0.5]])


def _supercell(basis: np.ndarray, reps, a: float):
    """reps: cells per direction (int, or three ints for a non-cubic box)."""
    r = (reps, reps, reps) if np.isscalar(reps) else tuple(int(v) for v in reps)
    g = [np.arange(v) for v in r]
    cells = np.stack(np.meshgrid(*g, indexing="ij"), -1).reshape(-1, 3)
    frac = (cells[:, None, :] + basis[None, :, :]).reshape(-1, 3)
    return frac * a, np.diag(np.array(r, dtype=np.float64) * a)


def ni3al_l12(reps: int, a: float, sigma: float, seed: int) -> Dict[str, np.ndarray]:
    """Ni3Al L1_2: Al on the cube corner, Ni on the three face centres."""
    pos, cell = _supercell(FCC_BASIS, reps, a)
    types = np.tile(np.array([1, 0, 0, 0], dtype=np.int32), reps ** 3)
    rng = np.random.default_rng(seed)
    pos = pos + rng.normal(0.0, sigma, size=pos.shape)
    return {"cell": cell, "pbc": np.array([1, 1, 1], dtype=np.int32),
            "positions": np.ascontiguousarray(pos), "types": types}


def config1(seed: int = 1) -> Dict[str, np.ndarray]:
    """256-atom Ni3Al (4x4x4 cubic fcc cells), a=3.52, sigma=0.05."""
    return ni3al_l12(4, 3.52, 0.05, seed)


def config3(seed: int = 3, reps: int = 64) -> Dict[str, np.ndarray]:
    """1,048,576-atom Ni3Al box (64x64x64 cells), a=3.52, sigma=0.08."""
    return ni3al_l12(reps, 3.52, 0.08, seed)


def _strained(cell: np.ndarray, pos: np.ndarray, rng, amp: float):
    e = rng.uniform(-amp, amp, size=(3, 3))
    e = 0.5 * (e + e.T)
    F = np.eye(3) + e
    return cell @ F, pos @ F


def config2(n_struct: int = 4096, seed: int = 2) -> List[Dict[str, np.ndarray]]:
    """Random Ni/Al/Cr fcc alloys of 32/108/256 atoms, a=3.55, symmetric
    strain U(-0.03, 0.03), sigma=0.1."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n_struct):
        reps = int(rng.choice([2, 3, 4]))
        pos, cell = _supercell(FCC_BASIS, reps, 3.55)
        cell, pos = _strained(cell, pos, rng, 0.03)
        pos = pos + rng.normal(0.0, 0.1, size=pos.shape)
        types = rng.integers(0, 3, size=pos.shape[0]).astype(np.int32)
        out.append({"cell": cell, "pbc": np.array([1, 1, 1], dtype=np.int32),
                    "positions": np.ascontiguousarray(pos), "types": types})
    return out


def config4_shapes():
    """(lattice, cells per direction, lattice constant) of the config-4
    supercells: every fcc (a = 3.55) and bcc (a = 2.86) box of 2..6 cells per
    direction, sorted dimensions, with 64..216 atoms."""
    out = []
    for kind, per, a in (("fcc", 4, 3.55), ("bcc", 2, 2.86)):
        for n1 in range(2, 7):
            for n2 in range(n1, 7):
                for n3 in range(n2, 7):
                    if 64 <= per * n1 * n2 * n3 <= 216:
                        out.append((kind, (n1, n2, n3), a))
    return out


def config4_structures(n_struct: int = 8192, seed: int = 4) -> List[Dict[str, np.ndarray]]:
    """Ni/Al fcc or bcc supercells of 64-216 atoms (config4_shapes, drawn
    uniformly), random composition, symmetric strain U(-0.03, 0.03),
    sigma=0.1."""
    rng = np.random.default_rng(seed)
    choices = config4_shapes()
    out = []
    for _ in range(n_struct):
        kind, reps, a = choices[int(rng.integers(0, len(choices)))]
        basis = FCC_BASIS if kind == "fcc" else BCC_BASIS
        pos, cell = _supercell(basis, reps, a)
        cell, pos = _strained(cell, pos, rng, 0.03)
        pos = pos + rng.normal(0.0, 0.1, size=pos.shape)
        frac_al = rng.uniform(0.0, 1.0)
        types = (rng.uniform(size=pos.shape[0]) < frac_al).astype(np.int32)
        out.append({"cell": cell, "pbc": np.array([1, 1, 1], dtype=np.int32),
                    "positions": np.ascontiguousarray(pos), "types": types})
    return out


def _rotation(rng):
    q, _ = np.linalg.qr(rng.normal(size=(3, 3)))
    return q * np.sign(np.linalg.det(q))


def ru_water_interface(seed: int) -> Dict[str, np.ndarray]:
    """hcp Ru(0001) 6x6x4 slab (144 Ru, a = 2.706, c = 4.282, ABAB stacking)
    under a 15 A region holding 64 H2O (O-H 0.96 A, H-O-H 104.5 deg) at
    1.0 g/cm^3 (a 4x4 in-plane grid of 4 staggered layers, random
    orientations, starting 2 A above the top Ru layer), then 10 A of vacuum;
    Gaussian sigma 0.05 on every atom.  Types: Ru 0, O 1, H 2."""
    rng = np.random.default_rng(seed)
    a, c = 2.706, 4.282
    a1 = np.array([a, 0.0, 0.0])
    a2 = np.array([0.5 * a, 0.5 * np.sqrt(3.0) * a, 0.0])
    dz = 0.5 * c
    ru = []
    for layer in range(4):
        shift = (0.0, 0.0) if layer % 2 == 0 else (1.0 / 3.0, 1.0 / 3.0)
        for i in range(6):
            for j in range(6):
                ru.append((i + shift[0]) * a1 + (j + shift[1]) * a2 + np.array([0, 0, layer * dz]))
    ru = np.array(ru)
    top = 3 * dz
    area = 36 * a * a * 0.5 * np.sqrt(3.0)
    height = 64 * 18.015 / 6.02214076e23 / 1.0 * 1e24 / area   # A, at 1.0 g/cm^3
    theta = np.deg2rad(104.5) / 2
    mol = np.array([[0.0, 0.0, 0.0], [0.96 * np.sin(theta), 0.0, 0.96 * np.cos(theta)],
                    [-0.96 * np.sin(theta), 0.0, 0.96 * np.cos(theta)]])
    waters, wtypes = [], []
    for layer in range(4):
        st = 0.5 if layer % 2 else 0.0
        for i in range(4):
            for j in range(4):
                o = (1.5 * (i + st)) * a1 + (1.5 * (j + st)) * a2 + \
                    np.array([0, 0, top + 2.0 + (layer + 0.5) * height / 4])
                waters.append(o + mol @ _rotation(rng).T)
                wtypes += [1, 2, 2]
    pos = np.concatenate([ru, np.concatenate(waters)])
    pos = pos + rng.normal(0.0, 0.05, size=pos.shape)
    cell = np.array([6 * a1, 6 * a2, [0.0, 0.0, top + 15.0 + 10.0]])
    types = np.concatenate([np.zeros(len(ru), np.int32), np.array(wtypes, np.int32)])
    return {"cell": cell, "pbc": np.array([1, 1, 1], dtype=np.int32),
            "positions": np.ascontiguousarray(pos), "types": types}


def config5(n_copies: int = 1000, seed: int = 5) -> List[Dict[str, np.ndarray]]:
    """n_copies independently perturbed Ru(0001)/water interfaces (336 atoms
    each)."""
    return [ru_water_interface(seed * 100003 + k) for k in range(n_copies)]


def level24_model(species_count: int = 2, rmin: float = 2.0, rmax: float = 5.0,
                  rb_size: int = 8, seed: int = 24) -> MTPModel:
    """Generated level-24 basis (basisgen) with seeded U(-0.1, 0.1)
    coefficients: the stand-in for the level-24 models of configs 4 and 5."""
    from .basisgen import generate
    m = generate(24, species_count=species_count, min_dist=rmin, max_dist=rmax,
                 rb_size=rb_size)
    return seeded_coefficients(m, seed)


def seeded_coefficients(model: MTPModel, seed: int, low: float = -0.1,
                        high: float = 0.1) -> MTPModel:
    """All radial, species and moment coefficients drawn U(low, high)."""
    rng = np.random.default_rng(seed)
    c = rng.uniform(low, high, size=model.coeff_count)
    return model.with_coefficients(c)


def with_species(model: MTPModel, species_count: int, rmin: float, rmax: float,
                 rb_size: int = None) -> MTPModel:
    """Adapts a coefficient-free template header (species count, radial
    interval and size) as the benchmark configurations require."""
    R = rb_size or model.rb_size
    K = species_count
    return dataclasses.replace(
        model, species_count=K, rb_size=R, min_dist=np.array([rmin]), max_dist=np.array([rmax]),
        radial_basis_split=False, radial_coeffs=np.zeros(K * K * model.radial_func_count * R),
        species_coeffs=np.zeros(K), moment_coeffs=np.zeros(model.alpha_scalar_moments))


def batch(structures: List[Dict[str, np.ndarray]]):
    """Concatenates structures: returns (atom_offsets, cells[S,9], pbc[S,3],
    positions[N,3], types[N])."""
    offs = np.zeros(len(structures) + 1, dtype=np.int32)
    for i, s in enumerate(structures):
        offs[i + 1] = offs[i] + s["positions"].shape[0]
    cells = np.stack([s["cell"].reshape(9) for s in structures]).astype(np.float64)
    pbc = np.stack([s["pbc"] for s in structures]).astype(np.int32)
    pos = np.concatenate([s["positions"] for s in structures]).astype(np.float64)
    types = np.concatenate([s["types"] for s in structures]).astype(np.int32)
    return offs, np.ascontiguousarray(cells), np.ascontiguousarray(pbc), \
        np.ascontiguousarray(pos), np.ascontiguousarray(types)
