"""GPM v2 model bundles for linear MTP models: reader and writer.

GPM is the reference's binary model container (tools/gpm_container.h, MTP
schema tools/gpm_mtp.h, written by potentials/gpm_codec.cpp and read by the
LAMMPS core's loader, runtime/mtp/mlip.cpp:350-423).  Layout:

* a 64-byte preamble: the magic ``GPMLMODL``, the major version 2 (u16 at
  byte 8), required flags 0 (u32 at 12), the JSON header length (u64 at 16)
  and the data offset (u64 at 24) = the header's end rounded up to 64 bytes;
* the JSON header: schema ``gpml.model``, units, species, ``root_model``, the
  ``models`` object and the ``blocks`` directory (id, dtype, shape, codec,
  offset, stored and raw size; counts as decimal strings);
* the blocks: little-endian ``f64`` / ``i32`` arrays, each starting on a
  64-byte boundary relative to the data offset (codec ``none``).

An MTP model node holds ``type`` "mtp", ``version`` 1, a ``configuration``
(species_count, radial_functions, radial_size, moments_count, the radial
bases as string-valued objects in .mtp vocabulary, metadata, head_fields) and
``parameters`` that name the coefficient and index blocks.  RBPolyB bases
carry their orthogonalisation matrix and normalisations as blocks (the
reference keeps the eigensolver's rounded matrix as part of the model).
Per-pair radial scalings are folded into the radial coefficients on reading,
as the reference's loader does.
"""
from __future__ import annotations

import dataclasses
import json
import struct
from typing import Dict, List, Optional, Tuple

import numpy as np

from .mtpfile import MTPModel, RadialFamily, _fmt

MAGIC = b"GPMLMODL"
UNITS = {"length": "angstrom", "energy": "eV", "charge": "e", "stress": "virial_eV"}
_WIDTH = {"f64": 8, "i64": 8, "u64": 8, "i32": 4, "u32": 4, "u8": 1}


def _align64(x: int) -> int:
    return (x + 63) & ~63


def _basis_object(model: MTPModel, pair: int, fam: RadialFamily, blocks: "_Blocks") -> dict:
    """One radial basis of the configuration, string-valued as the .mtp text."""
    lo = float(model.min_dist[pair if model.radial_basis_split else 0])
    hi = float(model.max_dist[pair if model.radial_basis_split else 0])
    o = {"radial_basis_type": fam.name, "min_dist": _fmt(lo), "max_dist": _fmt(hi),
         "radial_basis_size": str(int(model.rb_size)), "scaling": _fmt(model.scaling)}
    for line in fam.lines():
        key, value = (s.strip() for s in line.split("=", 1))
        o[key] = value
    if fam.name in ("RBPolyB", "RBPolyBCos"):
        R = int(model.rb_size)
        o["polynomial"] = {
            "version": 1, "layout": "column_major",
            "matrix": {"block": blocks.add(f"radial_basis.{pair}.matrix", "f64", [R, R],
                                           np.asarray(fam.poly_matrix, dtype="<f8"))},
            "normalizations": {"block": blocks.add(f"radial_basis.{pair}.normalizations", "f64",
                                                   [R], np.asarray(fam.poly_norm, dtype="<f8"))}}
    return o


class _Blocks:
    def __init__(self):
        self.items: List[Tuple[str, str, List[int], bytes]] = []

    def add(self, bid: str, dtype: str, shape: List[int], data: np.ndarray) -> str:
        raw = np.ascontiguousarray(data).astype("<f8" if dtype == "f64" else "<i4").tobytes()
        n = int(np.prod(shape)) if shape else 1
        if n * _WIDTH[dtype] != len(raw):
            raise ValueError(f"GPM block {bid}: shape does not match its data")
        self.items.append((bid, dtype, list(shape), raw))
        return bid


def to_bytes(model: MTPModel, metadata: Optional[dict] = None) -> bytes:
    """The model as GPM v2 bytes (one root model of type "mtp")."""
    K, mu, R = model.species_count, model.radial_func_count, model.rb_size
    blocks = _Blocks()
    pairs = K * K if model.radial_basis_split else 1
    fams = model.radial_family or [RadialFamily()]
    bases = [_basis_object(model, p, fams[p if len(fams) > 1 else 0], blocks)
             for p in range(pairs)]
    params = {
        "radial": {"block": blocks.add("mtp.radial", "f64", [K, K, mu, R],
                                       np.asarray(model.radial_coeffs))},
        "species": {"block": blocks.add("mtp.species", "f64", [K],
                                        np.asarray(model.species_coeffs))},
        "moments": {"block": blocks.add("mtp.moments", "f64", [model.alpha_scalar_moments],
                                        np.asarray(model.moment_coeffs))},
        "basic_indices": {"block": blocks.add("mtp.basic_indices", "i32",
                                              [model.alpha_index_basic_count, 4],
                                              np.asarray(model.alpha_index_basic))},
        "product_indices": {"block": blocks.add("mtp.product_indices", "i32",
                                                [model.alpha_index_times_count, 4],
                                                np.asarray(model.alpha_index_times))},
        "scalar_mapping": {"block": blocks.add("mtp.scalar_mapping", "i32",
                                               [model.alpha_scalar_moments],
                                               np.asarray(model.alpha_moment_mapping))},
    }
    node = {"type": "mtp", "version": 1,
            "configuration": {"species_count": K, "radial_functions": mu, "radial_size": R,
                              "moments_count": int(model.alpha_moments_count),
                              "radial_bases": bases, "metadata": dict(metadata or {}),
                              "head_fields": []},
            "parameters": params}
    directory, payload, cursor = [], bytearray(), 0
    for bid, dtype, shape, raw in blocks.items:
        offset = _align64(cursor)
        payload += b"\0" * (offset - cursor)
        payload += raw
        cursor = offset + len(raw)
        directory.append({"id": bid, "dtype": dtype, "shape": [str(n) for n in shape],
                          "codec": "none", "offset": str(offset), "stored_size": str(len(raw)),
                          "raw_size": str(len(raw))})
    header = {"schema": "gpml.model", "units": dict(UNITS), "species": [],
              "root_model": "root", "models": {"root": node}, "blocks": directory}
    text = json.dumps(header, separators=(",", ":"), ensure_ascii=True).encode()
    start = _align64(64 + len(text))
    pre = MAGIC + struct.pack("<HHIQQ", 2, 0, 0, len(text), start) + b"\0" * 32
    return pre + text + b"\0" * (start - 64 - len(text)) + bytes(payload)


def write_gpm(model: MTPModel, path: str, metadata: Optional[dict] = None) -> None:
    with open(path, "wb") as f:
        f.write(to_bytes(model, metadata))


class GPMReader:
    """Container level: the header and its blocks (codec "none" only)."""

    def __init__(self, data: bytes):
        if len(data) < 64 or data[:8] != MAGIC:
            raise ValueError("GPM: invalid magic")
        major, _minor, flags, length, start = struct.unpack("<HHIQQ", data[8:32])
        if major != 2 or flags != 0:
            raise ValueError("GPM: unsupported version or required flags")
        if start != _align64(64 + length) or start > len(data):
            raise ValueError("GPM: invalid header size")
        self.manifest = json.loads(data[64:64 + length].decode("utf-8"))
        if self.manifest.get("schema") != "gpml.model":
            raise ValueError("GPM: unknown schema")
        if self.manifest.get("required_features"):
            raise ValueError("GPM: unsupported required features")
        self.data, self.start = data, start
        self.blocks: Dict[str, dict] = {}
        for b in self.manifest["blocks"]:
            if b["id"] in self.blocks:
                raise ValueError("GPM: duplicate block id")
            off, size, raw = int(b["offset"]), int(b["stored_size"]), int(b["raw_size"])
            n = int(np.prod([int(x) for x in b["shape"]])) if b["shape"] else 1
            if n * _WIDTH[b["dtype"]] != raw or off % 64 or start + off + size > len(data):
                raise ValueError(f"GPM: invalid block {b['id']}")
            if b["codec"] != "none" or size != raw:
                raise ValueError(f"GPM: block {b['id']} uses codec {b['codec']} (only 'none')")
            self.blocks[b["id"]] = b

    def array(self, ref: dict) -> np.ndarray:
        if "block" not in ref:
            return np.zeros([int(x) for x in ref["shape"]],
                            dtype=np.float64 if ref["dtype"] == "f64" else np.int32)
        b = self.blocks[ref["block"]]
        off = self.start + int(b["offset"])
        dt = {"f64": "<f8", "i32": "<i4"}[b["dtype"]]
        a = np.frombuffer(self.data[off:off + int(b["raw_size"])], dtype=dt)
        return a.astype(np.float64 if b["dtype"] == "f64" else np.int32).reshape(
            [int(x) for x in b["shape"]])


def from_bytes(data: bytes) -> MTPModel:
    """The root MTP model of GPM bytes."""
    from .mtpfile import CUTOFF_TYPES, SHIFT_TYPES, RADIAL_TYPES
    r = GPMReader(data)
    if r.manifest.get("units") != UNITS:
        raise ValueError("GPM: unsupported units")
    node = r.manifest["models"][r.manifest["root_model"]]
    if node.get("type") != "mtp" or node.get("version") != 1:
        raise ValueError("GPM: the root model is not a version-1 linear MTP")
    c, p = node["configuration"], node["parameters"]
    K, mu, R = c["species_count"], c["radial_functions"], c["radial_size"]
    bases = c["radial_bases"]
    split = len(bases) > 1
    if len(bases) not in (1, K * K):
        raise ValueError("GPM: invalid radial bases")
    radial = r.array(p["radial"]).reshape(-1).copy()
    scales = [float(b["scaling"]) for b in bases]
    scaling = scales[0]
    if any(s != scaling for s in scales):
        # one global scale: fold each pair's scale into its coefficients, as
        # the reference loader does (tools/gpm_mtp.h mtp_text)
        for pair in range(K * K):
            radial[pair * mu * R:(pair + 1) * mu * R] *= scales[pair if split else 0]
        scaling = 1.0
    fams, mins, maxs = [], [], []
    for b in bases:
        name = b["radial_basis_type"]
        if name not in RADIAL_TYPES:
            raise ValueError(f"GPM: radial basis '{name}' is not supported")
        f = RadialFamily(name=name)
        if "rb_b" in b:
            f.b = float(b["rb_b"])
        if "basis_function_type" in b:
            f.one_minus_chebyshev = b["basis_function_type"] == "one_minus_chebyshev"
        if "cutoff_type" in b:
            f.cutoff_type = b["cutoff_type"]
            if f.cutoff_type not in CUTOFF_TYPES:
                raise ValueError(f"GPM: unknown cutoff_type {f.cutoff_type}")
        if "cutoff_b" in b:
            f.b = float(b["cutoff_b"])
        f.r1 = float(b.get("cutoff_r1", 0.0))
        f.r2 = float(b.get("cutoff_r2", 0.0))
        if "shift_type" in b:
            f.shift_type = b["shift_type"]
            if f.shift_type not in SHIFT_TYPES:
                raise ValueError(f"GPM: unknown shift_type {f.shift_type}")
        f.shift_lambda = float(b.get("shift_lambda", 0.0))
        f.shift_scale_lambda = float(b.get("shift_scale_lambda", 0.0))
        if "polynomial" in b:
            poly = b["polynomial"]
            if poly.get("version") != 1 or poly.get("layout") != "column_major":
                raise ValueError("GPM: unsupported polynomial data format")
            f.poly_matrix = r.array(poly["matrix"]).reshape(R, R).reshape(-1).copy()
            f.poly_norm = r.array(poly["normalizations"]).reshape(-1).copy()
        elif name in ("RBPolyB", "RBPolyBCos"):
            from .mtpfile import polyb_data
            f.poly_matrix, f.poly_norm = polyb_data(float(b["min_dist"]), float(b["max_dist"]), R)
        if int(b["radial_basis_size"]) != R:
            raise ValueError("GPM: radial basis size differs from radial_size")
        fams.append(f)
        mins.append(float(b["min_dist"]))
        maxs.append(float(b["max_dist"]))
    plain = all(f.name == "RBChebyshev" for f in fams)
    basic = r.array(p["basic_indices"]).reshape(-1, 4)
    times = r.array(p["product_indices"]).reshape(-1, 4)
    mapping = r.array(p["scalar_mapping"]).reshape(-1)
    return MTPModel(
        potential_name="GPM", species_count=K, radial_func_count=mu, rb_size=R,
        radial_basis_split=split, min_dist=np.array(mins), max_dist=np.array(maxs),
        scaling=scaling, alpha_moments_count=int(c["moments_count"]),
        alpha_index_basic=basic.astype(np.int32), alpha_index_times=times.astype(np.int32),
        alpha_moment_mapping=mapping.astype(np.int32), radial_coeffs=radial,
        species_coeffs=r.array(p["species"]).reshape(-1).copy(),
        moment_coeffs=r.array(p["moments"]).reshape(-1).copy(),
        radial_family=None if plain else fams)


def read_gpm(path: str) -> MTPModel:
    with open(path, "rb") as f:
        return from_bytes(f.read())
