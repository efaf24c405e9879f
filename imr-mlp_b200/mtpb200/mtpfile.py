"""Reader and writer for the MTP 1.1.0 text format (``.mtp``).

The layout follows the reference reader ``PotMTP::Load``
(potentials/potential_mtp.cpp:119-576) and the standalone reader
``MLIPCore::setup_from_text`` (runtime/mtp/mlip.cpp:430-805):

* header ``MTP`` / ``version = 1.1.0``, optional ``potential_name``, optional
  ``scaling`` (absent means 0.01 in ``PotMTP::Load`` but 1.0 in MLIPCore, so
  :func:`write_mtp` always writes it), ``species_count``, optional
  ``potential_tag``;
* one radial basis, or ``radial_basis_split = 1`` followed by one ``pair i j``
  block per ordered species pair; a basis is ``RBChebyshev``, ``RBChebyCos``,
  ``RBChebyshevPoly4`` / ``RBChebyshevPoly5`` (with ``rb_b``) or
  ``RBChebyshevConfigurable`` (``basis_function_type``, ``cutoff_type`` with
  ``cutoff_b`` / ``cutoff_r1``, ``cutoff_r2``, ``shift_type`` with
  ``shift_lambda`` / ``shift_scale_lambda``), as read by the basis loaders of
  basis/basis.cpp, basis/cutoff.cpp:450-460 and basis/xtrans.cpp:361-371;
* ``radial_funcs_count`` and optional ``radial_coeffs`` as ``i-j`` blocks of
  ``radial_funcs_count`` rows of ``radial_basis_size`` values;
* the moment graph: ``alpha_index_basic`` {mu, a, b, c}, ``alpha_index_times``
  {l1, l2, c, id}, ``alpha_moment_mapping``;
* optional ``species_coeffs`` and ``moment_coeffs``.

The polynomial families RBPolyB and RBPolyBCos are rejected with a clear
error (the B200 kernels implement the Chebyshev families above).
"""
from __future__ import annotations

import dataclasses
import re
from typing import List, Optional

import numpy as np

__all__ = ["MTPModel", "RadialFamily", "parse_mtp", "read_mtp", "write_mtp", "format_mtp"]

# numbering of mtpb_radial_type / mtpb_radial_cutoff / mtpb_radial_shift
# (include/mtpb200.h; RadialBasis, RadialCutoff, RadialTransform of
# runtime/mtp/gpu-direct/mtp_gpu_direct.h:152-186)
RADIAL_TYPES = {"RBChebyshev": 0, "RBChebyCos": 1, "RBChebyshevPoly5": 2,
                "RBChebyshevConfigurable": 3, "RBChebyshevPoly4": 4, "RBPolyB": 5,
                "RBPolyBCos": 6}
POLYB_TYPES = ("RBPolyB", "RBPolyBCos")


def polyb_data(rmin: float, rmax: float, size: int):
    """Orthogonalisation matrix (column-major, flattened [size*size]) and power
    normalisations [size] of the RBPolyB families, by their definition
    (runtime/mtp/radial_basis_setup.cpp, basis/basis.cpp): the power p = i + 1
    has normalisation sqrt((2p + 5) / (max - min)^(2p + 5)); the overlap matrix
    S_ij = sqrt((2p_i + 5)(2p_j + 5)) / (p_i + p_j + 5) gives M = S^(-1/2)
    through its eigendecomposition.  S is ill-conditioned (1.3e13 at R = 8), so
    M depends on the eigensolver's rounding: numpy's differs from the
    reference's (Eigen's) at ~1e-4 of its largest entry, which moves energies
    by ~1e-8 eV/atom.  For parity with the reference, a model must carry the
    reference loader's own matrix (the C++ binding passes it; the tests take it
    from the compiled reference); this one is an approximation for models
    that never met the reference."""
    p = np.arange(1, size + 1, dtype=np.float64)
    norm = np.sqrt((2 * p + 5) / np.power(rmax - rmin, 2 * p + 5))
    S = np.sqrt(np.outer(2 * p + 5, 2 * p + 5)) / (p[:, None] + p[None, :] + 5)
    w, V = np.linalg.eigh(S)
    if not np.all(w > 0):
        raise ValueError("RBPolyB overlap matrix is not positive definite")
    M = (V * (1.0 / np.sqrt(w))) @ V.T
    return np.ascontiguousarray(M.reshape(-1, order="F")), norm
CUTOFF_TYPES = {"quadratic": 0, "cosine": 1, "poly5": 2, "normalized_quadratic": 3,
                "cosine_left": 4, "cosine_unscaled": 5, "cosine_squared": 6,
                "sine_squared": 7, "poly3": 8, "poly4": 9, "smoothstep5": 10,
                "smoothstep7": 11}
SHIFT_TYPES = {"linear": 0, "exponential": 1, "exponential_left": 2, "i2": 3,
               "exponential_tanh": 4}


@dataclasses.dataclass
class RadialFamily:
    """One radial basis family with its parameters (mtpb_radial_family)."""
    name: str = "RBChebyshev"
    cutoff_type: str = "quadratic"         # configurable only
    shift_type: str = "linear"             # configurable only
    one_minus_chebyshev: bool = False      # configurable only
    b: float = 0.0                         # rb_b (Poly4/Poly5) or cutoff_b
    r1: float = 0.0                        # cutoff_r1 (smoothstep7)
    r2: float = 0.0                        # cutoff_r2
    shift_lambda: float = 0.0
    shift_scale_lambda: float = 0.0
    # RBPolyB / RBPolyBCos: orthogonalisation matrix (column-major [R*R]) and
    # normalisations [R] (polyb_data, or the reference loader's own)
    poly_matrix: Optional[np.ndarray] = dataclasses.field(default=None, compare=False,
                                                          repr=False)
    poly_norm: Optional[np.ndarray] = dataclasses.field(default=None, compare=False,
                                                        repr=False)

    @property
    def type_id(self) -> int:
        return RADIAL_TYPES[self.name]

    def lines(self) -> List[str]:
        """The family-specific lines written after radial_basis_size."""
        if self.name in ("RBChebyshevPoly4", "RBChebyshevPoly5"):
            return [f"\trb_b = {_fmt(self.b)}"]
        if self.name != "RBChebyshevConfigurable":
            return []
        out = ["\tbasis_function_type = " +
               ("one_minus_chebyshev" if self.one_minus_chebyshev else "chebyshev"),
               f"\tcutoff_type = {self.cutoff_type}"]
        if self.cutoff_type in ("poly3", "poly4", "poly5"):
            out.append(f"\tcutoff_b = {_fmt(self.b)}")
        if self.cutoff_type == "smoothstep7":
            out += [f"\tcutoff_r1 = {_fmt(self.r1)}", f"\tcutoff_r2 = {_fmt(self.r2)}"]
        out.append(f"\tshift_type = {self.shift_type}")
        if self.shift_type in ("exponential", "exponential_left", "exponential_tanh"):
            out.append(f"\tshift_lambda = {_fmt(self.shift_lambda)}")
        if self.shift_type == "exponential_tanh":
            out.append(f"\tshift_scale_lambda = {_fmt(self.shift_scale_lambda)}")
        return out


@dataclasses.dataclass
class MTPModel:
    species_count: int
    radial_func_count: int
    rb_size: int
    min_dist: np.ndarray          # [1] or [K*K]
    max_dist: np.ndarray          # [1] or [K*K]
    alpha_moments_count: int
    alpha_index_basic: np.ndarray  # int32 [nb, 4]
    alpha_index_times: np.ndarray  # int32 [T, 4]
    alpha_moment_mapping: np.ndarray  # int32 [S]
    radial_coeffs: np.ndarray      # float64 [K*K*mu*R]
    species_coeffs: np.ndarray     # float64 [K]
    moment_coeffs: np.ndarray      # float64 [S]
    scaling: float = 0.01
    radial_basis_split: bool = False
    potential_name: str = "MTP1m"
    radial_family: Optional[List[RadialFamily]] = None   # None: RBChebyshev; [1] or [K*K]

    def family(self, pair: int) -> RadialFamily:
        if not self.radial_family:
            return RadialFamily()
        return self.radial_family[pair if len(self.radial_family) > 1 else 0]

    @property
    def alpha_index_basic_count(self) -> int:
        return int(self.alpha_index_basic.shape[0])

    @property
    def alpha_index_times_count(self) -> int:
        return int(self.alpha_index_times.shape[0])

    @property
    def alpha_scalar_moments(self) -> int:
        return int(self.alpha_moment_mapping.shape[0])

    @property
    def cutoff(self) -> float:
        return float(np.max(self.max_dist))

    @property
    def radial_coeffs_count(self) -> int:
        K = self.species_count
        return K * K * self.radial_func_count * self.rb_size

    @property
    def coeff_count(self) -> int:
        return self.radial_coeffs_count + self.species_count + self.alpha_scalar_moments

    def coefficients(self) -> np.ndarray:
        """Native parameter order: radial, species, moment (PotMTP layout)."""
        return np.concatenate([self.radial_coeffs, self.species_coeffs, self.moment_coeffs])

    def with_coefficients(self, coeffs: np.ndarray) -> "MTPModel":
        c = np.asarray(coeffs, dtype=np.float64)
        if c.shape != (self.coeff_count,):
            raise ValueError(f"expected {self.coeff_count} coefficients, got {c.shape}")
        r = self.radial_coeffs_count
        K = self.species_count
        return dataclasses.replace(self, radial_coeffs=c[:r].copy(),
                                   species_coeffs=c[r:r + K].copy(),
                                   moment_coeffs=c[r + K:].copy())

    def pair_min(self, pair: int) -> float:
        return float(self.min_dist[pair] if self.radial_basis_split else self.min_dist[0])

    def pair_max(self, pair: int) -> float:
        return float(self.max_dist[pair] if self.radial_basis_split else self.max_dist[0])

    def basis_shape(self) -> List[int]:
        """Largest angular degree nu = a+b+c used with each radial channel mu
        (-1 where a channel is unused)."""
        out = [-1] * self.radial_func_count
        for mu, a, b, c in self.alpha_index_basic:
            out[mu] = max(out[mu], a + b + c)
        return out


class _Tokens:
    """Whitespace tokenizer that also splits the punctuation {},=."""

    _re = re.compile(r"[{},=]|[^\s{},=]+")

    def __init__(self, text: str):
        self.toks = self._re.findall(text)
        self.i = 0

    def peek(self) -> Optional[str]:
        return self.toks[self.i] if self.i < len(self.toks) else None

    def next(self) -> str:
        if self.i >= len(self.toks):
            raise ValueError("unexpected end of MTP text")
        t = self.toks[self.i]
        self.i += 1
        return t

    def expect(self, tok: str) -> None:
        t = self.next()
        if t != tok:
            raise ValueError(f"expected '{tok}', found '{t}'")

    def assignment(self, key: str) -> str:
        self.expect(key)
        self.expect("=")
        return self.next()

    def flat_array(self) -> List[str]:
        """Reads {v, v, ...} or nested {{..},{..}} and returns the leaf tokens."""
        self.expect("{")
        depth, out = 1, []
        while depth:
            t = self.next()
            if t == "{":
                depth += 1
            elif t == "}":
                depth -= 1
            elif t != ",":
                out.append(t)
        return out


def parse_mtp(text: str) -> MTPModel:
    lines = text.splitlines()
    if len(lines) < 2 or lines[0].strip() != "MTP":
        raise ValueError("expected MTP header")
    if lines[1].strip() != "version = 1.1.0":
        raise ValueError("only MTP version 1.1.0 is supported")
    # potential_name and potential_tag take the rest of their line
    body = []
    name = "MTP1m"
    for ln in lines[2:]:
        s = ln.strip()
        if s.startswith("potential_name"):
            name = s.split("=", 1)[1].strip() if "=" in s else name
            continue
        if s.startswith("potential_tag"):
            continue
        if s.startswith("#MVS_v1.1"):
            break
        body.append(ln)
    tk = _Tokens("\n".join(body))
    scaling = 0.01  # PotMTP::Load default when the field is absent
    if tk.peek() == "scaling":
        scaling = float(tk.assignment("scaling"))
    K = int(tk.assignment("species_count"))
    if K <= 0:
        raise ValueError("species_count must be positive")
    split = False
    if tk.peek() in ("radial_basis_split", "radial_split"):
        key = tk.next()
        tk.expect("=")
        split = int(tk.next()) != 0

    def read_basis():
        btype = tk.assignment("radial_basis_type")
        if btype not in RADIAL_TYPES:
            raise ValueError(f"radial basis '{btype}' is not supported (implemented: "
                             + ", ".join(RADIAL_TYPES) + ")")
        rmin = float(tk.assignment("min_dist"))
        rmax = float(tk.assignment("max_dist"))
        size = int(tk.assignment("radial_basis_size"))
        if size <= 0 or not rmax > rmin:
            raise ValueError("invalid radial basis interval or size")
        fam = RadialFamily(name=btype)
        if btype in POLYB_TYPES:
            fam.poly_matrix, fam.poly_norm = polyb_data(rmin, rmax, size)
        if btype in ("RBChebyshevPoly4", "RBChebyshevPoly5"):
            fam.b = float(tk.assignment("rb_b"))
        elif btype == "RBChebyshevConfigurable":
            if tk.peek() == "basis_function_type":
                kind = tk.assignment("basis_function_type")
                if kind not in ("chebyshev", "one_minus_chebyshev"):
                    raise ValueError(f"unknown basis_function_type '{kind}'")
                fam.one_minus_chebyshev = kind == "one_minus_chebyshev"
            fam.cutoff_type = tk.assignment("cutoff_type")
            if fam.cutoff_type not in CUTOFF_TYPES:
                raise ValueError(f"unknown cutoff_type '{fam.cutoff_type}'")
            if fam.cutoff_type in ("poly3", "poly4", "poly5"):
                fam.b = float(tk.assignment("cutoff_b"))
            if fam.cutoff_type == "smoothstep7":
                fam.r1 = float(tk.assignment("cutoff_r1"))
                fam.r2 = float(tk.assignment("cutoff_r2"))
                if not (rmin < fam.r1 <= fam.r2 < rmax):
                    raise ValueError("smoothstep7 requires min_dist < cutoff_r1 <= cutoff_r2 "
                                     "< max_dist")
            fam.shift_type = tk.assignment("shift_type")
            if fam.shift_type not in SHIFT_TYPES:
                raise ValueError(f"unknown shift_type '{fam.shift_type}'")
            if fam.shift_type in ("exponential", "exponential_left", "exponential_tanh"):
                fam.shift_lambda = float(tk.assignment("shift_lambda"))
            if fam.shift_type == "exponential_tanh":
                fam.shift_scale_lambda = float(tk.assignment("shift_scale_lambda"))
        return rmin, rmax, size, fam

    if split:
        mins = np.zeros(K * K)
        maxs = np.zeros(K * K)
        seen = set()
        R = None
        families = [None] * (K * K)
        for _ in range(K * K):
            tk.expect("pair")
            ci, cj = int(tk.next()), int(tk.next())
            if not (0 <= ci < K and 0 <= cj < K) or (ci, cj) in seen:
                raise ValueError("invalid or duplicate radial basis pair")
            seen.add((ci, cj))
            rmin, rmax, size, fam = read_basis()
            if R is not None and size != R:
                raise ValueError("split radial bases must share radial_basis_size")
            R = size
            mins[ci * K + cj], maxs[ci * K + cj] = rmin, rmax
            families[ci * K + cj] = fam
    else:
        rmin, rmax, R, fam = read_basis()
        mins, maxs = np.array([rmin]), np.array([rmax])
        families = [fam]
    if all(f.name == "RBChebyshev" for f in families):
        families = None
    mu = int(tk.assignment("radial_funcs_count"))
    radial = np.zeros(K * K * mu * R)
    if tk.peek() == "radial_coeffs":
        tk.next()
        for _ in range(K * K):
            pair_tok = tk.next()
            m = re.fullmatch(r"(\d+)-(\d+)", pair_tok)
            if m:
                ti, tj = int(m.group(1)), int(m.group(2))
            else:  # tolerate "i - j" spacing
                ti = int(pair_tok)
                tk.expect("-") if tk.peek() == "-" else None
                tj = int(tk.next())
            if not (0 <= ti < K and 0 <= tj < K):
                raise ValueError("invalid radial coefficient pair")
            for f in range(mu):
                vals = tk.flat_array()
                if len(vals) != R:
                    raise ValueError("radial coefficient row has the wrong length")
                off = (ti * K + tj) * mu * R + f * R
                radial[off:off + R] = [float(v) for v in vals]
    M = int(tk.assignment("alpha_moments_count"))
    nb = int(tk.assignment("alpha_index_basic_count"))
    tk.expect("alpha_index_basic")
    tk.expect("=")
    basic = np.array([int(v) for v in tk.flat_array()], dtype=np.int32).reshape(-1, 4)
    if basic.shape[0] != nb:
        raise ValueError("alpha_index_basic length mismatch")
    T = int(tk.assignment("alpha_index_times_count"))
    tk.expect("alpha_index_times")
    tk.expect("=")
    vals = tk.flat_array()
    times = np.array([int(v) for v in vals], dtype=np.int32).reshape(-1, 4) if T else \
        np.zeros((0, 4), dtype=np.int32)
    if times.shape[0] != T:
        raise ValueError("alpha_index_times length mismatch")
    S = int(tk.assignment("alpha_scalar_moments"))
    tk.expect("alpha_moment_mapping")
    tk.expect("=")
    mapping = np.array([int(v) for v in tk.flat_array()], dtype=np.int32)
    if mapping.shape[0] != S:
        raise ValueError("alpha_moment_mapping length mismatch")
    species = np.zeros(K)
    moment = np.zeros(S)
    while tk.peek() is not None:
        key = tk.next()
        if key == "species_coeffs":
            tk.expect("=")
            v = tk.flat_array()
            if len(v) != K:
                raise ValueError("species_coeffs length mismatch")
            species = np.array([float(x) for x in v])
        elif key == "moment_coeffs":
            tk.expect("=")
            v = tk.flat_array()
            if len(v) != S:
                raise ValueError("moment_coeffs length mismatch")
            moment = np.array([float(x) for x in v])
        elif key.startswith("#"):
            continue
        else:
            break
    model = MTPModel(species_count=K, radial_func_count=mu, rb_size=R, min_dist=mins,
                     max_dist=maxs, alpha_moments_count=M, alpha_index_basic=basic,
                     alpha_index_times=times, alpha_moment_mapping=mapping,
                     radial_coeffs=radial, species_coeffs=species, moment_coeffs=moment,
                     scaling=scaling, radial_basis_split=split, potential_name=name,
                     radial_family=families)
    validate(model)
    return model


def validate(m: MTPModel) -> None:
    """Graph checks of MLIPCore::setup_from_text (runtime/mtp/mlip.cpp:700-735)."""
    nb, M = m.alpha_index_basic_count, m.alpha_moments_count
    if nb <= 0 or nb > M:
        raise ValueError("basic moment count exceeds total moment slots")
    b = m.alpha_index_basic
    if (b[:, 0] < 0).any() or (b[:, 0] >= m.radial_func_count).any() or (b[:, 1:] < 0).any():
        raise ValueError("invalid basic moment index")
    defined = set(range(nb))
    consumed = set()
    for l1, l2, c, t in m.alpha_index_times:
        if (l1 not in defined or l2 not in defined or t < nb or t >= M or t in (l1, l2)
                or t in consumed):
            raise ValueError("moment graph has an undefined input, cycle or late accumulation")
        defined.add(int(t))
        consumed.add(int(l1))
        consumed.add(int(l2))
    for s in m.alpha_moment_mapping:
        if s not in defined:
            raise ValueError("scalar maps to an undefined moment")


def read_mtp(path: str) -> MTPModel:
    with open(path) as f:
        return parse_mtp(f.read())


def _fmt(x: float) -> str:
    return repr(float(x))


def format_mtp(m: MTPModel) -> str:
    K, mu, R = m.species_count, m.radial_func_count, m.rb_size
    out = ["MTP", "version = 1.1.0", f"potential_name = {m.potential_name}",
           f"scaling = {_fmt(m.scaling)}", f"species_count = {K}", "potential_tag = "]
    if m.radial_basis_split:
        out.append("radial_basis_split = 1")
        for i in range(K):
            for j in range(K):
                fam = m.family(i * K + j)
                out += [f"pair {i} {j}", f"radial_basis_type = {fam.name}",
                        f"\tmin_dist = {_fmt(m.min_dist[i * K + j])}",
                        f"\tmax_dist = {_fmt(m.max_dist[i * K + j])}",
                        f"\tradial_basis_size = {R}"] + fam.lines()
        out.append(f"\tradial_funcs_count = {mu}")
    else:
        fam = m.family(0)
        out += [f"radial_basis_type = {fam.name}", f"\tmin_dist = {_fmt(m.min_dist[0])}",
                f"\tmax_dist = {_fmt(m.max_dist[0])}", f"\tradial_basis_size = {R}"]
        out += fam.lines() + [f"\tradial_funcs_count = {mu}"]
    out.append("\tradial_coeffs")
    for i in range(K):
        for j in range(K):
            out.append(f"\t\t{i}-{j}")
            for f in range(mu):
                off = (i * K + j) * mu * R + f * R
                out.append("\t\t\t{" + ", ".join(_fmt(v) for v in m.radial_coeffs[off:off + R]) + "}")
    out.append(f"alpha_moments_count = {m.alpha_moments_count}")
    out.append(f"alpha_index_basic_count = {m.alpha_index_basic_count}")
    out.append("alpha_index_basic = {" + ", ".join(
        "{" + ", ".join(str(int(v)) for v in row) + "}" for row in m.alpha_index_basic) + "}")
    out.append(f"alpha_index_times_count = {m.alpha_index_times_count}")
    out.append("alpha_index_times = {" + ", ".join(
        "{" + ", ".join(str(int(v)) for v in row) + "}" for row in m.alpha_index_times) + "}")
    out.append(f"alpha_scalar_moments = {m.alpha_scalar_moments}")
    out.append("alpha_moment_mapping = {" + ", ".join(str(int(v)) for v in m.alpha_moment_mapping) + "}")
    out.append("species_coeffs = {" + ", ".join(_fmt(v) for v in m.species_coeffs) + "}")
    out.append("moment_coeffs = {" + ", ".join(_fmt(v) for v in m.moment_coeffs) + "}")
    return "\n".join(out) + "\n"


def write_mtp(m: MTPModel, path: str) -> None:
    with open(path, "w") as f:
        f.write(format_mtp(m))
