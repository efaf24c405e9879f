"""ctypes front end of the CPU parity checker.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py.  The product library never imports it.

* :class:`Oracle` wraps ``liboracle.so``, the plain-C restatement of the
  reference hot path (mtp_oracle.c, which cites the reference lines it
  follows).
* :class:`Reference` wraps ``_ref/libref.so``, the reference's own
  ``Neighborhoods`` builder and ``MLIPCore::compute`` compiled from the
  reference sources (ref_shim.cpp); it exists only where that build ran.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_dp = C.POINTER(C.c_double)
_ip = C.POINTER(C.c_int)


def _d(a):
    return a.ctypes.data_as(_dp) if a is not None else None


def _i(a):
    return a.ctypes.data_as(_ip) if a is not None else None


class OracleRadialFamily(C.Structure):
    """oracle_radial_family (same layout as mtpb_radial_family)."""
    _fields_ = [("type", C.c_int), ("cutoff_type", C.c_int), ("shift_type", C.c_int),
                ("one_minus_chebyshev", C.c_int), ("b", C.c_double), ("r1", C.c_double),
                ("r2", C.c_double), ("shift_lambda", C.c_double),
                ("shift_scale_lambda", C.c_double), ("poly_matrix", _dp), ("poly_norm", _dp)]


_RB_TYPES = {"RBChebyshev": 0, "RBChebyCos": 1, "RBChebyshevPoly5": 2,
             "RBChebyshevConfigurable": 3, "RBChebyshevPoly4": 4, "RBPolyB": 5,
             "RBPolyBCos": 6}
_CUTOFFS = {"quadratic": 0, "cosine": 1, "poly5": 2, "normalized_quadratic": 3,
            "cosine_left": 4, "cosine_unscaled": 5, "cosine_squared": 6, "sine_squared": 7,
            "poly3": 8, "poly4": 9, "smoothstep5": 10, "smoothstep7": 11}
_SHIFTS = {"linear": 0, "exponential": 1, "exponential_left": 2, "i2": 3,
           "exponential_tanh": 4}


class OracleModel(C.Structure):
    _fields_ = [
        ("species_count", C.c_int), ("radial_func_count", C.c_int), ("rb_size", C.c_int),
        ("radial_basis_split", C.c_int), ("min_dist", _dp), ("max_dist", _dp),
        ("scaling", C.c_double), ("alpha_moments_count", C.c_int),
        ("alpha_index_basic_count", C.c_int), ("alpha_index_times_count", C.c_int),
        ("alpha_scalar_moments", C.c_int), ("alpha_index_basic", _ip),
        ("alpha_index_times", _ip), ("alpha_moment_mapping", _ip), ("radial_coeffs", _dp),
        ("species_coeffs", _dp), ("moment_coeffs", _dp),
        ("radial_family", C.POINTER(OracleRadialFamily)),
    ]


class LossWeights(C.Structure):
    _fields_ = [("weight_eng", C.c_double), ("weight_force", C.c_double),
                ("weight_stress", C.c_double), ("weight_eng_power", C.c_double),
                ("weight_force_power", C.c_double), ("weight_stress_power", C.c_double)]


def model_struct(model):
    """Builds an OracleModel from an MTPModel; returns (struct, keepalive)."""
    keep = dict(
        mins=np.ascontiguousarray(model.min_dist, dtype=np.float64),
        maxs=np.ascontiguousarray(model.max_dist, dtype=np.float64),
        basic=np.ascontiguousarray(model.alpha_index_basic, dtype=np.int32),
        times=np.ascontiguousarray(model.alpha_index_times, dtype=np.int32).reshape(-1, 4),
        mapping=np.ascontiguousarray(model.alpha_moment_mapping, dtype=np.int32),
        radial=np.ascontiguousarray(model.radial_coeffs, dtype=np.float64),
        species=np.ascontiguousarray(model.species_coeffs, dtype=np.float64),
        moment=np.ascontiguousarray(model.moment_coeffs, dtype=np.float64),
    )
    fams = getattr(model, "radial_family", None)
    fam_ptr = None
    if fams:
        arr = (OracleRadialFamily * len(fams))()
        poly = []
        for i, f in enumerate(fams):
            pm = pn = None
            if getattr(f, "poly_matrix", None) is not None:
                poly += [np.ascontiguousarray(f.poly_matrix, dtype=np.float64),
                         np.ascontiguousarray(f.poly_norm, dtype=np.float64)]
                pm, pn = _d(poly[-2]), _d(poly[-1])
            arr[i] = OracleRadialFamily(_RB_TYPES[f.name], _CUTOFFS[f.cutoff_type],
                                        _SHIFTS[f.shift_type], int(f.one_minus_chebyshev),
                                        f.b, f.r1, f.r2, f.shift_lambda, f.shift_scale_lambda,
                                        pm, pn)
        keep["families"] = arr
        keep["poly"] = poly
        fam_ptr = C.cast(arr, C.POINTER(OracleRadialFamily))
    s = OracleModel(model.species_count, model.radial_func_count, model.rb_size,
                    int(model.radial_basis_split), _d(keep["mins"]), _d(keep["maxs"]),
                    float(model.scaling), model.alpha_moments_count,
                    model.alpha_index_basic_count, model.alpha_index_times_count,
                    model.alpha_scalar_moments, _i(keep["basic"]), _i(keep["times"]),
                    _i(keep["mapping"]), _d(keep["radial"]), _d(keep["species"]),
                    _d(keep["moment"]), fam_ptr)
    return s, keep


class NeighborList:
    """CSR neighbour list: offsets[n+1], nbr[E], rij[E,3]."""

    def __init__(self, offsets, nbr, rij):
        self.offsets = offsets
        self.nbr = nbr
        self.rij = rij

    @property
    def n_edges(self) -> int:
        return int(self.offsets[-1])

    def canonical(self):
        """Per-atom lists sorted by (neighbour, rx, ry, rz)."""
        off, nbr, rij = self.offsets, self.nbr, self.rij
        order = np.empty(len(nbr), dtype=np.int64)
        for i in range(len(off) - 1):
            a, b = off[i], off[i + 1]
            keys = (rij[a:b, 2], rij[a:b, 1], rij[a:b, 0], nbr[a:b])
            order[a:b] = a + np.lexsort(keys)
        return NeighborList(off.copy(), nbr[order], rij[order])


def concat_lists(lists, atom_offsets):
    """Concatenates per-structure lists into one list over global atom ids."""
    offs = [np.zeros(1, dtype=np.int32)]
    nbrs, rijs = [], []
    base_e = 0
    for s, nl in enumerate(lists):
        offs.append(nl.offsets[1:].astype(np.int64) + base_e)
        nbrs.append(nl.nbr + atom_offsets[s])
        rijs.append(nl.rij)
        base_e += nl.n_edges
    return NeighborList(np.concatenate(offs).astype(np.int32),
                        np.concatenate(nbrs).astype(np.int32) if nbrs else np.zeros(0, np.int32),
                        np.concatenate(rijs) if rijs else np.zeros((0, 3)))


class Oracle:
    def __init__(self, path: Optional[str] = None):
        path = path or os.path.join(HERE, "liboracle.so")
        self.lib = L = C.CDLL(path)
        L.oracle_neighbors.restype = C.c_long
        L.oracle_neighbors.argtypes = [_dp, _ip, C.c_int, _dp, C.c_double, _ip, _ip, _dp]
        L.oracle_wrap_positions.argtypes = [_dp, _ip, C.c_int, _dp, _dp]
        L.oracle_efs.argtypes = [C.POINTER(OracleModel), C.c_int, _ip, _ip, _ip, _dp, _dp, _dp,
                                 _dp, _dp]
        L.oracle_site_derivatives.argtypes = [C.POINTER(OracleModel), C.c_int, _ip, _ip, _ip,
                                              _dp, _dp, _dp]
        L.oracle_site_moments.argtypes = [C.POINTER(OracleModel), C.c_int, _ip, _ip, _ip, _dp,
                                          _dp, _dp]
        L.oracle_loss_grad.argtypes = [C.POINTER(OracleModel), C.POINTER(LossWeights), C.c_int,
                                       _ip, _ip, _ip, _ip, _dp, _dp, _dp, _dp, _ip, _ip, _ip,
                                       _dp, _dp, _dp]
        L.oracle_efs_batch.argtypes = [C.POINTER(OracleModel), C.c_int, _ip, _ip, _ip, _ip, _dp,
                                       _dp, _dp, _dp, C.c_int]

    def neighbors(self, cell, pbc, positions, cutoff) -> NeighborList:
        cell = np.ascontiguousarray(cell, dtype=np.float64).reshape(9)
        pbc = np.ascontiguousarray(pbc, dtype=np.int32)
        pos = np.ascontiguousarray(positions, dtype=np.float64)
        n = pos.shape[0]
        E = self.lib.oracle_neighbors(_d(cell), _i(pbc), n, _d(pos), cutoff, None, None, None)
        if E < 0:
            raise RuntimeError("oracle_neighbors failed")
        off = np.zeros(n + 1, dtype=np.int32)
        nbr = np.zeros(E, dtype=np.int32)
        rij = np.zeros((E, 3))
        self.lib.oracle_neighbors(_d(cell), _i(pbc), n, _d(pos), cutoff, _i(off), _i(nbr), _d(rij))
        return NeighborList(off, nbr, rij)

    def wrap(self, cell, pbc, positions):
        cell = np.ascontiguousarray(cell, dtype=np.float64).reshape(9)
        pbc = np.ascontiguousarray(pbc, dtype=np.int32)
        pos = np.ascontiguousarray(positions, dtype=np.float64)
        out = np.empty_like(pos)
        self.lib.oracle_wrap_positions(_d(cell), _i(pbc), pos.shape[0], _d(pos), _d(out))
        return out

    def efs(self, model, types, nl: NeighborList):
        ms, keep = model_struct(model)
        types = np.ascontiguousarray(types, dtype=np.int32)
        n = types.shape[0]
        e = np.zeros(1)
        se = np.zeros(n)
        f = np.zeros((n, 3))
        s = np.zeros(9)
        rc = self.lib.oracle_efs(C.byref(ms), n, _i(types), _i(nl.offsets), _i(nl.nbr),
                                 _d(np.ascontiguousarray(nl.rij)), _d(e), _d(se), _d(f), _d(s))
        if rc:
            raise RuntimeError("oracle_efs failed")
        return float(e[0]), se, f, s.reshape(3, 3)

    def site_derivatives(self, model, types, nl: NeighborList):
        ms, keep = model_struct(model)
        types = np.ascontiguousarray(types, dtype=np.int32)
        n = types.shape[0]
        se = np.zeros(n)
        d = np.zeros((nl.n_edges, 3))
        rc = self.lib.oracle_site_derivatives(C.byref(ms), n, _i(types), _i(nl.offsets),
                                              _i(nl.nbr), _d(np.ascontiguousarray(nl.rij)),
                                              _d(se), _d(d))
        if rc:
            raise RuntimeError("oracle_site_derivatives failed")
        return se, d

    def site_moments(self, model, types, nl: NeighborList):
        ms, keep = model_struct(model)
        types = np.ascontiguousarray(types, dtype=np.int32)
        n = types.shape[0]
        nb = model.alpha_index_basic_count
        b = np.zeros((n, nb))
        a = np.zeros((n, nb))
        rc = self.lib.oracle_site_moments(C.byref(ms), n, _i(types), _i(nl.offsets), _i(nl.nbr),
                                          _d(np.ascontiguousarray(nl.rij)), _d(b), _d(a))
        if rc:
            raise RuntimeError("oracle_site_moments failed")
        return b, a

    def efs_batch(self, model, atom_offsets, types, nl: NeighborList, threads: int = 0):
        ms, keep = model_struct(model)
        S = len(atom_offsets) - 1
        N = int(atom_offsets[-1])
        e = np.zeros(S)
        f = np.zeros((N, 3))
        s = np.zeros((S, 9))
        rc = self.lib.oracle_efs_batch(C.byref(ms), S, _i(np.ascontiguousarray(atom_offsets, dtype=np.int32)),
                                       _i(np.ascontiguousarray(types, dtype=np.int32)),
                                       _i(nl.offsets), _i(nl.nbr), _d(np.ascontiguousarray(nl.rij)),
                                       _d(e), _d(f), _d(s), threads)
        if rc:
            raise RuntimeError("oracle_efs_batch failed")
        return e, f, s.reshape(S, 3, 3)

    def loss_grad(self, model, atom_offsets, types, nl: NeighborList, target_energy,
                  target_forces, target_stress, weights=(1.0, 0.01, 0.0001, 1.0, 0.0, 1.0)):
        ms, keep = model_struct(model)
        w = LossWeights(*weights)
        S = len(atom_offsets) - 1
        loss = np.zeros(1)
        metrics = np.zeros(7)
        grad = np.zeros(model.coeff_count)
        te = None if target_energy is None else np.ascontiguousarray(target_energy, dtype=np.float64)
        tf = None if target_forces is None else np.ascontiguousarray(target_forces, dtype=np.float64)
        ts = None if target_stress is None else np.ascontiguousarray(target_stress, dtype=np.float64)
        rc = self.lib.oracle_loss_grad(C.byref(ms), C.byref(w), S,
                                       _i(np.ascontiguousarray(atom_offsets, dtype=np.int32)),
                                       _i(np.ascontiguousarray(types, dtype=np.int32)),
                                       _i(nl.offsets), _i(nl.nbr), _d(np.ascontiguousarray(nl.rij)),
                                       _d(te), _d(tf), _d(ts), None, None, None, _d(loss),
                                       _d(metrics), _d(grad))
        if rc:
            raise RuntimeError("oracle_loss_grad failed")
        return float(loss[0]), metrics, grad


class Reference:
    """The reference's own CPU code compiled from its sources (oracle/_ref)."""

    def __init__(self, path: Optional[str] = None):
        path = path or os.path.join(HERE, "_ref", "libref.so")
        self.lib = L = C.CDLL(path)
        L.ref_last_error.restype = C.c_char_p
        L.ref_neighbors.restype = C.c_long
        L.ref_neighbors.argtypes = [_dp, _ip, C.c_int, _dp, C.c_double, _ip, _ip, _dp]
        L.ref_mlip_setup.restype = C.c_void_p
        L.ref_mlip_setup.argtypes = [C.c_char_p, _ip, C.c_int, _dp]
        L.ref_mlip_destroy.argtypes = [C.c_void_p]
        L.ref_mlip_compute.argtypes = [C.c_void_p, C.c_int, _ip, C.c_int, _ip, _dp, _ip, _ip, _ip,
                                       _dp, _dp, _dp, _dp]
        L.ref_mlip_compute_omp.argtypes = [C.c_void_p, C.c_int, C.c_int, _ip, C.c_int, _ip, _dp,
                                           _ip, _ip, _ip, _dp, _dp]
        L.ref_mlip_polyb.argtypes = [C.c_void_p, C.c_int, _dp, _dp]
        L.ref_read_model_text.restype = C.c_long
        L.ref_read_model_text.argtypes = [C.c_char_p, C.c_char_p, C.c_long]
        L.ref_mlip_efs_omp.argtypes = [C.c_void_p, C.c_int, C.c_int, _ip, C.c_int, _ip, _dp,
                                       _ip, _ip, _ip, _dp, _dp, _dp, _dp]

    @staticmethod
    def available(path: Optional[str] = None) -> bool:
        return os.path.exists(path or os.path.join(HERE, "_ref", "libref.so"))

    def _err(self):
        return self.lib.ref_last_error().decode()

    def neighbors(self, cell, pbc, positions, cutoff) -> NeighborList:
        cell = np.ascontiguousarray(cell, dtype=np.float64).reshape(9)
        pbc = np.ascontiguousarray(pbc, dtype=np.int32)
        pos = np.ascontiguousarray(positions, dtype=np.float64)
        n = pos.shape[0]
        E = self.lib.ref_neighbors(_d(cell), _i(pbc), n, _d(pos), cutoff, None, None, None)
        if E < 0:
            raise RuntimeError(self._err())
        off = np.zeros(n + 1, dtype=np.int32)
        nbr = np.zeros(E, dtype=np.int32)
        rij = np.zeros((E, 3))
        self.lib.ref_neighbors(_d(cell), _i(pbc), n, _d(pos), cutoff, _i(off), _i(nbr), _d(rij))
        return NeighborList(off, nbr, rij)

    def model_text(self, path: str) -> str:
        """The .mtp text MLIPCore's loader reads from a model file (GPM bundles
        included)."""
        n = self.lib.ref_read_model_text(path.encode(), None, 0)
        if n < 0:
            raise RuntimeError(self._err())
        buf = C.create_string_buffer(n + 1)
        self.lib.ref_read_model_text(path.encode(), buf, n + 1)
        return buf.value.decode()

    def polyb(self, mtp_text: str, species: int):
        """Per ordered species pair, the RBPolyB orthogonalisation matrix
        (column-major, flattened) and normalisations that MLIPCore's loader
        computed for this model text (runtime/mtp/radial_basis_setup.cpp), or
        None for pairs of other families."""
        tmap = np.arange(species, dtype=np.int32)
        cut = np.zeros(1)
        h = self.lib.ref_mlip_setup(mtp_text.encode(), _i(tmap), species, _d(cut))
        if not h:
            raise RuntimeError(self._err())
        try:
            out = []
            for p in range(species * species):
                n = self.lib.ref_mlip_polyb(h, p, None, None)
                if n <= 0:
                    out.append(None)
                    continue
                M = np.zeros(n * n)
                N = np.zeros(n)
                self.lib.ref_mlip_polyb(h, p, _d(M), _d(N))
                out.append((M, N))
            return out
        finally:
            self.lib.ref_mlip_destroy(h)

    def mlip_efs(self, mtp_text: str, types, nl: NeighborList, positions):
        """MLIPCore::compute on explicit ghost atoms: every edge gets a ghost
        at x_i + r_ij, so the core sees exactly the neighbour list."""
        types = np.ascontiguousarray(types, dtype=np.int32)
        n = types.shape[0]
        K = int(types.max()) + 1 if n else 1
        tmap = np.arange(max(K, 1), dtype=np.int32)
        cut = np.zeros(1)
        h = self.lib.ref_mlip_setup(mtp_text.encode(), _i(tmap), len(tmap), _d(cut))
        if not h:
            raise RuntimeError(self._err())
        try:
            E = nl.n_edges
            pos = np.ascontiguousarray(positions, dtype=np.float64)
            centers = np.repeat(np.arange(n), np.diff(nl.offsets))
            ghosts = pos[centers] + nl.rij
            x = np.concatenate([pos, ghosts]).astype(np.float64)
            ntot = n + E
            ty = np.concatenate([types, types[nl.nbr]]).astype(np.int32)
            numneigh = np.zeros(ntot, dtype=np.int32)
            numneigh[:n] = np.diff(nl.offsets)
            flat = (n + np.arange(E)).astype(np.int32)
            foff = np.zeros(ntot, dtype=np.int32)
            foff[:n] = nl.offsets[:-1]
            ilist = np.arange(n, dtype=np.int32)
            en = np.zeros(1)
            se = np.zeros(ntot)
            f = np.zeros((ntot, 3))
            vir = np.zeros((ntot, 6))
            rc = self.lib.ref_mlip_compute(h, n, _i(ilist), ntot, _i(ty), _d(x), _i(numneigh),
                                           _i(foff), _i(flat), _d(en), _d(se), _d(f), _d(vir))
            if rc:
                raise RuntimeError(self._err())
            # fold ghost forces back onto their owners
            forces = f[:n].copy()
            np.add.at(forces, nl.nbr, f[n:])
            return float(en[0]), se[:n], forces, vir
        finally:
            self.lib.ref_mlip_destroy(h)


class ReferenceEFS:
    """The reference CPU path for one periodic structure, as the benchmark's
    CPU arm runs it: Neighborhoods (compiled reference) builds the lists, the
    images become explicit ghost atoms, and MLIPCore::compute evaluates the
    centres with OpenMP (ref_mlip_compute_omp)."""

    def __init__(self, mtp_text: str, species: int, threads: int = 0):
        self.ref = Reference()
        L = self.ref.lib
        tmap = np.arange(species, dtype=np.int32)
        self._tmap = tmap
        cut = np.zeros(1)
        self.handle = L.ref_mlip_setup(mtp_text.encode(), _i(tmap), len(tmap), _d(cut))
        if not self.handle:
            raise RuntimeError(self.ref._err())
        self.cutoff = float(cut[0])
        self.threads = threads

    def close(self):
        if self.handle:
            self.ref.lib.ref_mlip_destroy(self.handle)
            self.handle = None

    def build(self, cell, pbc, positions, types):
        """Reference neighbour build; returns the ghost-atom problem."""
        nl = self.ref.neighbors(cell, pbc, positions, self.cutoff)
        n = len(types)
        E = nl.n_edges
        from_oracle = Oracle()
        x0 = from_oracle.wrap(cell, pbc, positions)
        centers = np.repeat(np.arange(n), np.diff(nl.offsets))
        x = np.ascontiguousarray(np.concatenate([x0, x0[centers] + nl.rij]))
        ty = np.ascontiguousarray(np.concatenate([types, np.asarray(types)[nl.nbr]]).astype(np.int32))
        ntot = n + E
        numneigh = np.zeros(ntot, dtype=np.int32)
        numneigh[:n] = np.diff(nl.offsets)
        foff = np.zeros(ntot, dtype=np.int32)
        foff[:n] = nl.offsets[:-1]
        flat = (n + np.arange(E)).astype(np.int32)
        return dict(n=n, nl=nl, x=x, types=ty, numneigh=numneigh, foff=foff, flat=flat)

    def compute(self, prob):
        n = prob["n"]
        ntot = len(prob["types"])
        f = np.zeros((ntot, 3))
        en = np.zeros(1)
        ilist = np.arange(n, dtype=np.int32)
        rc = self.ref.lib.ref_mlip_compute_omp(self.handle, self.threads, n, _i(ilist), ntot,
                                               _i(prob["types"]), _d(prob["x"]),
                                               _i(prob["numneigh"]), _i(prob["foff"]),
                                               _i(prob["flat"]), _d(en), _d(f))
        if rc:
            raise RuntimeError(self.ref._err())
        forces = f[:n].copy()
        np.add.at(forces, prob["nl"].nbr, f[n:])
        return float(en[0]), forces

    def compute_full(self, prob):
        """Energy, site energies[n], forces[n,3] (ghost rows folded onto their
        owners) and the virial [xx yy zz xy xz yz] as the sum of MLIPCore's
        per-atom virials over centres and ghosts."""
        n = prob["n"]
        ntot = len(prob["types"])
        f = np.zeros((ntot, 3))
        se = np.zeros(ntot)
        sv = np.zeros((ntot, 6))
        en = np.zeros(1)
        ilist = np.arange(n, dtype=np.int32)
        rc = self.ref.lib.ref_mlip_efs_omp(self.handle, self.threads, n, _i(ilist), ntot,
                                           _i(prob["types"]), _d(prob["x"]),
                                           _i(prob["numneigh"]), _i(prob["foff"]),
                                           _i(prob["flat"]), _d(en), _d(f), _d(se), _d(sv))
        if rc:
            raise RuntimeError(self.ref._err())
        forces = f[:n].copy()
        np.add.at(forces, prob["nl"].nbr, f[n:])
        return float(en[0]), se[:n], forces, sv.sum(axis=0)


class ReferenceGpu:
    """The reference's own GPU trainer core (MTPGpuDirect compute_batch ->
    prepare_loss -> accumulate_gradient, deterministic FP64 reductions),
    compiled from the reference sources into ``_ref/librefgpu.so`` by
    ``oracle/Makefile`` (target ``refgpu``, ref_gpu_shim.cpp).  Test
    infrastructure: the gradient pin of the GPU tests."""

    def __init__(self, mtp_text: str, species: int, device: int = 0,
                 path: Optional[str] = None):
        self.lib = C.CDLL(path or os.path.join(HERE, "_ref", "librefgpu.so"))
        L = self.lib
        L.refgpu_last_error.restype = C.c_char_p
        L.refgpu_create.restype = C.c_void_p
        L.refgpu_create.argtypes = [C.c_char_p, C.c_int, C.c_int, _ip]
        L.refgpu_destroy.argtypes = [C.c_void_p]
        L.refgpu_loss_grad.argtypes = [C.c_void_p, C.c_int, _ip, _ip, _ip, _dp, _ip, _dp,
                                       _dp, _dp, _dp, _dp, _dp, _dp, _dp, _dp, _dp, _dp, _dp]
        n = C.c_int()
        self.handle = L.refgpu_create(mtp_text.encode(), species, device, C.byref(n))
        if not self.handle:
            raise RuntimeError(L.refgpu_last_error().decode())
        self.gradient_count = n.value

    @staticmethod
    def available(path: Optional[str] = None) -> bool:
        return os.path.exists(path or os.path.join(HERE, "_ref", "librefgpu.so"))

    def close(self):
        if self.handle:
            self.lib.refgpu_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def loss_grad(self, atom_offsets, nl: NeighborList, types, positions, target_energy,
                  energy_weight, target_force, force_weight, target_stress, stress_weight):
        """Metrics[7], un-normalised gradient, and the forward forces, site
        energies and site virials (xx yy zz xy xz yz) of one batch."""
        offs = np.ascontiguousarray(atom_offsets, dtype=np.int32)
        S = len(offs) - 1
        n = int(offs[-1])
        metrics = np.zeros(7)
        grad = np.zeros(self.gradient_count)
        f = np.zeros((n, 3))
        se = np.zeros(n)
        sv = np.zeros((n, 6))
        c = lambda a, t=np.float64: np.ascontiguousarray(a, dtype=t)   # noqa: E731
        args = [c(nl.offsets, np.int32), c(nl.nbr, np.int32), c(nl.rij), c(types, np.int32),
                c(positions), c(target_energy), c(energy_weight), c(target_force),
                c(force_weight), c(target_stress), c(stress_weight)]
        rc = self.lib.refgpu_loss_grad(
            self.handle, S, _i(offs), _i(args[0]), _i(args[1]), _d(args[2]), _i(args[3]),
            _d(args[4]), _d(args[5]), _d(args[6]), _d(args[7]), _d(args[8]), _d(args[9]),
            _d(args[10]), _d(metrics), _d(grad), _d(f), _d(se), _d(sv))
        if rc:
            raise RuntimeError(self.lib.refgpu_last_error().decode())
        return metrics, grad, f, se, sv


class ReferenceBinding:
    """The reference-side binding (MTPB200Direct, imr-mlp_b200/bindings/
    mtpb_direct.hpp) compiled against the reference headers with its
    mlip.cpp into ``_ref/librefdirect.so`` (ref_direct_shim.cpp).  Test
    infrastructure: checks that a maintainer's drop-in of the binding
    reproduces MLIPCore::compute."""

    def __init__(self, mtp_text: str, species: int, device: int = 0,
                 path: Optional[str] = None):
        self.lib = L = C.CDLL(path or os.path.join(HERE, "_ref", "librefdirect.so"))
        L.refdirect_last_error.restype = C.c_char_p
        L.refdirect_create.restype = C.c_void_p
        L.refdirect_create.argtypes = [C.c_char_p, C.c_int, C.c_int]
        L.refdirect_destroy.argtypes = [C.c_void_p]
        L.refdirect_compute_batch.argtypes = [C.c_void_p, C.c_int, C.c_int, _ip, _ip, _dp, _ip,
                                              _dp, _dp, _dp, _dp, _dp, _dp]
        L.refdirect_compute_lammps.argtypes = [C.c_void_p, C.c_int, _ip, C.c_int, _ip, _dp, _ip,
                                               _ip, _ip, C.c_int, _dp, _dp, _dp, _dp, _dp]
        self.handle = L.refdirect_create(mtp_text.encode(), species, device)
        if not self.handle:
            raise RuntimeError(L.refdirect_last_error().decode())

    @staticmethod
    def available(path: Optional[str] = None) -> bool:
        return os.path.exists(path or os.path.join(HERE, "_ref", "librefdirect.so"))

    def close(self):
        if self.handle:
            self.lib.refdirect_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def compute_batch(self, center_count, offsets, neighbors, types, x, vectors=None):
        nt = len(types)
        f = np.zeros((nt, 3))
        e = np.zeros(1)
        se = np.zeros(max(center_count, 1))
        sv = np.zeros((nt, 6))
        gv = np.zeros(6)
        c = lambda a, t=np.float64: np.ascontiguousarray(a, dtype=t)   # noqa: E731
        off, nbr, ty, xx = c(offsets, np.int32), c(neighbors, np.int32), c(types, np.int32), c(x)
        vec = None if vectors is None else c(vectors)
        rc = self.lib.refdirect_compute_batch(self.handle, center_count, nt, _i(off), _i(nbr),
                                              _d(vec), _i(ty), _d(xx), _d(f), _d(e), _d(se),
                                              _d(sv), _d(gv))
        if rc:
            raise RuntimeError(self.lib.refdirect_last_error().decode())
        return dict(energy=float(e[0]), force=f, site_energy=se[:center_count], site_virial=sv,
                    virial=gv)

    def compute_lammps(self, ilist, types, x, numneigh, first_off, flat, mask, force,
                       site_virial):
        """Adds forces into `force` (and per-atom virials into site_virial)."""
        nt = len(types)
        e = np.zeros(1)
        se = np.zeros(nt)
        gv = np.zeros(6)
        c = lambda a, t=np.int32: np.ascontiguousarray(a, dtype=t)   # noqa: E731
        xx = np.ascontiguousarray(x, dtype=np.float64)
        rc = self.lib.refdirect_compute_lammps(self.handle, len(ilist), _i(c(ilist)), nt,
                                               _i(c(types)), _d(xx), _i(c(numneigh)),
                                               _i(c(first_off)), _i(c(flat)), mask, _d(e), _d(se),
                                               _d(force), _d(site_virial), _d(gv))
        if rc:
            raise RuntimeError(self.lib.refdirect_last_error().decode())
        return float(e[0]), se, gv
