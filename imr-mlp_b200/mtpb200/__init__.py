"""mtpb200 -- Python front end of the B200 MTP energy/force/stress and
coefficient-gradient path.

The numerical work runs in ``libmtpb200.so`` (CUDA, sm_100a); this module only
marshals arrays through the C ABI declared in ``include/mtpb200.h``.  Names
follow the reference interfaces the ABI replaces:

* :class:`MTPGpuDirect` -- ``MLIPCore::GpuDirect::MTPGpuDirect``
  (runtime/mtp/gpu-direct/mtp_gpu_direct.h:789-926): one context per device,
  ``update_coefficients``, ``compute_batch`` (CSR lists), ``compute_lammps``;
* :class:`PotMTP` -- the ``getEFS`` / ``CalcEFS`` surface of
  ``Potentials::PotMTP`` (potentials/potential_mtp.cpp:1892-1933), with the
  neighbour lists built on the GPU;
* :meth:`MTPGpuDirect.loss_grad` -- ``Trainer_MTP::AccumulateGard``'s loss and
  gradient evaluator (train/train_mtp.cpp:3039-3094).
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import _lib
from .gpm import read_gpm, write_gpm
from .mtpfile import MTPModel, format_mtp, parse_mtp, read_mtp, write_mtp

__all__ = ["MTPGpuDirect", "PotMTP", "MTPBError", "MTPModel", "read_mtp", "parse_mtp",
           "read_gpm", "write_gpm",
           "write_mtp", "format_mtp", "device_count", "library"]

_LIB: Optional[C.CDLL] = None


def library() -> C.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = _lib.load()
    return _LIB


class MTPBError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"mtpb status {status}: {message}")
        self.status = status


def _check(rc: int) -> None:
    if rc != _lib.MTPB_OK:
        raise MTPBError(rc, library().mtpb_last_error().decode())


def _dp(a):
    return None if a is None else a.ctypes.data_as(_lib._dp)


def _ip(a):
    return None if a is None else a.ctypes.data_as(_lib._ip)


def _tdp(t):
    """Device pointer of a torch CUDA tensor (float64)."""
    return None if t is None else C.cast(C.c_void_p(t.data_ptr()), _lib._dp)


def _tip(t):
    return None if t is None else C.cast(C.c_void_p(t.data_ptr()), _lib._ip)


def device_count() -> int:
    n = C.c_int(0)
    rc = library().mtpb_device_count(C.byref(n))
    return n.value if rc == 0 else 0


def _f64(a):
    return np.ascontiguousarray(a, dtype=np.float64)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


class _ModelKeep:
    def __init__(self, m: MTPModel):
        self.mins = _f64(m.min_dist)
        self.maxs = _f64(m.max_dist)
        self.basic = _i32(m.alpha_index_basic)
        self.times = _i32(m.alpha_index_times).reshape(-1, 4)
        self.mapping = _i32(m.alpha_moment_mapping)
        self.radial = _f64(m.radial_coeffs)
        self.species = _f64(m.species_coeffs)
        self.moment = _f64(m.moment_coeffs)
        self.families, self.family_arrays = _lib.radial_family_array(m)
        self.view = _lib.ModelView(
            m.species_count, m.radial_func_count, m.rb_size, int(m.radial_basis_split),
            _dp(self.mins), _dp(self.maxs), float(m.scaling), m.alpha_moments_count,
            m.alpha_index_basic_count, m.alpha_index_times_count, m.alpha_scalar_moments,
            _ip(self.basic), _ip(self.times), _ip(self.mapping), _dp(self.radial),
            _dp(self.species), _dp(self.moment),
            C.cast(self.families, C.POINTER(_lib.RadialFamilyView)) if self.families else None)


class StructureBatch:
    """Host arrays of a structure batch (see configs.batch)."""

    def __init__(self, atom_offsets, cells, pbc, positions, types):
        self.atom_offsets = _i32(atom_offsets)
        self.cells = _f64(cells).reshape(-1, 9)
        self.pbc = None if pbc is None else _i32(pbc).reshape(-1, 3)
        self.positions = _f64(positions).reshape(-1, 3)
        self.types = _i32(types)

    @classmethod
    def from_structures(cls, structures: Sequence[Dict[str, np.ndarray]]):
        from .configs import batch
        return cls(*batch(list(structures)))

    @property
    def n_structures(self) -> int:
        return len(self.atom_offsets) - 1

    @property
    def n_atoms(self) -> int:
        return int(self.atom_offsets[-1])

    def c_struct(self):
        return _lib.Structures(self.n_structures, _ip(self.atom_offsets), _dp(self.cells),
                               _ip(self.pbc), _dp(self.positions), _ip(self.types))


class MTPGpuDirect:
    """One device context (MTPGpuDirect::set_device + initialize)."""

    def __init__(self, model: MTPModel, device: int = 0):
        self.lib = library()
        self.model = model
        self._keep = _ModelKeep(model)
        h = C.c_void_p()
        _check(self.lib.mtpb_create(int(device), C.byref(self._keep.view), C.byref(h)))
        self.ctx = h
        self._batch: Optional[StructureBatch] = None

    def close(self):
        if getattr(self, "ctx", None):
            self.lib.mtpb_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- model ---------------------------------------------------------
    def update_coefficients(self, radial, species, moment):
        r, s, m = _f64(radial), _f64(species), _f64(moment)
        _check(self.lib.mtpb_update_coefficients(self.ctx, _dp(r), _dp(s), _dp(m)))
        self.model = self.model.with_coefficients(np.concatenate([r, s, m]))

    def set_coefficients(self, coeffs):
        m = self.model.with_coefficients(coeffs)
        self.update_coefficients(m.radial_coeffs, m.species_coeffs, m.moment_coeffs)

    @property
    def cutoff(self) -> float:
        v = C.c_double()
        _check(self.lib.mtpb_cutoff(self.ctx, C.byref(v)))
        return v.value

    def set_stream(self, stream_handle: int):
        """Runs later work on a CUDA stream (e.g. torch.cuda.current_stream()
        .cuda_stream); 0 returns to the context's own stream."""
        _check(self.lib.mtpb_set_stream(self.ctx, C.c_void_p(stream_handle or None)))

    def set_skin(self, skin: float):
        _check(self.lib.mtpb_set_skin(self.ctx, float(skin)))

    # ---- structures path ------------------------------------------------
    def set_center_count(self, n: int):
        """Centres = the first n atoms of later builds (0 = all atoms)."""
        _check(self.lib.mtpb_set_center_count(self.ctx, int(n)))
        self._centers = int(n)

    def build_neighbors(self, batch: StructureBatch):
        self._batch = batch
        st = batch.c_struct()
        _check(self.lib.mtpb_build_neighbors(self.ctx, C.byref(st), _lib.MEMORY_HOST))

    def neighbor_count(self) -> int:
        n = C.c_long()
        _check(self.lib.mtpb_neighbor_count(self.ctx, C.byref(n)))
        return n.value

    def get_neighbors(self):
        """(offsets[N+1], nbr[E] global atom ids, rij[E,3], shift[E])."""
        E = self.neighbor_count()
        N = self._batch.n_atoms
        off = np.zeros(N + 1, np.int32)
        nbr = np.zeros(max(E, 1), np.int32)
        rij = np.zeros((max(E, 1), 3))
        sh = np.zeros(max(E, 1), np.int32)
        _check(self.lib.mtpb_get_neighbors(self.ctx, _ip(off), _ip(nbr), _dp(rij), _ip(sh)))
        return off, nbr[:E], rij[:E], sh[:E]

    def compute(self, site_energy: bool = False):
        """EFS of the last built batch: (energy[S], forces[N,3], stress[S,3,3],
        site_energy[centres] or None); with a centre count the forces are the
        partial sums of those centres' site terms."""
        b = self._batch
        S, N = b.n_structures, b.n_atoms
        nc = min(getattr(self, "_centers", 0) or N, N)
        e = np.zeros(max(S, 1))
        f = np.zeros((max(N, 1), 3))
        st = np.zeros((max(S, 1), 9))
        se = np.zeros(max(nc, 1)) if site_energy else None
        out = _lib.EfsOutput(_dp(e), _dp(f), _dp(st), _dp(se))
        _check(self.lib.mtpb_efs_compute(self.ctx, _lib.MEMORY_HOST, C.byref(out)))
        return e[:S], f[:N], st[:S].reshape(S, 3, 3), (se[:nc] if se is not None else None)

    def efs_structures(self, batch: StructureBatch, reuse_neighbors: bool = False,
                       out=None):
        """mtpb_efs_structures with host arrays: builds (or, with reuse and an
        unchanged layout, refreshes) the lists from batch.positions and writes
        energy[S], forces[N,3], stress[S,9] into `out` (dict of arrays)."""
        self._batch = batch
        st = batch.c_struct()
        o = _lib.EfsOutput(_dp(out.get("energy")), _dp(out.get("forces")),
                           _dp(out.get("stress")), _dp(out.get("site_energy")))
        _check(self.lib.mtpb_efs_structures(self.ctx, C.byref(st), _lib.MEMORY_HOST,
                                            int(reuse_neighbors), C.byref(o)))

    def efs(self, batch: StructureBatch, site_energy: bool = False, reuse_neighbors=False):
        if not (reuse_neighbors and self._batch is not None):
            self.build_neighbors(batch)
        self._batch = batch
        return self.compute(site_energy=site_energy)

    # device-resident path (torch CUDA tensors; plumbing only)
    def efs_device(self, atom_offsets, cells, pbc, positions, types, energy, forces, stress,
                   reuse_neighbors: bool = False):
        st = _lib.Structures(int(atom_offsets.numel()) - 1, _tip(atom_offsets), _tdp(cells),
                             _tip(pbc), _tdp(positions), _tip(types))
        out = _lib.EfsOutput(_tdp(energy), _tdp(forces), _tdp(stress), None)
        _check(self.lib.mtpb_efs_structures(self.ctx, C.byref(st), _lib.MEMORY_DEVICE,
                                            int(reuse_neighbors), C.byref(out)))

    def build_neighbors_device(self, atom_offsets, cells, pbc, positions, types):
        st = _lib.Structures(int(atom_offsets.numel()) - 1, _tip(atom_offsets), _tdp(cells),
                             _tip(pbc), _tdp(positions), _tip(types))
        _check(self.lib.mtpb_build_neighbors(self.ctx, C.byref(st), _lib.MEMORY_DEVICE))

    def compute_device(self, energy, forces, stress):
        out = _lib.EfsOutput(_tdp(energy), _tdp(forces), _tdp(stress), None)
        _check(self.lib.mtpb_efs_compute(self.ctx, _lib.MEMORY_DEVICE, C.byref(out)))

    # ---- caller-supplied lists -----------------------------------------
    def compute_batch(self, offsets, neighbors, types, x, center_count=None,
                      neighbor_vectors=None, neighbor_mask=-1, site_virial=False):
        """MTPGpuDirect::compute_batch with host arrays.  Returns dict with
        energy, site_energy, force[ntotal,3], virial[6] and optionally
        site_virial[ntotal,6]."""
        offsets, neighbors, types, x = _i32(offsets), _i32(neighbors), _i32(types), _f64(x)
        NT = types.shape[0]
        NC = len(offsets) - 1 if center_count is None else int(center_count)
        vec = None if neighbor_vectors is None else _f64(neighbor_vectors)
        force = np.zeros((max(NT, 1), 3))
        se = np.zeros(max(NC, 1))
        en = np.zeros(1)
        gv = np.zeros(6)
        sv = np.zeros((max(NT, 1), 6)) if site_virial else None
        req = _lib.CsrRequest(NC, NT, _ip(offsets), _ip(neighbors), int(neighbor_mask), _dp(vec),
                              _ip(types), _dp(x), _dp(force), 0, _dp(en), _dp(se), _dp(sv),
                              _dp(gv))
        _check(self.lib.mtpb_efs_csr(self.ctx, C.byref(req), _lib.MEMORY_HOST))
        out = {"energy": float(en[0]), "site_energy": se[:NC], "force": force[:NT],
               "virial": gv}
        if site_virial:
            out["site_virial"] = sv[:NT]
        return out

    def compute_lammps(self, ilist, numneigh, firstneigh: List[np.ndarray], type_, type_map, x,
                       f, neighbor_mask=0x3FFFFFFF, energy=None, site_energy=None,
                       site_virial=None, virial=None):
        """PairMLIPGpuDirect::compute semantics: forces/virials are added."""
        ilist, numneigh, type_, type_map = _i32(ilist), _i32(numneigh), _i32(type_), _i32(type_map)
        lists = [_i32(l) for l in firstneigh]
        ptrs = (_lib._ip * len(lists))(*[_ip(l) for l in lists])
        req = _lib.LammpsRequest(len(ilist), _ip(ilist), _ip(numneigh), ptrs, int(neighbor_mask),
                                 type_.shape[0], _ip(type_), _ip(type_map), len(type_map), _dp(x),
                                 _dp(f), _dp(energy), _dp(site_energy), _dp(site_virial),
                                 _dp(virial))
        _check(self.lib.mtpb_efs_lammps(self.ctx, C.byref(req)))

    # ---- training -------------------------------------------------------
    def loss_grad(self, labels_energy=None, labels_forces=None, labels_stress=None,
                  weights=(1.0, 0.01, 0.0001, 1.0, 0.0, 1.0), norm_count: int = 0):
        """Loss, 7 metrics and gradient of the last built batch."""
        te = None if labels_energy is None else _f64(labels_energy)
        tf = None if labels_forces is None else _f64(labels_forces)
        ts = None if labels_stress is None else _f64(labels_stress)
        lab = _lib.Labels(_dp(te), _dp(tf), _dp(ts))
        w = _lib.LossWeights(*weights)
        loss = np.zeros(1)
        metrics = np.zeros(7)
        grad = np.zeros(self.model.coeff_count)
        _check(self.lib.mtpb_loss_grad(self.ctx, C.byref(lab), C.byref(w), int(norm_count),
                                       _lib.MEMORY_HOST, _dp(loss), _dp(metrics), _dp(grad)))
        return float(loss[0]), metrics, grad

    def loss_grad_device(self, labels_energy, labels_forces, labels_stress, loss, metrics, grad,
                         weights=(1.0, 0.01, 0.0001, 1.0, 0.0, 1.0), norm_count: int = 0):
        """mtpb_loss_grad with device arrays (torch CUDA tensors; a label may be
        None): loss[1], metrics[7] and grad[coeff_count] are written on the
        context stream without a host synchronisation."""
        lab = _lib.Labels(_tdp(labels_energy), _tdp(labels_forces), _tdp(labels_stress))
        w = _lib.LossWeights(*weights)
        _check(self.lib.mtpb_loss_grad(self.ctx, C.byref(lab), C.byref(w), int(norm_count),
                                       _lib.MEMORY_DEVICE, _tdp(loss), _tdp(metrics),
                                       _tdp(grad)))

    def check_training_values(self) -> int:
        """Finite check of the last loss_grad call: -1 when the loss, metrics
        and gradient are all finite; otherwise raises MTPBError (status 6)
        naming the first non-finite value."""
        first = C.c_long()
        _check(self.lib.mtpb_check_training_values(self.ctx, C.byref(first)))
        return first.value

    def check_device_status(self) -> None:
        """Synchronises and raises MTPBError (status MTPB_ERR_CUDA) when a
        graph kernel's bounded wait gave up since the last check (device-
        memory calls do not check this themselves)."""
        _check(self.lib.mtpb_check_device_status(self.ctx))

    def last_train_timings(self):
        t = np.zeros(6)
        _check(self.lib.mtpb_last_train_timings(self.ctx, _dp(t)))
        return t

    # ---- diagnostics ----------------------------------------------------
    def last_timings(self):
        t = np.zeros(5)
        _check(self.lib.mtpb_last_timings(self.ctx, _dp(t)))
        return t

    def last_launch_count(self) -> int:
        n = C.c_int()
        _check(self.lib.mtpb_last_launch_count(self.ctx, C.byref(n)))
        return n.value

    def site_moments(self):
        N = self._batch.n_atoms
        nb = self.model.alpha_index_basic_count
        b = np.zeros((N, nb))
        a = np.zeros((N, nb))
        _check(self.lib.mtpb_get_site_moments(self.ctx, _dp(b), _dp(a)))
        return b, a

    def edge_derivatives(self, n_edges: int):
        d = np.zeros((max(n_edges, 1), 3))
        _check(self.lib.mtpb_get_edge_derivatives(self.ctx, _dp(d)))
        return d[:n_edges]


class PotMTP:
    """getEFS of one structure with GPU neighbour lists (PotMTP::getEFS)."""

    def __init__(self, model: MTPModel, device: int = 0):
        self.gpu = MTPGpuDirect(model, device)

    def getEFS(self, structure: Dict[str, np.ndarray]):
        batch = StructureBatch.from_structures([structure])
        e, f, s, se = self.gpu.efs(batch, site_energy=True)
        return float(e[0]), f, s[0], se
