"""ctypes declarations of include/mtpb200.h.

The shared library is built in-tree (``imr-mlp_b200/libmtpb200.so``, see the
package Makefile); importing this module without it raises ImportError: there
is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("MTPB200_LIB", os.path.join(PKG_ROOT, "libmtpb200.so"))

_dp = C.POINTER(C.c_double)
_ip = C.POINTER(C.c_int)

MTPB_OK = 0
MTPB_ERR_ARGUMENT = 1
MTPB_ERR_UNSUPPORTED = 2
MTPB_ERR_CUDA = 3
MTPB_ERR_MEMORY = 4
MTPB_ERR_STATE = 5
MEMORY_HOST = 0
MEMORY_DEVICE = 1


class RadialFamilyView(C.Structure):
    _fields_ = [("type", C.c_int), ("cutoff_type", C.c_int), ("shift_type", C.c_int),
                ("one_minus_chebyshev", C.c_int), ("b", C.c_double), ("r1", C.c_double),
                ("r2", C.c_double), ("shift_lambda", C.c_double),
                ("shift_scale_lambda", C.c_double), ("poly_matrix", _dp), ("poly_norm", _dp)]


class ModelView(C.Structure):
    _fields_ = [
        ("species_count", C.c_int), ("radial_func_count", C.c_int), ("rb_size", C.c_int),
        ("radial_basis_split", C.c_int), ("min_dist", _dp), ("max_dist", _dp),
        ("scaling", C.c_double), ("alpha_moments_count", C.c_int),
        ("alpha_index_basic_count", C.c_int), ("alpha_index_times_count", C.c_int),
        ("alpha_scalar_moments", C.c_int), ("alpha_index_basic", _ip),
        ("alpha_index_times", _ip), ("alpha_moment_mapping", _ip), ("radial_coeffs", _dp),
        ("species_coeffs", _dp), ("moment_coeffs", _dp),
        ("radial_family", C.POINTER(RadialFamilyView)),
    ]


def radial_family_array(model):
    """ctypes array of the model's radial families (None for RBChebyshev) and
    the numpy arrays its RBPolyB pointers refer to (keep both alive)."""
    from .mtpfile import CUTOFF_TYPES, SHIFT_TYPES
    fams = model.radial_family
    if not fams:
        return None, []
    arr = (RadialFamilyView * len(fams))()
    keep = []
    for i, f in enumerate(fams):
        pm = pn = None
        if f.poly_matrix is not None:
            keep += [np.ascontiguousarray(f.poly_matrix, dtype=np.float64),
                     np.ascontiguousarray(f.poly_norm, dtype=np.float64)]
            pm, pn = keep[-2].ctypes.data_as(_dp), keep[-1].ctypes.data_as(_dp)
        arr[i] = RadialFamilyView(f.type_id, CUTOFF_TYPES[f.cutoff_type],
                                  SHIFT_TYPES[f.shift_type], int(f.one_minus_chebyshev),
                                  float(f.b), float(f.r1), float(f.r2), float(f.shift_lambda),
                                  float(f.shift_scale_lambda), pm, pn)
    return arr, keep


class Structures(C.Structure):
    _fields_ = [("n_structures", C.c_int), ("atom_offsets", _ip), ("cells", _dp),
                ("pbc", _ip), ("positions", _dp), ("types", _ip)]


class EfsOutput(C.Structure):
    _fields_ = [("energy", _dp), ("forces", _dp), ("stress", _dp), ("site_energy", _dp)]


class CsrRequest(C.Structure):
    _fields_ = [("center_count", C.c_int), ("ntotal", C.c_int), ("offsets", _ip),
                ("neighbors", _ip), ("neighbor_mask", C.c_int), ("neighbor_vectors", _dp),
                ("types", _ip), ("x", _dp), ("force", _dp), ("accumulate_force", C.c_int),
                ("total_energy", _dp), ("site_energy", _dp), ("site_virial", _dp),
                ("global_virial", _dp)]


class LammpsRequest(C.Structure):
    _fields_ = [("inum", C.c_int), ("ilist", _ip), ("numneigh", _ip),
                ("firstneigh", C.POINTER(_ip)), ("neighbor_mask", C.c_int), ("ntotal", C.c_int),
                ("type", _ip), ("type_map", _ip), ("type_map_count", C.c_int), ("x", _dp),
                ("f", _dp), ("energy", _dp), ("site_energy", _dp), ("site_virial", _dp),
                ("virial", _dp)]


class LossWeights(C.Structure):
    _fields_ = [("weight_eng", C.c_double), ("weight_force", C.c_double),
                ("weight_stress", C.c_double), ("weight_eng_power", C.c_double),
                ("weight_force_power", C.c_double), ("weight_stress_power", C.c_double)]


class Labels(C.Structure):
    _fields_ = [("energy", _dp), ("forces", _dp), ("stress", _dp)]


# (name, restype, argtypes) of every exported entry point
SIGNATURES = [
    ("mtpb_last_error", C.c_char_p, []),
    ("mtpb_abi_version", C.c_int, []),
    ("mtpb_device_count", C.c_int, [_ip]),
    ("mtpb_create", C.c_int, [C.c_int, C.POINTER(ModelView), C.POINTER(C.c_void_p)]),
    ("mtpb_destroy", C.c_int, [C.c_void_p]),
    ("mtpb_update_coefficients", C.c_int, [C.c_void_p, _dp, _dp, _dp]),
    ("mtpb_set_stream", C.c_int, [C.c_void_p, C.c_void_p]),
    ("mtpb_cutoff", C.c_int, [C.c_void_p, _dp]),
    ("mtpb_set_skin", C.c_int, [C.c_void_p, C.c_double]),
    ("mtpb_build_neighbors", C.c_int, [C.c_void_p, C.POINTER(Structures), C.c_int]),
    ("mtpb_neighbor_count", C.c_int, [C.c_void_p, C.POINTER(C.c_long)]),
    ("mtpb_get_neighbors", C.c_int, [C.c_void_p, _ip, _ip, _dp, _ip]),
    ("mtpb_efs_compute", C.c_int, [C.c_void_p, C.c_int, C.POINTER(EfsOutput)]),
    ("mtpb_efs_structures", C.c_int, [C.c_void_p, C.POINTER(Structures), C.c_int, C.c_int,
                                      C.POINTER(EfsOutput)]),
    ("mtpb_efs_csr", C.c_int, [C.c_void_p, C.POINTER(CsrRequest), C.c_int]),
    ("mtpb_efs_lammps", C.c_int, [C.c_void_p, C.POINTER(LammpsRequest)]),
    ("mtpb_efs_csr_noalloc", C.c_int, [C.c_void_p, C.POINTER(CsrRequest)]),
    ("mtpb_loss_grad", C.c_int, [C.c_void_p, C.POINTER(Labels), C.POINTER(LossWeights), C.c_int,
                                 C.c_int, _dp, _dp, _dp]),
    ("mtpb_last_timings", C.c_int, [C.c_void_p, _dp]),
    ("mtpb_last_train_timings", C.c_int, [C.c_void_p, _dp]),
    ("mtpb_check_training_values", C.c_int, [C.c_void_p, C.POINTER(C.c_long)]),
    ("mtpb_check_device_status", C.c_int, [C.c_void_p]),
    ("mtpb_debug_flag_device_error", C.c_int, [C.c_void_p]),
    ("mtpb_set_center_count", C.c_int, [C.c_void_p, C.c_int]),
    ("mtpb_last_launch_count", C.c_int, [C.c_void_p, _ip]),
    ("mtpb_get_site_moments", C.c_int, [C.c_void_p, _dp, _dp]),
    ("mtpb_get_edge_derivatives", C.c_int, [C.c_void_p, _dp]),
    ("mtpb_graph_program", C.c_int, [C.POINTER(ModelView), _ip, _ip, _ip, _ip, _ip, _ip, _ip, _ip,
                                     C.POINTER(C.c_long), C.POINTER(C.c_uint)]),
]


def load(path: str = LIB_PATH) -> C.CDLL:
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `make -C imr-mlp_b200` "
            "(or __graft_entry__.build()); there is no CPU fallback")
    lib = C.CDLL(path)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib
