"""C ABI and host-side checks that need no GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import MODELS, ROOT, load_model

HEADER = os.path.join(ROOT, "include", "mtpb200.h")


def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(mtpb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from mtpb200 import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    syms = header_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/mtpb200.h but not exported"


def test_python_signatures_cover_header():
    from mtpb200 import _lib
    declared = set(header_symbols())
    bound = {name for name, _, _ in _lib.SIGNATURES}
    assert declared == bound


def test_abi_version_and_error_without_device():
    import mtpb200
    lib = mtpb200.library()
    assert lib.mtpb_abi_version() == 3
    if mtpb200.device_count() > 0:
        pytest.skip("a device is present")
    m = load_model("pair_k1.mtp")
    with pytest.raises(mtpb200.MTPBError) as ei:
        mtpb200.MTPGpuDirect(m, 0)
    assert ei.value.status in (3, 1)
    assert lib.mtpb_last_error().decode()


def test_null_arguments_rejected():
    import mtpb200
    lib = mtpb200.library()
    assert lib.mtpb_create(0, None, None) == 1
    assert lib.mtpb_destroy(None) == 0
    assert lib.mtpb_efs_compute(None, 0, None) == 1


def test_mtp_roundtrip_all_models():
    from mtpb200 import format_mtp, parse_mtp
    for name in sorted(os.listdir(MODELS)):
        m = load_model(name)
        m2 = parse_mtp(format_mtp(m))
        for f in ("alpha_index_basic", "alpha_index_times", "alpha_moment_mapping",
                  "radial_coeffs", "species_coeffs", "moment_coeffs", "min_dist", "max_dist"):
            assert np.array_equal(getattr(m, f), getattr(m2, f)), (name, f)
        assert m.scaling == m2.scaling and m.radial_basis_split == m2.radial_basis_split


def test_mtp_parser_rejects_bad_graph():
    from mtpb200 import format_mtp, parse_mtp
    m = load_model("pair_k1.mtp")
    bad = m.alpha_index_times.copy()
    bad[0, 3] = 1   # a basic moment as product target
    text = format_mtp(m.__class__(**{**m.__dict__, "alpha_index_times": bad}))
    with pytest.raises(ValueError):
        parse_mtp(text)


def test_mtp_parser_reads_reference_templates():
    """The shipped Shapeev templates parse with the PotMTP scaling default."""
    from mtpb200 import read_mtp
    corpus = os.path.join(os.environ.get("IMRMLP_REFERENCE", "/root/reference"),
                          "unitest", "test-data", "mtp-basis-corpus")
    if not os.path.isdir(corpus):
        pytest.skip("reference checkout absent")
    m = read_mtp(os.path.join(corpus, "shapeev-20.mtp"))
    assert (m.alpha_index_basic_count, m.alpha_index_times_count, m.alpha_scalar_moments,
            m.alpha_moments_count) == (295, 4665, 288, 1035)
    assert m.scaling == 0.01
    assert m.basis_shape() == [8, 6, 4, 2, 0]


@pytest.mark.parametrize("field,value,message", [
    ("type", 7, b"unsupported radial basis type 7"),          # a legacy family
    ("type", 5, b"RBPolyB / RBPolyBCos need poly_matrix"),    # RBPolyB without its matrix
    ("cutoff_type", 12, b"unknown configurable cutoff_type"),
    ("r2", 6.0, b"smoothstep7 cutoff requires"),
    ("shift_lambda", float("nan"), b"non-finite radial parameter"),
])
def test_radial_family_validation(field, value, message):
    """Model validation of the radial families runs before any device call:
    unsupported families and invalid parameters are refused by mtpb_create."""
    import ctypes as C
    import mtpb200
    from helpers import with_radial_family
    m = with_radial_family(load_model("l16_k2.mtp"), "cfg_smooth7_tanh_flip")
    keep = mtpb200._ModelKeep(m)
    setattr(keep.families[0], field, value)
    lib = mtpb200.library()
    ctx = C.c_void_p()
    rc = lib.mtpb_create(0, C.byref(keep.view), C.byref(ctx))
    assert rc == 1 and message in lib.mtpb_last_error(), lib.mtpb_last_error()
    assert not ctx.value
