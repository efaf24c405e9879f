"""GPM v2 bundles (mtpb200.gpm) on the CPU: write / read round trips of
plain, split, multi-family and RBPolyB models, and the reference's own loader
(MLIPCore's read_model_text / setup, runtime/mtp/mlip.cpp:350-428, compiled
in oracle/_ref/libref.so) reading the bundles this module writes: the model
it derives gives the same energies and forces as the original model.
Needs no GPU."""
import dataclasses

import numpy as np
import pytest

from conftest import load_model
from helpers import with_polyb, with_radial_family
from mtpb200 import configs, format_mtp, parse_mtp
from mtpb200.gpm import GPMReader, from_bytes, read_gpm, to_bytes, write_gpm


def _models(reference=None):
    l16 = load_model("l16_k2.mtp")
    out = {"l16": l16, "l20_k3": load_model("l20_k3.mtp"),
           "split_k3": load_model("many_body_k3.mtp"),
           "configurable": with_radial_family(l16, "cfg_smooth7_tanh_flip"),
           "poly5": with_radial_family(l16, "poly5_min26")}
    if reference is not None:
        out["polyb"] = with_polyb(l16, "RBPolyB", reference)
        out["polybcos_split"] = with_polyb(l16, "RBPolyBCos", reference, split=True)
    return out


def _same(a, b):
    for f in dataclasses.fields(a):
        if f.name == "potential_name":
            continue
        x, y = getattr(a, f.name), getattr(b, f.name)
        if f.name == "radial_family":
            assert (x is None) == (y is None)
            if x:
                assert x == y
                for fa, fb in zip(x, y):
                    for arr in ("poly_matrix", "poly_norm"):
                        pa, pb = getattr(fa, arr), getattr(fb, arr)
                        assert (pa is None) == (pb is None)
                        if pa is not None:
                            assert np.array_equal(np.asarray(pa), np.asarray(pb))
        elif isinstance(x, np.ndarray) or isinstance(y, np.ndarray):
            assert np.array_equal(np.asarray(x), np.asarray(y)), f.name
        else:
            assert x == y, f.name


def test_round_trip(tmp_path):
    for name, m in _models().items():
        path = str(tmp_path / f"{name}.gpm")
        write_gpm(m, path)
        _same(m, read_gpm(path))


def test_round_trip_polyb_keeps_the_matrix(reference, tmp_path):
    for name in ("polyb", "polybcos_split"):
        m = _models(reference)[name]
        _same(m, from_bytes(to_bytes(m)))


def test_container_layout():
    data = to_bytes(load_model("l16_k2.mtp"), metadata={"source": "test"})
    assert data[:8] == b"GPMLMODL"
    r = GPMReader(data)
    assert r.start % 64 == 0
    assert all(int(b["offset"]) % 64 == 0 for b in r.blocks.values())
    node = r.manifest["models"][r.manifest["root_model"]]
    assert node["type"] == "mtp" and node["configuration"]["metadata"] == {"source": "test"}
    bad = bytearray(data)
    bad[8] = 3                                   # major version 3
    with pytest.raises(ValueError):
        GPMReader(bytes(bad))


@pytest.mark.parametrize("name", ["l16", "l20_k3", "split_k3", "configurable", "poly5",
                                  "polyb", "polybcos_split"])
def test_reference_loader_reads_our_bundles(oracle, reference, tmp_path, name):
    """The reference derives .mtp text from our bundle (folding the radial
    scaling into the coefficients); that model's EFS equals the original's."""
    m = _models(reference)[name]
    path = str(tmp_path / f"{name}.gpm")
    write_gpm(m, path)
    text = reference.model_text(path)
    st = configs.config1()
    if m.species_count == 3:
        st = configs.config2(1, seed=91)[0]
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], m.cutoff)
    wrapped = oracle.wrap(st["cell"], st["pbc"], st["positions"])
    e0, se0, f0, _ = reference.mlip_efs(format_mtp(m), st["types"], nl, wrapped)
    e1, se1, f1, _ = reference.mlip_efs(text, st["types"], nl, wrapped)
    n = len(st["types"])
    assert abs(e1 - e0) / n < 1e-13 * max(1.0, abs(e0))
    assert np.max(np.abs(f1 - f0)) < 1e-12 * max(1.0, np.max(np.abs(f0)))
    assert np.max(np.abs(f0)) > 0
    if not name.startswith("polyb"):
        # the derived text parses back into the same graph and coefficients
        back = parse_mtp(text)
        assert np.array_equal(back.alpha_index_times, m.alpha_index_times)
        assert np.allclose(back.radial_coeffs * back.scaling, m.radial_coeffs * m.scaling,
                           rtol=1e-15, atol=0)
