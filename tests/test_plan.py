"""The moment-graph program that the device executes, run on the CPU by a
numpy interpreter of the record semantics and compared with the oracle's
site energies and basic-moment adjoints.  Needs no GPU."""
import ctypes as C

import numpy as np
import pytest

from conftest import load_model
from mtpb200 import configs

END, GLOBAL, ENERGY = 2, 4, 8


def program(model):
    import mtpb200
    from mtpb200 import _ModelKeep, _lib
    lib = mtpb200.library()
    keep = _ModelKeep(model)
    ints = [C.c_int() for _ in range(6)]
    nrec = C.c_long()
    sob = np.zeros(model.alpha_index_basic_count, np.int32)
    phases = np.zeros(64, np.int32)
    rc = lib.mtpb_graph_program(C.byref(keep.view), C.byref(ints[0]),
                                sob.ctypes.data_as(_lib._ip), C.byref(ints[1]), C.byref(ints[2]),
                                C.byref(ints[3]), C.byref(ints[4]), C.byref(ints[5]),
                                phases.ctypes.data_as(_lib._ip), C.byref(nrec), None)
    assert rc == 0, lib.mtpb_last_error()
    recs = np.zeros((nrec.value, 4), np.uint32)
    rc = lib.mtpb_graph_program(C.byref(keep.view), None, None, None, None, None, None, None,
                                None, None, recs.ctypes.data_as(C.POINTER(C.c_uint)))
    assert rc == 0
    nslot, nrows, one, zero, nf, nr = (v.value for v in ints)
    streams = nrec.value // int(phases[:nf + nr].sum())
    return dict(nslot=nslot, sob=sob, nrows=nrows, one=one, zero=zero, n_fwd=nf, n_rev=nr,
                phase_rows=phases[:nf + nr], recs=recs, streams=streams)


def interpret(prog, basic_slots, species_part):
    """Executes the record streams (efs.cu k_dag semantics) for all atoms."""
    S = prog["streams"]
    natoms = basic_slots.shape[1]
    rows = np.zeros((prog["nrows"], natoms))
    rows[:prog["nslot"]] = basic_slots
    rows[prog["one"]] = 1.0
    recs = prog["recs"].reshape(-1, S, 4)
    coef = recs[:, :, 2:4].copy().view(np.float64)[:, :, 0]
    s1, s2 = recs[:, :, 0] & 0xFFFF, recs[:, :, 0] >> 16
    out, fl = recs[:, :, 1] & 0xFFFF, recs[:, :, 1] >> 16
    acc = np.zeros((S, natoms))
    E = np.zeros((S, natoms))
    adj = np.zeros((prog["nslot"], natoms))
    r = 0
    energy = None
    for ph, nrow in enumerate(prog["phase_rows"]):
        acc[:] = 0.0
        for _ in range(nrow):
            writes = []
            for s in range(S):
                c = coef[r, s]
                acc[s] = acc[s] + c * rows[s1[r, s]] * rows[s2[r, s]]
                if fl[r, s] & ENERGY:
                    E[s] += c * acc[s]
                if fl[r, s] & END:
                    if fl[r, s] & GLOBAL:
                        adj[out[r, s]] = acc[s]
                    else:
                        writes.append((out[r, s], acc[s].copy()))
                    acc[s] = 0.0
            for o, v in writes:
                rows[o] = v
            r += 1
        if ph + 1 == prog["n_fwd"]:
            energy = species_part + E.sum(0)
    return energy, adj


@pytest.mark.parametrize("name", ["pair_k1.mtp", "many_body_k3.mtp", "l16_k2.mtp", "l20_k3.mtp"])
def test_program_matches_oracle(oracle, name):
    m = load_model(name)
    prog = program(m)
    assert prog["n_fwd"] >= 1 and prog["n_rev"] >= 1
    st = configs.config2(1, seed=71)[0]
    st["types"] = np.minimum(st["types"], m.species_count - 1).astype(np.int32)
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], m.cutoff)
    se, _ = oracle.site_derivatives(m, st["types"], nl)
    b, a = oracle.site_moments(m, st["types"], nl)
    n = min(24, b.shape[0])
    slots = np.zeros((prog["nslot"], n))
    slots[prog["sob"]] = b[:n].T
    e, adj = interpret(prog, slots, m.species_coeffs[st["types"][:n]])
    assert np.max(np.abs(e - se[:n])) < 1e-12 * max(1, np.max(np.abs(se)))
    assert np.max(np.abs(adj[prog["sob"]].T - a[:n])) < 1e-11 * max(1, np.max(np.abs(a)))
    unused = np.setdiff1d(np.arange(prog["nslot"]), prog["sob"])
    assert np.all(adj[unused] == 0)


def test_program_stream_balance_level20():
    """Padding stays small: items longer than a phase's even share are split
    into partial sums plus a combine phase, and the level-20 graph runs on 64
    streams; its rows still fit shared memory at 16 atoms per block."""
    m = load_model("l20_k2.mtp")
    prog = program(m)
    assert prog["streams"] == 64
    recs = prog["recs"].reshape(-1, 64, 4)
    pad = np.sum((recs[:, :, 2] == 0) & (recs[:, :, 3] == 0) & (recs[:, :, 1] >> 16 == 0))
    assert pad / recs.shape[0] / 64 < 0.08
    assert prog["nrows"] * 16 * 8 <= 180 * 1024


def test_level24_program_balance():
    """The generated level-24 graph: at most 4% padding after splitting."""
    prog = program(configs.level24_model())
    S = prog["streams"]
    recs = prog["recs"].reshape(-1, S, 4)
    pad = np.sum((recs[:, :, 2] == 0) & (recs[:, :, 3] == 0) & (recs[:, :, 1] >> 16 == 0))
    assert pad / recs.shape[0] / S < 0.04


def test_level24_program_64_streams_matches_oracle(oracle):
    """The generated level-24 graph (beyond shared memory) is planned on 64
    streams; its program still reproduces the oracle's site energies and
    basic-moment adjoints."""
    m = configs.level24_model()
    prog = program(m)
    assert prog["streams"] == 64
    st = configs.config4_structures(1, seed=72)[0]
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], m.cutoff)
    se, _ = oracle.site_derivatives(m, st["types"], nl)
    b, a = oracle.site_moments(m, st["types"], nl)
    n = 4
    slots = np.zeros((prog["nslot"], n))
    slots[prog["sob"]] = b[:n].T
    e, adj = interpret(prog, slots, m.species_coeffs[st["types"][:n]])
    assert np.max(np.abs(e - se[:n])) < 1e-12 * max(1, np.max(np.abs(se)))
    assert np.max(np.abs(adj[prog["sob"]].T - a[:n])) < 1e-11 * max(1, np.max(np.abs(a)))
