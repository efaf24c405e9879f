"""mtpb_efs_csr_noalloc, the entry point for callers that cannot allocate
device memory while they run (an MD engine or plug-in host that has already
claimed the GPU's memory for its own pool, or a real-time loop that must not
enter the allocator).  Its scratch lives in a fixed array inside the library,
so it is compared here with the allocating CSR entry point on the same device
inputs, several calls in a row with different systems (the array keeps the
previous call's contents).  Collected last so that a failure here leaves the
rest of the suite already run."""
import ctypes as C

import numpy as np
import pytest

from mtpb200 import configs

pytestmark = pytest.mark.gpu

TOL_E_ATOM = 1e-10
TOL_F = 1e-9
TOL_W = 1e-9
MASK_BIT = 0x40000000   # a LAMMPS-style flag bit above the index mask


def _problem(oracle, model, st):
    """Periodic structure as a CSR request with explicit edge vectors."""
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], model.cutoff)
    return dict(offsets=nl.offsets.astype(np.int32), neighbors=nl.nbr.astype(np.int32),
                vectors=np.ascontiguousarray(nl.rij), types=st["types"].astype(np.int32),
                x=oracle.wrap(st["cell"], st["pbc"], st["positions"]),
                center_count=len(st["types"]))


def _ghost_problem(oracle, model, st):
    """The structure with its periodic images as explicit ghost atoms, one per
    distinct (atom, image) pair, as a domain-decomposed MD code supplies them:
    neighbours of the centres are centres or ghosts, edge vectors implied by
    the positions (no neighbor_vectors)."""
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], model.cutoff)
    n = len(st["types"])
    cell = np.asarray(st["cell"], dtype=np.float64).reshape(3, 3)
    x0 = oracle.wrap(st["cell"], st["pbc"], st["positions"])
    centers = np.repeat(np.arange(n), np.diff(nl.offsets))
    img = np.rint((x0[centers] + nl.rij - x0[nl.nbr]) @ np.linalg.inv(cell)).astype(np.int64)
    assert np.all(np.abs(img) < 16)
    key = (nl.nbr.astype(np.int64) << 15) + ((img[:, 0] + 16) << 10) + ((img[:, 1] + 16) << 5) \
        + (img[:, 2] + 16)
    own = np.all(img == 0, axis=1)
    uniq, inv = np.unique(key[~own], return_inverse=True)
    ghost_atom = uniq >> 15
    gimg = np.stack([((uniq >> 10) & 31) - 16, ((uniq >> 5) & 31) - 16, (uniq & 31) - 16], axis=1)
    xg = x0[ghost_atom] + gimg @ cell
    nbr = nl.nbr.astype(np.int32).copy()
    nbr[~own] = (n + inv).astype(np.int32)
    return dict(offsets=nl.offsets.astype(np.int32), neighbors=nbr | MASK_BIT,
                types=np.concatenate([st["types"], st["types"][ghost_atom]]).astype(np.int32),
                x=np.ascontiguousarray(np.concatenate([x0, xg])), center_count=n,
                mask=0x3FFFFFFF)


def _join(a, b):
    """Two ghosted requests as one: the centres of both first, then the ghosts
    of both (neighbour indices renumbered, the flag bit kept)."""
    mask = 0x3FFFFFFF
    na, nb = a["center_count"], b["center_count"]
    ga, gb = len(a["types"]) - na, len(b["types"]) - nb
    nc = na + nb

    def renum(nbr, n, center0, ghost0):
        j = nbr & mask
        return np.where(j < n, center0 + j, ghost0 + (j - n)).astype(np.int32) | (nbr & ~mask)

    return dict(
        offsets=np.concatenate([a["offsets"], a["offsets"][-1] + b["offsets"][1:]]).astype(np.int32),
        neighbors=np.concatenate([renum(a["neighbors"], na, 0, nc),
                                  renum(b["neighbors"], nb, na, nc + ga)]),
        types=np.concatenate([a["types"][:na], b["types"][:nb], a["types"][na:],
                              b["types"][nb:]]).astype(np.int32),
        x=np.ascontiguousarray(np.concatenate([a["x"][:na], b["x"][:nb], a["x"][na:],
                                               b["x"][nb:]])),
        center_count=nc, mask=mask)


def _run(gpu, prob, noalloc, torch, accumulate=False):
    from mtpb200 import _check, _lib
    dev = torch.device("cuda", 0)
    t = {k: torch.from_numpy(v).to(dev) for k, v in prob.items()
         if isinstance(v, np.ndarray)}
    nt = len(prob["types"])
    nc = prob["center_count"]
    f0 = np.linspace(-1.0, 1.0, 3 * nt).reshape(nt, 3) if accumulate else np.zeros((nt, 3))
    out = dict(force=torch.from_numpy(f0).to(dev),
               energy=torch.zeros(1, dtype=torch.float64, device=dev),
               site_energy=torch.zeros(max(nc, 1), dtype=torch.float64, device=dev),
               site_virial=torch.zeros((nt, 6), dtype=torch.float64, device=dev),
               virial=torch.zeros(6, dtype=torch.float64, device=dev))
    dp = lambda a: C.cast(C.c_void_p(a.data_ptr()), _lib._dp)   # noqa: E731
    ip = lambda a: C.cast(C.c_void_p(a.data_ptr()), _lib._ip)   # noqa: E731
    vec = dp(t["vectors"]) if "vectors" in t else None
    req = _lib.CsrRequest(nc, nt, ip(t["offsets"]), ip(t["neighbors"]), prob.get("mask", -1),
                          vec, ip(t["types"]), dp(t["x"]), dp(out["force"]), int(accumulate),
                          dp(out["energy"]), dp(out["site_energy"]), dp(out["site_virial"]),
                          dp(out["virial"]))
    torch.cuda.synchronize()
    if noalloc:
        _check(gpu.lib.mtpb_efs_csr_noalloc(gpu.ctx, C.byref(req)))
    else:
        _check(gpu.lib.mtpb_efs_csr(gpu.ctx, C.byref(req), _lib.MEMORY_DEVICE))
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in out.items()}


def _compare(gpu, prob, torch, accumulate=False):
    """The no-allocation call against mtpb_efs_csr on the same device inputs;
    mtpb_efs_csr adds into caller forces only for host arrays, so with
    accumulation the reference is its plain result plus the caller's forces."""
    ref = _run(gpu, prob, False, torch, False)
    got = _run(gpu, prob, True, torch, accumulate)
    if accumulate:
        nt = len(prob["types"])
        ref["force"] = ref["force"] + np.linspace(-1.0, 1.0, 3 * nt).reshape(nt, 3)
    nc = prob["center_count"]
    assert abs(got["energy"][0] - ref["energy"][0]) / max(nc, 1) < TOL_E_ATOM
    assert np.max(np.abs(got["site_energy"] - ref["site_energy"])) < TOL_E_ATOM
    assert np.max(np.abs(got["force"] - ref["force"])) < TOL_F
    assert np.max(np.abs(got["virial"] - ref["virial"])) < TOL_W
    assert np.max(np.abs(got["site_virial"] - ref["site_virial"])) < TOL_W
    if nc:
        assert np.max(np.abs(ref["force"])) > 0
    return got


def test_noalloc_matches_allocating_entry_point_twice(oracle, model_l16):
    torch = pytest.importorskip("torch")
    from mtpb200 import MTPGpuDirect
    first = configs.config1()
    second = configs.config2(1, seed=55)[0]
    second["types"] = np.minimum(second["types"], 1).astype(np.int32)
    with MTPGpuDirect(model_l16, 0) as gpu:
        for st in (first, second):
            _compare(gpu, _problem(oracle, model_l16, st), torch)


def test_noalloc_ghosts_implicit_vectors_accumulate(oracle, model_l16, model_l20_k3):
    """Ghost atoms (ntotal > center_count, more than 1024 atoms so the sums run
    over several segments), masked neighbour indices, edge vectors from the
    positions, forces added to what the caller holds; then a K=3 level-20 model
    on a strained 3-species cell, each call after the other on one array."""
    torch = pytest.importorskip("torch")
    from mtpb200 import MTPGpuDirect
    st1 = configs.config1()
    st3 = next(st for st in configs.config2(16, seed=7) if len(st["types"]) == 256)
    st2 = dict(st3, types=np.minimum(st3["types"], 1).astype(np.int32))
    prob = _join(_ghost_problem(oracle, model_l16, st1), _ghost_problem(oracle, model_l16, st2))
    assert 1024 < len(prob["types"]) <= 4096
    with MTPGpuDirect(model_l16, 0) as gpu:
        _compare(gpu, prob, torch, accumulate=True)
        _compare(gpu, prob, torch, accumulate=False)
    prob3 = _join(_ghost_problem(oracle, model_l20_k3, st3),
                  _ghost_problem(oracle, model_l20_k3, st1))
    assert 1024 < len(prob3["types"]) <= 4096
    with MTPGpuDirect(model_l20_k3, 0) as gpu:
        _compare(gpu, prob3, torch)
        _compare(gpu, _problem(oracle, model_l20_k3, st3), torch)


def _bad_call(gpu, torch, prob):
    from mtpb200 import MTPBError, _check, _lib
    dev = torch.device("cuda", 0)
    t = {k: torch.from_numpy(v).to(dev) for k, v in prob.items() if isinstance(v, np.ndarray)}
    n = len(prob["types"])
    force = torch.zeros((n, 3), dtype=torch.float64, device=dev)
    ip = lambda a: C.cast(C.c_void_p(a.data_ptr()), _lib._ip)   # noqa: E731
    dp = lambda a: C.cast(C.c_void_p(a.data_ptr()), _lib._dp)   # noqa: E731
    req = _lib.CsrRequest(prob["center_count"], n, ip(t["offsets"]), ip(t["neighbors"]), -1,
                          None, ip(t["types"]), dp(t["x"]), dp(force), 0, None, None, None,
                          None)
    with pytest.raises(MTPBError) as ei:
        _check(gpu.lib.mtpb_efs_csr_noalloc(gpu.ctx, C.byref(req)))
    torch.cuda.synchronize()
    return ei.value


def test_noalloc_rejects_bad_indices(oracle, model_l16):
    """Out-of-range neighbour indices, types and offsets are reported as
    argument errors before any kernel indexes with them; a good call after
    them still matches the allocating entry point."""
    torch = pytest.importorskip("torch")
    from mtpb200 import MTPGpuDirect
    base = _problem(oracle, model_l16, configs.config1())
    base.pop("vectors")
    n = base["center_count"]
    with MTPGpuDirect(model_l16, 0) as gpu:
        p = dict(base, neighbors=base["neighbors"].copy())
        p["neighbors"][17] = n + 5
        err = _bad_call(gpu, torch, p)
        assert err.status == 1 and "neighbor index out of range at edge 17" in str(err)
        p = dict(base, neighbors=base["neighbors"].copy())
        p["neighbors"][3] = -2
        assert "edge 3" in str(_bad_call(gpu, torch, p))
        p = dict(base, types=base["types"].copy())
        p["types"][40] = model_l16.species_count
        err = _bad_call(gpu, torch, p)
        assert err.status == 1 and "type out of range at atom 40" in str(err)
        p = dict(base, offsets=base["offsets"].copy())
        p["offsets"][10] = p["offsets"][12] + 1
        err = _bad_call(gpu, torch, p)
        assert err.status == 1 and "non-decreasing" in str(err)
        # offsets shifted by one (the neighbour array still holds offsets[n] entries)
        p = dict(base, offsets=base["offsets"] + 1,
                 neighbors=np.concatenate([base["neighbors"], [0]]).astype(np.int32))
        assert "offsets[0]" in str(_bad_call(gpu, torch, p))
        _compare(gpu, _problem(oracle, model_l16, configs.config1()), torch)


def test_noalloc_rejects_oversized_request(model_l16):
    torch = pytest.importorskip("torch")
    from mtpb200 import MTPBError, MTPGpuDirect, _check, _lib
    n = 5000   # above the 4096-atom limit of the scratch array
    dev = torch.device("cuda", 0)
    off = torch.zeros(n + 1, dtype=torch.int32, device=dev)
    types = torch.zeros(n, dtype=torch.int32, device=dev)
    x = torch.zeros((n, 3), dtype=torch.float64, device=dev)
    ip = lambda a: C.cast(C.c_void_p(a.data_ptr()), _lib._ip)   # noqa: E731
    dp = lambda a: C.cast(C.c_void_p(a.data_ptr()), _lib._dp)   # noqa: E731
    req = _lib.CsrRequest(n, n, ip(off), ip(off), -1, None, ip(types), dp(x), None, 0, None,
                          None, None, None)
    with MTPGpuDirect(model_l16, 0) as gpu:
        with pytest.raises(MTPBError) as ei:
            _check(gpu.lib.mtpb_efs_csr_noalloc(gpu.ctx, C.byref(req)))
    assert ei.value.status == 1 and "limit" in str(ei.value)
