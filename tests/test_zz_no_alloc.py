"""mtpb_efs_csr_noalloc, the entry point for callers that cannot allocate
device memory while they run (an MD engine or plug-in host that has already
claimed the GPU's memory for its own pool, or a real-time loop that must not
enter the allocator).  Its scratch lives in a fixed array inside the library,
so it is compared here with the allocating CSR entry point on the same device
inputs, twice in a row with different systems (the array keeps the previous
call's contents).  Collected last so that a failure here leaves the rest of
the suite already run."""
import ctypes as C

import numpy as np
import pytest

from conftest import load_model
from mtpb200 import configs

pytestmark = pytest.mark.gpu

TOL_E_ATOM = 1e-10
TOL_F = 1e-9
TOL_W = 1e-9


def _problem(oracle, model, st):
    """Periodic structure as a CSR request with explicit edge vectors."""
    nl = oracle.neighbors(st["cell"], st["pbc"], st["positions"], model.cutoff)
    return dict(offsets=nl.offsets.astype(np.int32), neighbors=nl.nbr.astype(np.int32),
                vectors=np.ascontiguousarray(nl.rij), types=st["types"].astype(np.int32),
                x=oracle.wrap(st["cell"], st["pbc"], st["positions"]))


def _run(gpu, prob, noalloc, torch):
    from mtpb200 import _lib, _check
    dev = torch.device("cuda", 0)
    t = {k: torch.from_numpy(v).to(dev) for k, v in prob.items()}
    n = len(prob["types"])
    out = dict(force=torch.zeros((n, 3), dtype=torch.float64, device=dev),
               energy=torch.zeros(1, dtype=torch.float64, device=dev),
               site_energy=torch.zeros(n, dtype=torch.float64, device=dev),
               site_virial=torch.zeros((n, 6), dtype=torch.float64, device=dev),
               virial=torch.zeros(6, dtype=torch.float64, device=dev))
    dp = lambda a: C.cast(C.c_void_p(a.data_ptr()), _lib._dp)   # noqa: E731
    ip = lambda a: C.cast(C.c_void_p(a.data_ptr()), _lib._ip)   # noqa: E731
    req = _lib.CsrRequest(n, n, ip(t["offsets"]), ip(t["neighbors"]), -1, dp(t["vectors"]),
                          ip(t["types"]), dp(t["x"]), dp(out["force"]), 0, dp(out["energy"]),
                          dp(out["site_energy"]), dp(out["site_virial"]), dp(out["virial"]))
    torch.cuda.synchronize()
    if noalloc:
        _check(gpu.lib.mtpb_efs_csr_noalloc(gpu.ctx, C.byref(req)))
    else:
        _check(gpu.lib.mtpb_efs_csr(gpu.ctx, C.byref(req), _lib.MEMORY_DEVICE))
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in out.items()}


def test_noalloc_matches_allocating_entry_point_twice(oracle, model_l16):
    torch = pytest.importorskip("torch")
    from mtpb200 import MTPGpuDirect
    first = configs.config1()
    second = configs.config2(1, seed=55)[0]
    second["types"] = np.minimum(second["types"], 1).astype(np.int32)
    with MTPGpuDirect(model_l16, 0) as gpu:
        for st in (first, second):
            prob = _problem(oracle, model_l16, st)
            ref = _run(gpu, prob, False, torch)
            got = _run(gpu, prob, True, torch)
            n = len(prob["types"])
            assert abs(got["energy"][0] - ref["energy"][0]) / n < TOL_E_ATOM
            assert np.max(np.abs(got["site_energy"] - ref["site_energy"])) < TOL_E_ATOM
            assert np.max(np.abs(got["force"] - ref["force"])) < TOL_F
            assert np.max(np.abs(got["virial"] - ref["virial"])) < TOL_W
            assert np.max(np.abs(got["site_virial"] - ref["site_virial"])) < TOL_W
            assert np.max(np.abs(ref["force"])) > 0


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
