"""Reporting of a graph kernel's bounded wait that gave up (MTPB_ERR_CUDA).

The record-stream waits of the graph kernels poll their mbarrier a bounded
number of times and then set a device flag instead of hanging.  No test makes
a wait run out: the flag is set from the host (mtpb_debug_flag_device_error,
no kernel involved), and the tests check that
  * a host-memory EFS call reports MTPB_ERR_CUDA with the wait message, clears
    the flag, and the next call succeeds with the usual results;
  * device-memory calls do not read the flag, and mtpb_check_device_status
    reports and clears it once;
  * a host-memory loss/gradient call reports it as well."""
import numpy as np
import pytest

from mtpb200 import configs

pytestmark = pytest.mark.gpu


def test_host_call_reports_and_clears(model_l16):
    from mtpb200 import MTPBError, MTPGpuDirect, StructureBatch, _lib
    sts = configs.config2(3, seed=71)
    for s in sts:
        s["types"] = np.minimum(s["types"], 1).astype(np.int32)
    b = StructureBatch.from_structures(sts)
    with MTPGpuDirect(model_l16, 0) as gpu:
        e0, f0, s0, _ = gpu.efs(b)
        assert gpu.lib.mtpb_debug_flag_device_error(gpu.ctx) == _lib.MTPB_OK
        with pytest.raises(MTPBError) as err:
            gpu.efs(b)
        assert err.value.status == _lib.MTPB_ERR_CUDA
        assert "wait gave up" in str(err.value)
        e1, f1, s1, _ = gpu.efs(b)   # the flag was cleared by the report
        assert np.array_equal(e0, e1) and np.array_equal(f0, f1) and np.array_equal(s0, s1)
        gpu.check_device_status()


def test_device_calls_report_through_status_check(model_l16):
    import torch
    from mtpb200 import MTPBError, MTPGpuDirect, StructureBatch, _lib
    st = configs.config3(reps=3)
    b = StructureBatch.from_structures([st])
    dev = torch.device("cuda", 0)
    n = len(st["types"])
    args = [torch.from_numpy(b.atom_offsets).to(dev), torch.from_numpy(b.cells).to(dev),
            torch.ones((1, 3), dtype=torch.int32, device=dev),
            torch.from_numpy(b.positions).to(dev), torch.from_numpy(b.types).to(dev),
            torch.zeros(1, dtype=torch.float64, device=dev),
            torch.zeros((n, 3), dtype=torch.float64, device=dev),
            torch.zeros((1, 9), dtype=torch.float64, device=dev)]
    with MTPGpuDirect(model_l16, 0) as gpu:
        gpu.check_device_status()                      # nothing pending
        gpu.efs_device(*args)
        e0 = float(args[5].item())
        assert gpu.lib.mtpb_debug_flag_device_error(gpu.ctx) == _lib.MTPB_OK
        gpu.efs_device(*args, reuse_neighbors=True)    # device calls do not check
        with pytest.raises(MTPBError) as err:
            gpu.check_device_status()
        assert err.value.status == _lib.MTPB_ERR_CUDA
        gpu.check_device_status()                      # reported once, then clear
        gpu.efs_device(*args, reuse_neighbors=True)
        torch.cuda.synchronize()
        assert float(args[5].item()) == e0


def test_loss_grad_reports(model_l16):
    from mtpb200 import MTPBError, MTPGpuDirect, StructureBatch, _lib
    sts = configs.config2(3, seed=72)
    for s in sts:
        s["types"] = np.minimum(s["types"], 1).astype(np.int32)
    n = sum(len(s["types"]) for s in sts)
    rng = np.random.default_rng(5)
    te, tf, ts = rng.normal(size=len(sts)), rng.normal(0, 0.1, (n, 3)), rng.normal(size=(len(sts), 9))
    w = (1.0, 0.01, 0.001, 1.0, 0.0, 1.0)
    with MTPGpuDirect(model_l16, 0) as gpu:
        gpu.build_neighbors(StructureBatch.from_structures(sts))
        loss0, _, g0 = gpu.loss_grad(te, tf, ts, w)
        assert gpu.lib.mtpb_debug_flag_device_error(gpu.ctx) == _lib.MTPB_OK
        with pytest.raises(MTPBError) as err:
            gpu.loss_grad(te, tf, ts, w)
        assert err.value.status == _lib.MTPB_ERR_CUDA
        loss1, _, g1 = gpu.loss_grad(te, tf, ts, w)
        assert loss1 == loss0 and np.array_equal(g0, g1)
