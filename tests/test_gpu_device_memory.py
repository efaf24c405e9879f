"""Device-memory structures path (mtpb_efs_structures with MTPB_MEMORY_DEVICE,
the calc_efs / trainer batch pass of the benchmark): back-to-back batches
queued on one stream give bit-for-bit the host path's energies, forces and
virials, and a species index outside 0..K-1 is rejected by the device-side
check without spoiling the context."""
import numpy as np
import pytest

from mtpb200 import configs

pytestmark = pytest.mark.gpu


def _device_inputs(torch, b, dev):
    S = b.n_structures
    return {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in
            dict(off=b.atom_offsets, cells=b.cells, pbc=np.ones((S, 3), np.int32),
                 pos=b.positions, types=b.types).items()}


def test_device_batches_match_host_path(model_l20_k3):
    import torch
    from mtpb200 import MTPGpuDirect, StructureBatch
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(91)
    base = configs.config2(48, seed=91)
    batches = []
    for _ in range(3):   # same layout, moved atoms: a rebuild per batch
        sts = [dict(x, positions=x["positions"] + rng.normal(0, 0.02, x["positions"].shape))
               for x in base]
        batches.append(StructureBatch.from_structures(sts))
    with MTPGpuDirect(model_l20_k3, 0) as gpu:
        ref = [gpu.efs(b) for b in batches]
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream), MTPGpuDirect(model_l20_k3, 0) as gpu:
        gpu.set_stream(stream.cuda_stream)
        outs = []
        inputs = [_device_inputs(torch, b, dev) for b in batches]
        stream.synchronize()
        for b, t in zip(batches, inputs):   # queued without host synchronisation
            S, N = b.n_structures, b.n_atoms
            o = dict(e=torch.zeros(S, dtype=torch.float64, device=dev),
                     f=torch.zeros((N, 3), dtype=torch.float64, device=dev),
                     s=torch.zeros((S, 9), dtype=torch.float64, device=dev))
            gpu.efs_device(t["off"], t["cells"], t["pbc"], t["pos"], t["types"],
                           o["e"], o["f"], o["s"])
            outs.append(o)
        stream.synchronize()
        for (e, f, s, _), o in zip(ref, outs):
            assert np.array_equal(o["e"].cpu().numpy(), e)
            assert np.array_equal(o["f"].cpu().numpy(), f)
            assert np.array_equal(o["s"].cpu().numpy().reshape(-1, 3, 3), s)


def test_species_outside_range_rejected(model_l16):
    from mtpb200 import MTPBError, MTPGpuDirect, StructureBatch
    st = configs.config1()
    bad = dict(st, types=st["types"].copy())
    bad["types"][5] = model_l16.species_count      # one past the last species
    bad["types"][9] = -1
    with MTPGpuDirect(model_l16, 0) as gpu:
        with pytest.raises(MTPBError) as exc:
            gpu.efs(StructureBatch.from_structures([bad]))
        assert exc.value.status == 1 and "atom 5 " in str(exc.value)
        e_ok, f_ok, _, _ = gpu.efs(StructureBatch.from_structures([st]))
    with MTPGpuDirect(model_l16, 0) as gpu:
        e_ref, f_ref, _, _ = gpu.efs(StructureBatch.from_structures([st]))
    assert np.array_equal(e_ok, e_ref) and np.array_equal(f_ok, f_ref)
