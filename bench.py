"""Benchmark of the MTP energy/force/stress path (BASELINE.json metric
"MTP EFS atoms/sec (1M-atom, level 20)").

Workload (configs[2] of BASELINE.json): 1,048,576-atom Ni3Al L1_2 box (64^3
fcc cells, a = 3.52 A, Gaussian sigma 0.08 A, seed 3), level-20 MTP
(Shapeev level-20 graph, 2 species, R = 8, r_cut = 5 A, seeded U(-0.1, 0.1)
coefficients), MD-style EFS steps: the positions move every step (seeded
displacement fields, any two steps within skin/2), the GPU neighbour lists are
built with a 0.5 A skin every 10 steps, and the steps between upload the new
positions and recompute every edge vector from the stored periodic images.  Synthetic seeded data; the working set
(~6 GB) is far larger than the 126 MB L2, so no L2 flush is needed.

The same line carries a "train" object for the second half of the metric,
"train configs/sec": config 4 of BASELINE.json, 8192 Ni/Al fcc/bcc supercells
of 64-216 atoms (seed 4), a seeded level-24 student MTP (generated basis, see
mtpb200/basisgen.py) fitted to labels of a seeded level-24 teacher plus
Gaussian noise (1 meV/atom on E/N, 10 meV/A per force component, 0.1 GPa per
stress component as virial), weights E 1, F 0.01, S 0.001 with the reference's
default powers.  One step = loss and coefficient gradient over all 8192
configurations (EFS pass, loss, gradient kernels, reductions).

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
Multi-GPU: launched by torch.distributed.run, one rank per GPU; the box is
split into x-slabs, one per rank, each with ghost layers of r_c + skin from
its two neighbours (mtpb200/slab.py): every step exchanges the halo positions
with grouped ncclSend/ncclRecv, evaluates the rank's owned centres over owned
and ghost atoms, returns the ghost forces to their owners and all-reduces
energy and virial; atoms migrate between slabs at rebuilds (strong scaling:
total atoms of the one box per second).  The training leg shards the 8192
configurations over the ranks and sums loss, metrics and gradient with an
NCCL all-reduce (strong scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "imr-mlp_b200"))
MODEL = os.path.join(ROOT, "tests", "golden", "models", "l20_k2.mtp")
METRIC = "MTP EFS atoms/sec (1M-atom, level 20)"
UNIT = "atoms/s"
REBUILD_EVERY = 10
SKIN = 0.5             # neighbour-list skin, Angstrom
N_DISP = 4             # seeded per-step displacement fields, cycled
DISP_AMPLITUDE = 0.07  # Angstrom per component: two steps differ by < skin / 2
DISP_SEED = 31
TRAIN_METRIC = "MTP train configs/sec (config 4: 8192 configs of 64-216 atoms, level 24)"
TRAIN_UNIT = "configs/s"
TRAIN_WEIGHTS = (1.0, 0.01, 0.001, 1.0, 0.0, 1.0)   # E, F, S and the default powers
EV_PER_GPA_A3 = 1.0 / 160.21766208                    # 1 GPa * 1 A^3 in eV

# DRAM traffic (read + write) per atom of each kernel, from the ncu captures
# summarised in profiles/ncu_moments_graph_config3-131k_l20.md (forward and
# graph) and profiles/ncu_moments_rev_active_config3-md-131k_l20.md (the
# reverse kernel's active-edge variant that the skin of the MD steps selects);
# 131,072 atoms, scaled by atoms
NCU_TRAFFIC_BYTES_PER_ATOM = {"k_moments<fwd>": (179.81e6 + 255.75e6) / 131072,
                              "k_dag": (310.19e6 + 263.53e6) / 131072,
                              "k_moments<rev>": (672.31e6 + 180.24e6) / 131072}
SMEM_BYTES_PER_SM_CLOCK = 128   # shared-memory bandwidth of an SM (nominal)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--reps", type=int, default=64, help="fcc cells per box edge")
    ap.add_argument("--ref-reps", type=int, default=10,
                    help="box edge (cells) of the bounded CPU sample")
    ap.add_argument("--train-configs", type=int, default=8192)
    ap.add_argument("--train-steps", type=int, default=5)
    ap.add_argument("--train-warmup", type=int, default=3)
    ap.add_argument("--no-train", action="store_true", help="skip the training leg")
    ap.add_argument("--no-batch", action="store_true",
                    help="skip the batched-EFS legs (configs 2 and 5)")
    ap.add_argument("--profile-train", action="store_true",
                    help="training leg only, device loop only (the command used for ncu "
                         "captures of the gradient kernels)")
    ap.add_argument("--profile", action="store_true",
                    help="device loop only (no e2e loop, peak probe or CPU baseline): the "
                         "command used for ncu captures")
    return ap.parse_args()


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def fp64_peak_tflops(torch, device) -> float:
    """Measured FP64 throughput of cuBLAS DGEMM (torch.matmul, float64,
    8192^3), best of 5: the FP64 peak denominator."""
    n = 8192
    a = torch.randn(n, n, dtype=torch.float64, device=device)
    b = torch.randn(n, n, dtype=torch.float64, device=device)
    for _ in range(2):
        torch.matmul(a, b)
    torch.cuda.synchronize()
    best = 1e30
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch.matmul(a, b)
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e) / 1e3)
    del a, b
    torch.cuda.empty_cache()
    return 2.0 * n ** 3 / best / 1e12


# ---------------------------------------------------------------------------
# Algorithmic FLOPs (FMA = 2, add/mul/div/sqrt = 1) of the factorised
# formulation the kernels execute, counted per valid edge and per atom from
# the model's basis shape.  Numbers per kernel:
#   fwd  staging (distance, Chebyshev recurrence, f_mu) + chains (monomial
#        products and one FMA per basic moment)
#   rev  staging (+ f'_mu) + chains (P, P', Horner value/derivative, chain
#        epilogue) + per-edge force assembly
#   dag  three FLOPs per real record (product and accumulate)
# and the reference-formulation count of the survey (per atom
#   n_e (64 + 4 mu R + 4 nu_max + 1 + 38 nb + 24) + 11 T + 2 S + 1).
# ---------------------------------------------------------------------------
def shape_chains(numax):
    NU = max(numax)

    def cnt(nu):
        return sum(1 for v in numax if v >= nu)

    chains = []
    for s in range(NU + 1):
        for b in range(s, -1, -1):
            c = s - b
            L = NU - s + 1
            chains.append((b, c, L, [cnt(a + s) for a in range(L)]))
    return chains


def flop_model(model, nmu_used, edges_per_atom, dag_records):
    numax = model.basis_shape()
    numax = [v for v in numax if v >= 0]
    R = model.rb_size
    chains = shape_chains(numax)
    stage_f = 25 + 8 * max(R - 2, 0) + 2 * R * nmu_used
    stage_r = stage_f + 2 * R * nmu_used
    fwd = 0
    rev = 0
    for b, c, L, cnts in chains:
        base = 1 if (b and c) else 0
        fwd += base + (L - 1) + 2 * sum(cnts)
        rev += base + sum(2 * (2 * k - 1) for k in cnts) + 6 * (L - 1) + 4
        rev += (3 if b else 0) + (3 if c else 0) + 5
    fwd += 16                  # y, z power tables
    rev += 16 + 11             # power tables, force assembly
    per_edge_fwd = stage_f + fwd
    per_edge_rev = stage_r + rev
    nb = model.alpha_index_basic_count
    T = model.alpha_index_times_count
    S = model.alpha_scalar_moments
    mu = model.radial_func_count
    ref = edges_per_atom * (16 + 8 * (R - 2) + 4 * mu * R + 4 * max(numax) + 1 + 38 * nb + 24) \
        + 11 * T + 2 * S + 1
    return {"fwd_per_atom": per_edge_fwd * edges_per_atom,
            "rev_per_atom": per_edge_rev * edges_per_atom,
            "dag_per_atom": 3.0 * dag_records,
            "ref_formulation_per_atom": ref}


def dag_record_count(model):
    """Real (non-padding) records of the graph program (host-only query)."""
    import ctypes as C
    import mtpb200
    from mtpb200 import _ModelKeep
    lib = mtpb200.library()
    keep = _ModelKeep(model)
    n = C.c_long()
    if lib.mtpb_graph_program(C.byref(keep.view), None, None, None, None, None, None, None,
                              None, C.byref(n), None):
        return 0
    recs = np.zeros((n.value, 4), np.uint32)
    lib.mtpb_graph_program(C.byref(keep.view), None, None, None, None, None, None, None, None,
                           None, recs.ctypes.data_as(C.POINTER(C.c_uint)))
    pad = (recs[:, 2] == 0) & (recs[:, 3] == 0) & ((recs[:, 1] >> 16) == 0)
    return int((~pad).sum())


def cpu_reference_sample(model, reps, steps, warmup, threads):
    """Reference CPU path (compiled reference Neighborhoods + MLIPCore::compute
    over OpenMP) on a bounded periodic sample of the same box; atoms/s with a
    neighbour rebuild every REBUILD_EVERY steps (the build time amortised)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import ReferenceEFS  # test infrastructure: baseline leg only
    from mtpb200 import configs, format_mtp
    st = configs.config3(reps=reps)
    ref = ReferenceEFS(format_mtp(model), model.species_count, threads=threads)
    t0 = time.perf_counter()
    prob = ref.build(st["cell"], st["pbc"], st["positions"], st["types"])
    t_build = time.perf_counter() - t0
    for _ in range(warmup):
        ref.compute(prob)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        ref.compute(prob)
        times.append(time.perf_counter() - t0)
    ref.close()
    t_step = statistics.median(times) + t_build / REBUILD_EVERY
    n = len(st["types"])
    return {"value": n / t_step, "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": f"{n}-atom Ni3Al box ({reps}^3 fcc cells, sigma 0.08), level 20; "
                      f"median of {steps} EFS evaluations after {warmup} warm-up, plus 1/"
                      f"{REBUILD_EVERY} of one neighbour build ({t_build * 1e3:.1f} ms); "
                      "MPI unavailable, OpenMP only",
            "ms_per_step": t_step * 1e3}


# ---------------------------------------------------------------------------
# Batched EFS workloads (configs 2 and 5)
# ---------------------------------------------------------------------------
BATCH_STEPS = 5


def batch_problem(name):
    """(structures, model, description) of a batched-EFS configuration."""
    from mtpb200 import configs, read_mtp
    if name == "config2":
        model = read_mtp(os.path.join(ROOT, "tests", "golden", "models", "l20_k3.mtp"))
        return (configs.config2(4096, seed=2), model,
                "config 2: 4096 Ni/Al/Cr fcc alloys of 32/108/256 atoms, level 20, K=3")
    model = configs.level24_model(species_count=3, rmin=0.8, rmax=6.0, rb_size=10, seed=55)
    return (configs.config5(1000, seed=5), model,
            "config 5: 1000 Ru(0001)/water interfaces of 336 atoms, level-24 generated basis, "
            "K=3, R=10, r_cut=6")


def cpu_batch_sample(model, sts, threads, n_sample):
    """Reference CPU path per structure (Neighborhoods build + MLIPCore over
    OpenMP centres), the calc_efs loop, on the first n_sample structures."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import ReferenceEFS  # test infrastructure: baseline leg only
    from mtpb200 import format_mtp
    ref = ReferenceEFS(format_mtp(model), model.species_count, threads=threads)
    t_total = 0.0
    atoms = 0
    for x in sts[:n_sample]:
        t0 = time.perf_counter()
        prob = ref.build(x["cell"], x["pbc"], x["positions"], x["types"])
        ref.compute(prob)
        t_total += time.perf_counter() - t0
        atoms += len(x["types"])
    ref.close()
    n = min(n_sample, len(sts))
    return {"value": n / t_total, "unit": "configs/s", "cores": threads, "kind": "reference",
            "sample": f"first {n} structures ({atoms} atoms): reference Neighborhoods + "
                      "MLIPCore::compute (OpenMP over centres) per structure",
            "atoms_per_s": atoms / t_total}


def run_batch(name, args, torch, dist, ws, rank, local, dev, stream):
    """Batched EFS of one configuration: structures sharded over the ranks
    (no data-path collective; one all-reduce of the energy total per step),
    neighbour lists built every step as a calc_efs pass does."""
    from mtpb200 import MTPGpuDirect, StructureBatch
    from mtpb200.shards import shard_lpt, shard_of
    sts, model, desc = batch_problem(name)
    sizes = [len(x["types"]) for x in sts]
    owner = shard_lpt(sizes, ws)
    mine, _ = shard_of(sts, owner, rank)
    b = StructureBatch.from_structures(mine)
    gpu = MTPGpuDirect(model, local)
    gpu.set_stream(stream.cuda_stream)
    S, N = b.n_structures, b.n_atoms
    t = {k: torch.from_numpy(v).to(dev) for k, v in
         dict(off=b.atom_offsets, cells=b.cells, pbc=np.ones((S, 3), np.int32),
              pos=b.positions, types=b.types).items()}
    e_d = torch.zeros(S, dtype=torch.float64, device=dev)
    f_d = torch.zeros((N, 3), dtype=torch.float64, device=dev)
    s_d = torch.zeros((S, 9), dtype=torch.float64, device=dev)
    tot = torch.zeros(1, dtype=torch.float64, device=dev)

    def step():
        gpu.efs_device(t["off"], t["cells"], t["pbc"], t["pos"], t["types"], e_d, f_d, s_d)
        if ws > 1:
            torch.sum(e_d, dim=0, keepdim=True, out=tot)
            dist.all_reduce(tot)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    t0.record(stream)
    for _ in range(BATCH_STEPS):
        step()
        launches += gpu.last_launch_count()
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if ws > 1:
        m = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
    km = gpu.last_timings()
    edges = gpu.neighbor_count()
    gpu.close()
    if rank != 0:
        return None
    total = len(sts)
    res = {"metric": f"MTP batched EFS configs/sec ({name})", "value": total * BATCH_STEPS /
           (ms / 1e3), "unit": "configs/s", "atoms_per_s": sum(sizes) * BATCH_STEPS / (ms / 1e3),
           "n_gpus": ws, "steps": BATCH_STEPS, "warmup": 3, "ms_per_step": ms / BATCH_STEPS,
           "scaling": "strong", "dtype": "f64",
           "config": {"workload": desc + "; one step = neighbour build and EFS of every "
                                         "structure", "structures_per_gpu": S,
                      "atoms_per_gpu": N, "edges_per_gpu": edges,
                      "parallelism": f"shards{ws} (LPT by atoms)" if ws > 1 else "single"},
           "kernel_ms": {"neighbor_build": float(km[0]), "moments_fwd": float(km[1]),
                         "graph": float(km[2]), "moments_rev": float(km[3]),
                         "gather_reduce": float(km[4])},
           "gpu_launches": int(launches)}
    return res, (model, sts)


# ---------------------------------------------------------------------------
# Training workload (config 4)
# ---------------------------------------------------------------------------
def train_problem(n_configs):
    from mtpb200 import configs
    sts = configs.config4_structures(n_configs, seed=4)
    teacher = configs.level24_model(seed=41)
    student = configs.level24_model(seed=42)
    return sts, teacher, student


def noisy_labels(sts, energy, forces, stress, seed=44):
    """Teacher outputs plus Gaussian noise: 1 meV/atom on E/N, 10 meV/A per
    force component, 0.1 GPa per stress component (virial = sigma V)."""
    rng = np.random.default_rng(seed)
    n = np.array([len(s["types"]) for s in sts], dtype=np.float64)
    vol = np.array([abs(np.linalg.det(s["cell"])) for s in sts])
    te = energy + rng.normal(0.0, 1e-3, len(sts)) * n
    tf = forces + rng.normal(0.0, 0.01, forces.shape)
    ts = stress.reshape(-1, 9) + rng.normal(0.0, 0.1, (len(sts), 9)) * \
        (vol * EV_PER_GPA_A3)[:, None]
    return te, np.ascontiguousarray(tf), np.ascontiguousarray(ts)


def _cpu_train_worker(job):
    """One process of the CPU training baseline: loss and gradient of a shard
    with the C restatement (oracle port), neighbour lists built untimed."""
    model, sts, te, tf, ts = job
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "imr-mlp_b200"))
    from oracle import Oracle, concat_lists  # test infrastructure: baseline leg only
    from mtpb200 import configs
    O = Oracle()
    offs, _, _, _, types = configs.batch(sts)
    nl = concat_lists([O.neighbors(s["cell"], s["pbc"], s["positions"], model.cutoff)
                       for s in sts], offs)
    t0 = time.perf_counter()
    loss, metrics, grad = O.loss_grad(model, offs, types, nl, te, tf, ts, TRAIN_WEIGHTS)
    return time.perf_counter() - t0, loss, grad


def cpu_train_sample(student, sts, labels, threads, per_worker=8):
    """Oracle port of the reference trainer's loss and gradient over a bounded
    sample (per_worker configurations on each of `threads` spawned
    processes); configs/s = sample size / slowest worker."""
    import concurrent.futures as cf
    import multiprocessing as mp
    te, tf, ts = labels
    n = min(len(sts), per_worker * threads)
    offs = np.cumsum([0] + [len(s["types"]) for s in sts[:n]])
    jobs = []
    for w in range(threads):
        idx = list(range(w * per_worker, min(n, (w + 1) * per_worker)))
        if not idx:
            break
        jobs.append((student, [sts[i] for i in idx], te[idx],
                     np.concatenate([tf[offs[i]:offs[i + 1]] for i in idx]), ts[idx]))
    with cf.ProcessPoolExecutor(max_workers=len(jobs),
                                mp_context=mp.get_context("spawn")) as ex:
        res = list(ex.map(_cpu_train_worker, jobs))
    slowest = max(r[0] for r in res)
    atoms = int(offs[n])
    return {"value": n / slowest, "unit": TRAIN_UNIT, "cores": len(jobs), "kind": "port",
            "sample": f"{n} config-4 structures ({atoms} atoms), level-24 student, oracle port "
                      f"of AddLossGard + AccumulateEFSCombinationGard, {len(jobs)} processes "
                      f"x {per_worker} configs; slowest process {slowest:.2f} s",
            "ms_per_config": slowest / per_worker * 1e3}


def train_flops(model, edges_per_atom, records):
    """Executed FLOPs per atom of the gradient kernels (FMA = 2)."""
    numax = [v for v in model.basis_shape() if v >= 0]
    nmu, R = len(numax), model.rb_size
    chains = shape_chains(numax)
    stage = 25 + 8 * max(R - 2, 0) + 4 * R * nmu + 20 + nmu
    tan = edge = 0
    for b, c, L, cnts in chains:
        tan += 6 + 4 * (L - 1) + 4 * sum(cnts)
        edge += 6 + 4 * (L - 1) + 6 * sum(cnts)
    return {"tangent_per_atom": (stage + tan) * edges_per_atom,
            "edge_per_atom": (35 + edge) * edges_per_atom,
            "dual_graph_per_atom": 8.0 * records,
            "radial_per_atom": (4 * R + 4 * R * nmu) * edges_per_atom}


def train_ref_flops(model, edges, atoms, configs_count):
    """Reference-formulation FLOPs of one loss-and-gradient pass (the survey's
    count: per atom n_e (64 + 4 mu R + 4 nu_max + 1 + 38 nb + 24) + 11 T + 2 S
    + 1 for EFS and n_e (23 nb + 29 + 4 mu R) + 15 T + 3 S + 1 for the
    gradient, 12 N + 40 per configuration for the loss), for this rank."""
    R, mu = model.rb_size, model.radial_func_count
    nb, T, S = (model.alpha_index_basic_count, model.alpha_index_times_count,
                model.alpha_scalar_moments)
    numax = max(v for v in model.basis_shape() if v >= 0)
    ne = edges / max(atoms, 1)
    per_atom = (ne * (16 + 8 * (R - 2) + 4 * mu * R + 4 * numax + 1 + 38 * nb + 24)
                + 11 * T + 2 * S + 1 + ne * (23 * nb + 29 + 4 * mu * R) + 15 * T + 3 * S + 1)
    return per_atom * atoms + 12 * atoms + 40 * configs_count


def run_train(args, torch, dist, ws, rank, local, dev, stream):
    """Training leg on every rank; returns the JSON object on rank 0."""
    from mtpb200 import MTPGpuDirect, StructureBatch
    from mtpb200.shards import allreduce_loss_grad, shard_lpt, shard_of
    sts, teacher, student = train_problem(args.train_configs)
    owner = shard_lpt([len(x["types"]) for x in sts], ws)   # whole structures, balanced
    mine, _ = shard_of(sts, owner, rank)
    batch = StructureBatch.from_structures(mine)
    with MTPGpuDirect(teacher, local) as tg:   # labels (untimed)
        e, f, st, _ = tg.efs(batch)
    te, tf, ts = noisy_labels(mine, e, f, st)
    gpu = MTPGpuDirect(student, local)
    gpu.set_stream(stream.cuda_stream)
    gpu.build_neighbors(batch)
    ncoef = student.coeff_count
    te_d, tf_d, ts_d = (torch.from_numpy(a).to(dev) for a in (te, tf, ts))
    out = torch.zeros(8 + ncoef, dtype=torch.float64, device=dev)
    loss_d, metrics_d, grad_d = out[0:1], out[1:8], out[8:]
    total = len(sts)

    def step():
        gpu.loss_grad_device(te_d, tf_d, ts_d, loss_d, metrics_d, grad_d, TRAIN_WEIGHTS,
                             norm_count=total)
        if ws > 1:
            allreduce_loss_grad(dist, out)

    for _ in range(args.train_warmup):
        step()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    t0.record(stream)
    for _ in range(args.train_steps):
        step()
        launches += gpu.last_launch_count() + (1 if ws > 1 else 0)
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if ws > 1:
        dist.barrier()
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tms = gpu.last_train_timings()
    ems = gpu.last_timings()
    loss = float(loss_d.item())
    # end to end through the host API: labels H2D and loss/metrics/gradient
    # D2H every step (single GPU only: the shards' sum needs the device path)
    e2e = None
    if ws == 1 and not args.profile_train:
        for _ in range(2):
            gpu.loss_grad(te, tf, ts, TRAIN_WEIGHTS, total)
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        for _ in range(args.train_steps):
            gpu.loss_grad(te, tf, ts, TRAIN_WEIGHTS, total)
        h_ms = (time.perf_counter() - h0) * 1e3
        e2e = {"value": total * args.train_steps / (h_ms / 1e3), "unit": TRAIN_UNIT,
               "h2d_bytes_per_step": int(te.nbytes + tf.nbytes + ts.nbytes),
               "d2h_bytes_per_step": int(8 * (8 + ncoef)),
               "timer": "host wall clock around the blocking host-memory calls"}
    N = batch.n_atoms
    edges = gpu.neighbor_count()
    gpu.close()
    if rank != 0:
        return None
    recs = dag_record_count(student)
    fl = train_flops(student, edges / N, recs)
    names = {2: ("k_grad_moments<tangent>", fl["tangent_per_atom"]),
             3: ("k_dag_grad", fl["dual_graph_per_atom"]),
             4: ("k_grad_moments<edge>", fl["edge_per_atom"])}
    dom = max(names, key=lambda i: tms[i])
    kname, kflops = names[dom]
    achieved = kflops * N / (tms[dom] / 1e3) / 1e12
    res = {
        "metric": TRAIN_METRIC, "value": total * args.train_steps / (ms / 1e3),
        "unit": TRAIN_UNIT, "n_gpus": ws, "steps": args.train_steps,
        "warmup": args.train_warmup, "ms_per_step": ms / args.train_steps,
        "higher_is_better": True, "scaling": "strong", "dtype": "f64",
        "data": "synthetic (seeded config-4 structures, teacher labels plus seeded noise)",
        "config": {"workload": f"config 4: {total} configurations, level-24 generated basis "
                               f"(nb {student.alpha_index_basic_count}, T "
                               f"{student.alpha_index_times_count}, S "
                               f"{student.alpha_scalar_moments}), K=2, R=8, r_cut=5",
                   "atoms_per_gpu": N, "edges_per_gpu": edges,
                   "parallelism": f"dp{ws}" if ws > 1 else "single",
                   "weights": TRAIN_WEIGHTS, "loss": loss,
                   "l2": "working set ~25 GB per GPU, larger than L2 (no flush)"},
        "kernel_ms": {"efs_pass": float(tms[0]), "efs_moments_fwd": float(ems[1]),
                      "efs_graph": float(ems[2]), "efs_moments_rev": float(ems[3]),
                      "efs_gather_reduce": float(ems[4]), "loss_weights_buckets": float(tms[1]),
                      "tangent_moments": float(tms[2]), "dual_graph": float(tms[3]),
                      "edge_records": float(tms[4]), "radial_reduce": float(tms[5])},
        "gpu_launches": int(launches),
        "roofline": {"bound": "fp64", "kernel": kname, "achieved": achieved, "unit": "TFLOP/s",
                     "flops_per_atom": kflops,
                     # the dual graph reads two (value, tangent) operand pairs,
                     # 32 B, per real record and atom from its L2-resident rows
                     "dual_graph_operands": {
                         "bytes_per_atom": 32.0 * recs,
                         "achieved_tb_s": 32.0 * recs * N / (tms[3] / 1e3) / 1e12,
                         "peak": None,
                         "note": "L1/L2 operand read rate; no measured L2 figure"}},
        # rank 0 GPU: its shard's reference-formulation FLOPs over the pass time
        "step_tflops_ref_formulation": train_ref_flops(student, edges, N, len(mine))
        / (ms / args.train_steps / 1e3) / 1e12,
        "e2e": e2e,
    }
    return res, (student, sts, (te, tf, ts))


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist
    from mtpb200 import MTPGpuDirect, StructureBatch, configs, read_mtp

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    model = read_mtp(MODEL)
    st = configs.config3(reps=args.reps)
    N = len(st["types"])
    # MD-style steps: positions of step k are base + D[k % 4], with four
    # seeded displacement fields |D| <= DISP_AMPLITUDE per component, so any
    # two steps differ by less than skin/2 and the lists stay valid between
    # rebuilds (the reuse steps recompute every edge vector)
    rng = np.random.default_rng(DISP_SEED)
    disp = rng.uniform(-DISP_AMPLITUDE, DISP_AMPLITUDE, (N, 3 * N_DISP))
    assert 2 * DISP_AMPLITUDE * 3 ** 0.5 < SKIN / 2
    gpu = MTPGpuDirect(model, local)
    gpu.set_skin(SKIN)
    # a dedicated stream shared by the library and the timing events
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    gpu.set_stream(stream.cuda_stream)
    slab = ws > 1   # one box over all ranks: x-slabs with a ghost-atom halo
    if slab:
        from mtpb200.slab import DistributedSlab, SlabDomain, SlabEFS, halo_bytes_per_step
        D = SlabDomain(st["cell"], ws, rank, model.cutoff + SKIN, device=dev)
        D.assign(st["positions"], st["types"], payload=disp)
        S = SlabEFS(gpu, DistributedSlab(D, dist))
        base = None
        f_own = None
    else:
        batch = StructureBatch.from_structures([st])
        offs_d = torch.from_numpy(batch.atom_offsets).to(dev)
        cells_d = torch.from_numpy(batch.cells).to(dev)
        pbc_d = torch.ones((1, 3), dtype=torch.int32, device=dev)
        base_d = torch.from_numpy(batch.positions).to(dev)
        disp_d = torch.from_numpy(disp).to(dev)
        pos_d = torch.empty_like(base_d)
        types_d = torch.from_numpy(batch.types).to(dev)
        energy_d = torch.zeros(1, dtype=torch.float64, device=dev)
        forces_d = torch.zeros((N, 3), dtype=torch.float64, device=dev)
        stress_d = torch.zeros((1, 9), dtype=torch.float64, device=dev)
    totals_d = None

    def step(k):
        nonlocal base, f_own, totals_d
        j = 3 * (k % N_DISP)
        rebuild = k % REBUILD_EVERY == 0
        if slab:
            if base is not None:
                D.pos = base + D.payload[:, j:j + 3]
            if rebuild:    # migration, halo lists, then a list build
                S.rebuild()
                base = D.pos - D.payload[:, j:j + 3]
            f_own, totals_d = S.compute()
        else:
            torch.add(base_d, disp_d[:, j:j + 3], out=pos_d)
            gpu.efs_device(offs_d, cells_d, pbc_d, pos_d, types_d, energy_d, forces_d, stress_d,
                           reuse_neighbors=not rebuild)

    def barrier():
        if ws > 1:
            dist.barrier()

    def max_over_ranks(x):
        if ws == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    edges = gpu.neighbor_count()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    kernel_ms = np.zeros(5)
    t0.record(stream)
    for k in range(args.steps):
        step(k)
        launches += gpu.last_launch_count()
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = max_over_ranks(t0.elapsed_time(t1))
    halo = halo_bytes_per_step(D) if slab else None
    n_centers = D.n_own if slab else N
    n_ghost = D.n_ghost if slab else 0
    # per-kernel device time of a reuse step and of a rebuild step (events
    # recorded by the library on the same stream)
    step(1)
    torch.cuda.synchronize()
    kernel_ms = gpu.last_timings()
    step(0)
    torch.cuda.synchronize()
    build_ms = gpu.last_timings()[0]
    energy = float(totals_d[0].item()) if slab else float(energy_d.item())

    if args.profile:
        if rank == 0:
            print(json.dumps({"profile_run": True, "atoms": N, "edges": edges,
                              "ms_per_step": ms / args.steps, "energy_eV": energy}))
        if ws > 1:
            dist.destroy_process_group()
        return None
    # end-to-end through the public host API: pinned host buffers, H2D of the
    # positions every step, D2H of the energy, forces and virial every step.
    # With slabs each rank copies its owned atoms' positions in and their
    # forces and the totals out, and at a rebuild (which changes ownership)
    # reads the new owned positions back.
    n_rebuild = sum(1 for k in range(args.steps) if k % REBUILD_EVERY == 0)
    if slab:
        cap = N
        base_h = torch.zeros((cap, 3), dtype=torch.float64).pin_memory()
        f_h = torch.zeros((cap, 3), dtype=torch.float64).pin_memory()
        t_h = torch.zeros(10, dtype=torch.float64).pin_memory()
        base_h[:base.shape[0]].copy_(base)
        own_n = [base.shape[0]]

        def e2e_step(k):
            nonlocal base
            n = own_n[0]
            base = base_h[:n].to(dev, non_blocking=True)
            step(k)
            if k % REBUILD_EVERY == 0:
                own_n[0] = base.shape[0]
                base_h[:own_n[0]].copy_(base, non_blocking=True)
            f_h[:f_own.shape[0]].copy_(f_own, non_blocking=True)
            t_h.copy_(totals_d, non_blocking=True)
            stream.synchronize()

        h2d = n_centers * 24
        d2h = n_centers * 24 + 80 + n_rebuild * n_centers * 24 / args.steps
    else:
        pos_h = [torch.from_numpy(st["positions"] + disp[:, 3 * j:3 * j + 3]).pin_memory()
                 for j in range(N_DISP)]
        types_h = torch.from_numpy(batch.types).pin_memory()
        hbs = [StructureBatch(batch.atom_offsets, batch.cells, None, p.numpy(), types_h.numpy())
               for p in pos_h]
        out = {"energy": torch.zeros(1, dtype=torch.float64).pin_memory().numpy(),
               "forces": torch.zeros((N, 3), dtype=torch.float64).pin_memory().numpy(),
               "stress": torch.zeros((1, 9), dtype=torch.float64).pin_memory().numpy()}

        def e2e_step(k):
            gpu.efs_structures(hbs[k % N_DISP], reuse_neighbors=(k % REBUILD_EVERY) != 0,
                               out=out)

        h2d = (N * 24 * args.steps + n_rebuild * (N * 4 + 9 * 8 + 8)) / args.steps
        d2h = N * 24 + 8 + 72
    for k in range(args.warmup):
        e2e_step(k)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(args.steps):
        e2e_step(k)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    # both loops end on step steps-1 from the same rebuild, so the energies agree
    step_last = args.steps - 1
    e2e_energy = float(t_h[0]) if slab else float(out["energy"][0])
    step(step_last - step_last % REBUILD_EVERY)
    for k in range(step_last - step_last % REBUILD_EVERY + 1, step_last + 1):
        step(k)
    torch.cuda.synchronize()
    energy = float(totals_d[0].item()) if slab else float(energy_d.item())
    e2e_ok = abs(e2e_energy - energy) <= 1e-9 * max(1.0, abs(energy))

    train = None if args.no_train else run_train(args, torch, dist, ws, rank, local, dev, stream)
    batches = [] if args.no_batch else [run_batch(nm, args, torch, dist, ws, rank, local, dev,
                                                  stream) for nm in ("config2", "config5")]
    peak = fp64_peak_tflops(torch, dev) if rank == 0 else None
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None
    # roofline of the dominant kernel (FP64 CUDA-core bound)
    recs = dag_record_count(model)
    fm = flop_model(model, len([v for v in model.basis_shape() if v >= 0]), edges / n_centers,
                    recs)
    names = {1: ("k_moments<fwd>", fm["fwd_per_atom"]), 2: ("k_dag", fm["dag_per_atom"]),
             3: ("k_moments<rev>", fm["rev_per_atom"])}
    dom = max(names, key=lambda i: kernel_ms[i])
    kname, kflops = names[dom]
    achieved = kflops * n_centers / (kernel_ms[dom] / 1e3) / 1e12
    total_atoms = N * (1 if slab else ws) * args.steps
    value = total_atoms / (ms / 1e3)
    step_ms = float(kernel_ms[1:].sum())
    fp64_view = {"achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                 "frac": achieved / peak if peak else None, "flops_per_atom": kflops,
                 "peak_source": "measured by bench.py: cuBLAS DGEMM 8192^3 (torch.matmul "
                                "float64); MEASURED_PEAKS.json has no FP64 figure"}
    traffic = NCU_TRAFFIC_BYTES_PER_ATOM[kname] * n_centers
    if kname == "k_dag":
        # the graph kernel is bound by its shared-memory operand reads: two
        # 8-byte rows per real record and atom
        import torch as _t
        sms = _t.cuda.get_device_properties(dev).multi_processor_count
        mhz = clocks.get("sm_mhz") or 1965.0
        smem_peak = sms * SMEM_BYTES_PER_SM_CLOCK * mhz * 1e6 / 1e9
        bytes_ = 16.0 * recs * n_centers
        ach = bytes_ / (kernel_ms[dom] / 1e3) / 1e9
        roofline = {"bound": "smem", "kernel": kname, "achieved": ach, "peak": smem_peak,
                    "unit": "GB/s", "frac": ach / smem_peak, "traffic": traffic,
                    "algorithmic_bytes_per_atom": 16.0 * recs,
                    "peak_source": f"nominal shared-memory bandwidth: {sms} SMs x "
                                   f"{SMEM_BYTES_PER_SM_CLOCK} B per clock x {mhz:.0f} MHz "
                                   "(measured clock); MEASURED_PEAKS.json has no shared-memory "
                                   "figure",
                    "traffic_source": "ncu dram__bytes_read+write of the 131k-atom capture, "
                                      "scaled by atoms",
                    "fp64": fp64_view}
    else:
        roofline = dict(fp64_view, bound="fp64", kernel=kname, traffic=traffic)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded Ni3Al L1_2 box, seeded level-20 coefficients, seeded "
                "per-step displacements)",
        "config": {"workload": f"config 3: {N}-atom Ni3Al box, level-20 MTP, MD-style EFS "
                               f"steps (positions move every step by seeded displacements, "
                               f"neighbour lists with a {SKIN} A skin rebuilt every "
                               f"{REBUILD_EVERY} steps, every edge vector recomputed on the "
                               "steps between)"
                               + (f"; one box over {ws} GPUs in x-slabs with ghost layers of "
                                  f"r_c + skin: per step a grouped P2P exchange of halo "
                                  "positions, EFS of the owned atoms, reverse exchange of "
                                  "ghost forces, all-reduce of energy and virial; atoms "
                                  "migrate between slabs at rebuilds" if slab else ""),
                   "atoms_per_gpu": n_centers, "ghost_atoms_per_gpu": n_ghost,
                   "edges_per_gpu": edges, "level": 20,
                   "species": 2, "rb_size": 8, "r_cut": 5.0, "skin": SKIN,
                   "displacement": f"{N_DISP} seeded fields U(-{DISP_AMPLITUDE}, "
                                   f"{DISP_AMPLITUDE}) A per component, cycled (seed "
                                   f"{DISP_SEED}); any two steps differ by < skin/2",
                   "parallelism": f"slab{ws}" if slab else "single",
                   "halo_bytes_per_step_rank0": halo,
                   "l2": "working set ~6 GB per GPU, larger than L2 (no flush)"},
        "e2e": {"value": total_atoms / (e2e_ms / 1e3), "unit": UNIT,
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "matches_device_energy": e2e_ok},
        "gpu_launches": int(launches),
        "roofline": roofline,
        "kernel_ms": {"refresh": float(kernel_ms[0]), "neighbor_build": float(build_ms),
                      "moments_fwd": float(kernel_ms[1]), "graph": float(kernel_ms[2]),
                      "moments_rev": float(kernel_ms[3]), "gather_reduce": float(kernel_ms[4])},
        "step_tflops_executed": (fm["fwd_per_atom"] + fm["rev_per_atom"] + fm["dag_per_atom"])
        * n_centers / (step_ms / 1e3) / 1e12,
        "step_tflops_ref_formulation": fm["ref_formulation_per_atom"] * n_centers
        / (step_ms / 1e3) / 1e12,
        "clocks": clocks,
        "energy_eV": energy,
    }
    threads = os.cpu_count() or 1
    try:
        line["cpu_baseline"] = cpu_reference_sample(model, args.ref_reps, 3, 1, threads)
    except Exception as exc:   # reference build absent on this machine
        line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                                "sample": f"unavailable: {exc}"}
    if train is not None:
        tline, (student, tsts, labels) = train
        tline["roofline"]["peak"] = peak
        tline["roofline"]["frac"] = tline["roofline"]["achieved"] / peak if peak else None
        if ws == 1:
            try:
                tline["cpu_baseline"] = cpu_train_sample(student, tsts, labels, threads)
            except Exception as exc:
                tline["cpu_baseline"] = {"value": None, "unit": TRAIN_UNIT, "cores": 0,
                                         "kind": "port", "sample": f"unavailable: {exc}"}
        line["train"] = tline
    for res in batches:
        if res is None:
            continue
        bline, (bmodel, bsts) = res
        if ws == 1:
            try:
                bline["cpu_baseline"] = cpu_batch_sample(bmodel, bsts, threads, 32)
            except Exception as exc:
                bline["cpu_baseline"] = {"value": None, "unit": "configs/s", "cores": 0,
                                         "kind": "reference", "sample": f"unavailable: {exc}"}
        line.setdefault("batch", []).append(bline)
    return line


def run_reference(args):
    ws, rank, local = dist_env()
    if rank != 0:
        return None
    from mtpb200 import read_mtp
    model = read_mtp(MODEL)
    threads = os.cpu_count() or 1
    r = cpu_reference_sample(model, args.ref_reps, max(args.steps, 1), max(args.warmup, 0),
                             threads)
    train = None
    if not args.no_train:
        train = reference_train_line(args, threads, ws)
    line = {"metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded Ni3Al L1_2 box, seeded level-20 coefficients)",
            "config": {"workload": "config 3 sample: reference CPU path (Neighborhoods + "
                                   "MLIPCore::compute, OpenMP over centres) on a bounded box",
                       "parallelism": f"openmp{threads}"},
            "impl": "reference", "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores",
                                                                   "kind", "sample")},
            "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    if train is not None:
        line["train"] = train
    if not args.no_batch:
        for nm in ("config2", "config5"):
            sts, bmodel, desc = batch_problem(nm)
            r = cpu_batch_sample(bmodel, sts, threads, 32)
            line.setdefault("batch", []).append({
                "metric": f"MTP batched EFS configs/sec ({nm})", "value": r["value"],
                "unit": "configs/s", "atoms_per_s": r["atoms_per_s"], "n_gpus": ws,
                "impl": "reference", "config": {"workload": desc},
                "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": r["value"], "unit": "configs/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}})
    return line


def reference_train_line(args, threads, ws):
    """CPU training baseline for the reference arm: teacher labels from the
    oracle EFS (untimed), then the oracle port's loss and gradient on all
    host cores.  The reference's own trainer (train/train_mtp.cpp) does not
    compile here, so the port stands in for it."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle  # test infrastructure: reference arm only
    n = min(args.train_configs, 8 * threads)
    sts, teacher, student = train_problem(n)
    O = Oracle()
    es, fs, ss = [], [], []
    for x in sts:
        nl = O.neighbors(x["cell"], x["pbc"], x["positions"], teacher.cutoff)
        e, _, f, w = O.efs(teacher, x["types"], nl)
        es.append(e)
        fs.append(f)
        ss.append(w.reshape(9))
    labels = noisy_labels(sts, np.array(es), np.concatenate(fs), np.stack(ss))
    r = cpu_train_sample(student, sts, labels, threads)
    return {"metric": TRAIN_METRIC, "value": r["value"], "unit": TRAIN_UNIT, "n_gpus": ws,
            "ms_per_step": r["ms_per_config"] * args.train_configs / r["cores"],
            "higher_is_better": True, "scaling": "strong", "dtype": "f64",
            "impl": "reference", "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores",
                                                                   "kind", "sample")},
            "e2e": {"value": r["value"], "unit": TRAIN_UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def run_profile_train(args):
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    res = run_train(args, torch, None, 1, 0, 0, dev, stream)
    line = res[0]
    return {"profile_run": True, "train_ms_per_step": line["ms_per_step"],
            "kernel_ms": line["kernel_ms"], "atoms": line["config"]["atoms_per_gpu"]}


def main():
    args = parse()
    if args.profile_train:
        print(json.dumps(run_profile_train(args)), flush=True)
        return
    line = run_reference(args) if args.impl == "reference" else run_ours(args)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
