// noalloc.cu -- mtpb_efs_csr_noalloc: the CSR energy/force/virial request for
// small systems, with every per-call scratch buffer carved out of one
// file-scope device array instead of device allocations.
//
// Some callers cannot allocate device memory while they run: code inside a
// memory pool or budget owned by a host application (an MD engine that has
// already reserved the GPU memory), real-time loops that must not hit the
// allocator, or plug-ins whose host forbids cudaMalloc after start-up.  This
// entry point serves them: it calls no cudaMalloc/cudaFree and no allocating
// library routine.  The scratch array (g_noalloc_scratch below, a fixed size
// of about 9.6 MB) is part of the library image and stays resident on every
// GPU that loads the library until the process exits.
#include "context.hpp"

#include <mutex>

namespace mtpb {

// Limits of the no-allocation path (the scratch array is sized for them).
constexpr int NOALLOC_MAX_CENTERS = 1024;
constexpr int NOALLOC_MAX_ATOMS = 4096;     // centres + ghosts
constexpr long NOALLOC_MAX_EDGES = 65536;
constexpr int NOALLOC_MAX_SLOTS = 320;      // basic-moment slots of the kernel shape
constexpr int NOALLOC_MAX_SEGMENTS = (NOALLOC_MAX_ATOMS + 1023) / 1024;

// byte layout of the scratch array (all offsets 256-byte aligned)
constexpr size_t al256(size_t x) { return (x + 255) / 256 * 256; }
constexpr size_t NA_BASIC = 0;
constexpr size_t NA_ADJ = NA_BASIC + al256(8ull * NOALLOC_MAX_SLOTS * NOALLOC_MAX_CENTERS);
constexpr size_t NA_RX = NA_ADJ + al256(8ull * NOALLOC_MAX_SLOTS * NOALLOC_MAX_CENTERS);
constexpr size_t NA_RY = NA_RX + al256(8ull * NOALLOC_MAX_EDGES);
constexpr size_t NA_RZ = NA_RY + al256(8ull * NOALLOC_MAX_EDGES);
constexpr size_t NA_DX = NA_RZ + al256(8ull * NOALLOC_MAX_EDGES);
constexpr size_t NA_DY = NA_DX + al256(8ull * NOALLOC_MAX_EDGES);
constexpr size_t NA_DZ = NA_DY + al256(8ull * NOALLOC_MAX_EDGES);
constexpr size_t NA_NBR = NA_DZ + al256(8ull * NOALLOC_MAX_EDGES);
constexpr size_t NA_IN_EDGES = NA_NBR + al256(4ull * NOALLOC_MAX_EDGES);
constexpr size_t NA_IN_COUNT = NA_IN_EDGES + al256(4ull * NOALLOC_MAX_EDGES);
constexpr size_t NA_IN_OFF = NA_IN_COUNT + al256(4ull * (NOALLOC_MAX_ATOMS + 1));
constexpr size_t NA_IN_CURSOR = NA_IN_OFF + al256(4ull * (NOALLOC_MAX_ATOMS + 1));
constexpr size_t NA_MAXDEG = NA_IN_CURSOR + al256(4ull * (NOALLOC_MAX_ATOMS + 1));
constexpr size_t NA_SITE_E = NA_MAXDEG + al256(4ull * (NOALLOC_MAX_CENTERS / 32 + 1));
constexpr size_t NA_SITE_E_ALL = NA_SITE_E + al256(8ull * NOALLOC_MAX_CENTERS);
constexpr size_t NA_FORCE = NA_SITE_E_ALL + al256(8ull * NOALLOC_MAX_ATOMS);
constexpr size_t NA_VROWS = NA_FORCE + al256(24ull * NOALLOC_MAX_ATOMS);
constexpr size_t NA_SEGS = NA_VROWS + al256(72ull * NOALLOC_MAX_ATOMS);
constexpr size_t NA_PARTIALS = NA_SEGS + al256(4ull * (2 * NOALLOC_MAX_SEGMENTS + 2));
constexpr size_t NA_SUMS = NA_PARTIALS + al256(80ull * NOALLOC_MAX_SEGMENTS);
constexpr size_t NA_CHECK = NA_SUMS + al256(8ull * 20);
constexpr size_t NA_TOTAL = NA_CHECK + al256(4ull * 8);

// The scratch array.  In host code this name is only a host-side stand-in:
// its device address comes from cudaGetSymbolAddress (scratch_base below).
static __device__ __align__(256) unsigned char g_noalloc_scratch[NA_TOTAL];

// Device address of the array, looked up once per device with that device
// current (the first call on a device does it; make that first call before
// any stream capture).
static std::mutex g_noalloc_mutex;
static void *g_noalloc_addr[128] = {};

static int scratch_base(int device, unsigned char **base)
{
    if (device < 0 || device >= 128)
        return fail(MTPB_ERR_ARGUMENT, "device index out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_addr[device]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess)
            return cuda_fail(e, "cudaGetSymbolAddress(no-allocation scratch)");
        g_noalloc_addr[device] = p;
    }
    *base = static_cast<unsigned char *>(g_noalloc_addr[device]);
    return MTPB_OK;
}

static inline int nblk_na(long n, int t) { return (int)((n + t - 1) / t); }

// Input validation of a request, run before any kernel indexes with its
// contents (the same checks mtpb_efs_csr makes on the host).  status[0..4]
// start at NA_CHECK_NONE and receive the smallest offending position:
// [0] offsets[0] != 0 (0), [1] first i with offsets[i+1] < offsets[i],
// [2] first edge whose masked neighbour index is outside [0, ntotal),
// [3] first atom whose type is outside [-1, K), [4] edge count above the limit;
// status[5] = offsets[center_count].  Neighbour indices are only read when the
// edge count is within [0, NOALLOC_MAX_EDGES] and the array is present (a
// request without centres may pass none; its nonzero offsets[0] is reported).
// The host clears the status words with the byte 0x7f, so "none" reads
// 0x7f7f7f7f, larger than any index a request can hold.
constexpr int NA_CHECK_NONE = 0x7f7f7f7f;

__global__ void k_na_validate(int NC, int NT, const int *__restrict__ offsets,
                              const int *__restrict__ nbr_in, int mask,
                              const int *__restrict__ types, int K, int *__restrict__ status)
{
    const int E = offsets[NC];
    const bool e_ok = E >= 0 && E <= NOALLOC_MAX_EDGES && (E == 0 || nbr_in);
    const long stride = (long)gridDim.x * blockDim.x;
    const long t0 = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t0 == 0) {
        status[5] = E;
        if (offsets[0] != 0)
            atomicMin(status + 0, 0);
        if (!e_ok)
            atomicMin(status + 4, 0);
    }
    for (long i = t0; i < NC; i += stride)
        if (offsets[i + 1] < offsets[i])
            atomicMin(status + 1, (int)i);
    if (e_ok)
        for (long e = t0; e < E; e += stride) {
            const int j = nbr_in[e] & mask;
            if (j < 0 || j >= NT)
                atomicMin(status + 2, (int)e);
        }
    for (long i = t0; i < NT; i += stride) {
        const int t = types[i];
        if (t < -1 || t >= K)
            atomicMin(status + 3, (int)i);
    }
}

__global__ void k_na_prepare(long E, const int *__restrict__ nbr_in, int mask,
                             int *__restrict__ nbr, int *__restrict__ in_count)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < E) {
        const int j = nbr_in[e] & mask;
        nbr[e] = j;
        atomicAdd(in_count + j, 1);
    }
}

__global__ void k_na_split(long E, const double *__restrict__ v, double *__restrict__ rx,
                           double *__restrict__ ry, double *__restrict__ rz)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < E) {
        rx[e] = v[3 * e];
        ry[e] = v[3 * e + 1];
        rz[e] = v[3 * e + 2];
    }
}

// exclusive scan of n <= NOALLOC_MAX_ATOMS counts in one block
__global__ void k_na_scan(int n, const int *__restrict__ in, int *__restrict__ out)
{
    __shared__ int part[1024];
    const int per = (n + blockDim.x - 1) / blockDim.x;
    const int b = threadIdx.x * per, e = min(n, b + per);
    int s = 0;
    for (int i = b; i < e; ++i)
        s += in[i];
    part[threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int t = 0; t < (int)blockDim.x; ++t) {
            const int v = part[t];
            part[t] = acc;
            acc += v;
        }
        out[n] = acc;
    }
    __syncthreads();
    int acc = part[threadIdx.x];
    for (int i = b; i < e; ++i) {
        out[i] = acc;
        acc += in[i];
    }
}

__global__ void k_na_fill(long E, const int *__restrict__ nbr, const int *__restrict__ in_off,
                          int *__restrict__ cursor, int *__restrict__ in_edges)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < E) {
        const int j = nbr[e];
        in_edges[in_off[j] + atomicAdd(cursor + j, 1)] = (int)e;
    }
}

__global__ void k_na_sort(int n, const int *__restrict__ start, int *__restrict__ data)
{
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n)
        return;
    for (int i = start[s] + 1; i < start[s + 1]; ++i) {
        const int v = data[i];
        int j = i - 1;
        while (j >= start[s] && data[j] > v) {
            data[j + 1] = data[j];
            --j;
        }
        data[j + 1] = v;
    }
}

// per-atom virial split 0.5 / 0.25 onto both atoms (runtime/mtp/mlip.cpp:
// 1164-1190), written as rows [q][ntotal] (q = 0..5; rows 6..8 zero)
__global__ void k_na_virial(int ncenter, int ntotal, const int *__restrict__ offsets,
                            const int *__restrict__ in_off, const int *__restrict__ in_edges,
                            const double *__restrict__ dx, const double *__restrict__ dy,
                            const double *__restrict__ dz, const double *__restrict__ rx,
                            const double *__restrict__ ry, const double *__restrict__ rz,
                            double *__restrict__ rows)
{
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= ntotal)
        return;
    double v[6] = {0, 0, 0, 0, 0, 0};
    auto add = [&](int e) {
        const double d0 = dx[e], d1 = dy[e], d2 = dz[e];
        const double r0 = rx[e], r1 = ry[e], r2 = rz[e];
        v[0] -= 0.5 * d0 * r0;
        v[1] -= 0.5 * d1 * r1;
        v[2] -= 0.5 * d2 * r2;
        v[3] -= 0.25 * (d1 * r0 + d0 * r1);
        v[4] -= 0.25 * (d2 * r0 + d0 * r2);
        v[5] -= 0.25 * (d2 * r1 + d1 * r2);
    };
    if (k < ncenter)
        for (int e = offsets[k]; e < offsets[k + 1]; ++e)
            add(e);
    for (int q = in_off[k]; q < in_off[k + 1]; ++q)
        add(in_edges[q]);
    for (int q = 0; q < 6; ++q)
        rows[(size_t)q * ntotal + k] = v[q];
    for (int q = 6; q < 9; ++q)
        rows[(size_t)q * ntotal + k] = 0.0;
}

__global__ void k_na_outputs(int ntotal, const double *__restrict__ f, const double *__restrict__ vrows,
                             double *__restrict__ force, int accumulate, double *__restrict__ site_virial)
{
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= ntotal)
        return;
    if (force)
        for (int d = 0; d < 3; ++d)
            force[3 * k + d] = accumulate ? force[3 * k + d] + f[3 * k + d] : f[3 * k + d];
    if (site_virial)
        for (int q = 0; q < 6; ++q)
            site_virial[6 * (size_t)k + q] = vrows[(size_t)q * ntotal + k];
}

int noalloc_compute(mtpb_context *c, const mtpb_csr_request *r)
{
    if (!c || !r)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    const int NC = r->center_count, NT = r->ntotal;
    if (NC < 0 || NT < NC)
        return fail(MTPB_ERR_ARGUMENT, "need 0 <= center_count <= ntotal");
    if (NC > NOALLOC_MAX_CENTERS || NT > NOALLOC_MAX_ATOMS)
        return fail(MTPB_ERR_ARGUMENT,
                    "no-allocation path limit exceeded: at most " +
                        std::to_string(NOALLOC_MAX_CENTERS) + " centres and " +
                        std::to_string(NOALLOC_MAX_ATOMS) + " atoms (use mtpb_efs_csr)");
    if (c->nslot > NOALLOC_MAX_SLOTS)
        return fail(MTPB_ERR_UNSUPPORTED, "model basis too large for the no-allocation path "
                                          "(at most " + std::to_string(NOALLOC_MAX_SLOTS) +
                                              " basic-moment slots)");
    if (c->plan.global_rows)
        return fail(MTPB_ERR_UNSUPPORTED, "moment graph too large for shared memory: the "
                                          "no-allocation path has no room for its rows");
    if (!r->offsets || (NT > 0 && (!r->types || !r->x)) || (NC > 0 && !r->neighbors))
        return fail(MTPB_ERR_ARGUMENT, "offsets, neighbors, types and x are required");
    int rc = set_device(c);
    if (rc)
        return rc;
    unsigned char *base = nullptr;
    if ((rc = scratch_base(c->device, &base)))
        return rc;
    cudaStream_t s = c->stream;
    c->ev_valid = false;   // no stage timings for this call
    // validate offsets, neighbour indices and types on the device, then read
    // the verdict and the edge count before any kernel indexes with them
    int *check = (int *)(base + NA_CHECK);
    CUDA_TRY(cudaMemsetAsync(check, 0x7f, sizeof(int) * 6, s), "clear check");
    k_na_validate<<<16, 256, 0, s>>>(NC, NT, r->offsets, r->neighbors, r->neighbor_mask,
                                     r->types, c->model.K, check);
    CUDA_TRY(cudaGetLastError(), "validate request");
    int hcheck[6];
    CUDA_TRY(cudaMemcpyAsync(hcheck, check, sizeof(hcheck), cudaMemcpyDeviceToHost, s),
             "read validation");
    CUDA_TRY(cudaStreamSynchronize(s), "sync");
    if (hcheck[4] != NA_CHECK_NONE)
        return fail(MTPB_ERR_ARGUMENT, "no-allocation path limit exceeded: at most " +
                                           std::to_string(NOALLOC_MAX_EDGES) + " edges");
    if (hcheck[0] != NA_CHECK_NONE)
        return fail(MTPB_ERR_ARGUMENT, "offsets[0] must be 0");
    if (hcheck[1] != NA_CHECK_NONE)
        return fail(MTPB_ERR_ARGUMENT, "offsets must be non-decreasing (at centre " +
                                           std::to_string(hcheck[1]) + ")");
    if (hcheck[2] != NA_CHECK_NONE)
        return fail(MTPB_ERR_ARGUMENT, "neighbor index out of range at edge " +
                                           std::to_string(hcheck[2]));
    if (hcheck[3] != NA_CHECK_NONE)
        return fail(MTPB_ERR_ARGUMENT, "type out of range at atom " + std::to_string(hcheck[3]));
    const int E = hcheck[5];
    double *basic = (double *)(base + NA_BASIC), *adjoint = (double *)(base + NA_ADJ);
    double *rx = (double *)(base + NA_RX), *ry = (double *)(base + NA_RY),
           *rz = (double *)(base + NA_RZ);
    double *dx = (double *)(base + NA_DX), *dy = (double *)(base + NA_DY),
           *dz = (double *)(base + NA_DZ);
    int *nbr = (int *)(base + NA_NBR), *in_edges = (int *)(base + NA_IN_EDGES);
    int *in_count = (int *)(base + NA_IN_COUNT), *in_off = (int *)(base + NA_IN_OFF);
    int *cursor = (int *)(base + NA_IN_CURSOR), *maxdeg = (int *)(base + NA_MAXDEG);
    double *site_e = (double *)(base + NA_SITE_E), *site_e_all = (double *)(base + NA_SITE_E_ALL);
    double *force = (double *)(base + NA_FORCE), *vrows = (double *)(base + NA_VROWS);
    int *segs = (int *)(base + NA_SEGS);
    double *partials = (double *)(base + NA_PARTIALS), *sums = (double *)(base + NA_SUMS);
    c->launches = 0;
    c->have_list = false;
    c->have_efs = false;
    // the array keeps the previous call's contents: clear what accumulates
    CUDA_TRY(cudaMemsetAsync(in_count, 0, sizeof(int) * (NT + 1), s), "clear");
    CUDA_TRY(cudaMemsetAsync(cursor, 0, sizeof(int) * (NT + 1), s), "clear");
    if (NT)
        CUDA_TRY(cudaMemsetAsync(site_e_all, 0, sizeof(double) * NT, s), "clear");
    if (E) {
        k_na_prepare<<<nblk_na(E, 256), 256, 0, s>>>(E, r->neighbors, r->neighbor_mask, nbr,
                                                     in_count);
        if (r->neighbor_vectors)
            k_na_split<<<nblk_na(E, 256), 256, 0, s>>>(E, r->neighbor_vectors, rx, ry, rz);
        else
            CUDA_TRY(edge_vectors(NC, r->offsets, nbr, r->x, rx, ry, rz, s), "edge vectors");
    }
    k_na_scan<<<1, 1024, 0, s>>>(NT, in_count, in_off);
    if (E)
        k_na_fill<<<nblk_na(E, 256), 256, 0, s>>>(E, nbr, in_off, cursor, in_edges);
    if (NT)
        k_na_sort<<<nblk_na(NT, 128), 128, 0, s>>>(NT, in_off, in_edges);
    CUDA_TRY(cudaGetLastError(), "in-edge lists");
    // moments, graph, edge derivatives (existing kernels, explicit buffers)
    c->npad = ((NC + 31) / 32) * 32;
    EdgeArgs a = edge_args(c, NC, r->types, r->offsets, nbr, rx, ry, rz);
    a.group_maxdeg = maxdeg;
    CUDA_TRY(launch_group_maxdeg(NC, r->offsets, maxdeg, s), "group_maxdeg");
    CUDA_TRY(launch_moments_fwd(c->shape, a, basic, s), "moments forward");
    CUDA_TRY(launch_dag(c->plan, c->d_recs, c->d_phase_row0, c->nslot, NC, c->npad, r->types,
                        c->d_species, basic, adjoint, site_e, nullptr, c->d_err, s),
             "moment graph");
    CUDA_TRY(launch_moments_rev(c->shape, a, adjoint, dx, dy, dz, s), "moments reverse");
    CUDA_TRY(launch_force_gather(NC, NT, r->offsets, in_off, in_edges, dx, dy, dz, rx, ry, rz,
                                 force, nullptr, 0, s),
             "force gather");
    if (NT)
        k_na_virial<<<nblk_na(NT, 128), 128, 0, s>>>(NC, NT, r->offsets, in_off, in_edges, dx,
                                                     dy, dz, rx, ry, rz, vrows);
    if (NC)
        CUDA_TRY(cudaMemcpyAsync(site_e_all, site_e, sizeof(double) * NC, cudaMemcpyDeviceToDevice,
                                 s),
                 "site energies");
    // deterministic sums over <= 1024-atom segments
    int hseg[2 * NOALLOC_MAX_SEGMENTS + 2];
    int nseg = 0;
    for (int b = 0; b < (NT > 0 ? NT : 1); b += 1024, ++nseg) {
        hseg[nseg] = b;
        hseg[NOALLOC_MAX_SEGMENTS + nseg] = NT < b + 1024 ? NT : b + 1024;
    }
    hseg[2 * NOALLOC_MAX_SEGMENTS] = 0;
    hseg[2 * NOALLOC_MAX_SEGMENTS + 1] = nseg;
    CUDA_TRY(cudaMemcpyAsync(segs, hseg, sizeof(hseg), cudaMemcpyHostToDevice, s), "segments");
    CUDA_TRY(launch_segment_reduce(nseg, segs, segs + NOALLOC_MAX_SEGMENTS, site_e_all,
                                   NT ? vrows : nullptr, NT, partials, s),
             "segment reduce");
    CUDA_TRY(launch_struct_reduce(1, segs + 2 * NOALLOC_MAX_SEGMENTS, partials, sums, sums + 10, s),
             "reduce");
    if (NT)
        k_na_outputs<<<nblk_na(NT, 128), 128, 0, s>>>(NT, force, vrows, r->force,
                                                      r->accumulate_force, r->site_virial);
    if (r->site_energy && NC)
        CUDA_TRY(cudaMemcpyAsync(r->site_energy, site_e, sizeof(double) * NC,
                                 cudaMemcpyDeviceToDevice, s),
                 "copy site energy");
    if (r->total_energy)
        CUDA_TRY(cudaMemcpyAsync(r->total_energy, sums, sizeof(double), cudaMemcpyDeviceToDevice, s),
                 "copy energy");
    if (r->global_virial)
        CUDA_TRY(cudaMemcpyAsync(r->global_virial, sums + 10, 6 * sizeof(double),
                                 cudaMemcpyDeviceToDevice, s),
                 "copy virial");
    CUDA_TRY(cudaGetLastError(), "no-allocation EFS");
    // hseg lives on this host stack frame: wait for the copies before returning
    CUDA_TRY(cudaStreamSynchronize(s), "no-allocation EFS");
    c->launches = 14;
    return check_device_error(c);
}

} // namespace mtpb

extern "C" int mtpb_efs_csr_noalloc(mtpb_context *c, const mtpb_csr_request *req)
{
    mtpb::NvtxRange range("mtpb:efs_csr_noalloc");
    return mtpb::noalloc_compute(c, req);
}
