// csr.cu -- caller-supplied neighbour lists: the MTPGpuBatchRequest-style
// CSR request and the LAMMPS pair-style request.
//
// Semantics follow MLIPCore::compute (runtime/mtp/mlip.cpp:906-1193): centres
// or neighbours whose type maps to -1 are skipped, r_ij = x[j] - x[i], forces
// are -dE/dx on centres and neighbours (ghosts included), and the per-atom
// virial puts 0.5 (diagonal) / 0.25 (off-diagonal) of every pair term on each
// of the two atoms (:1164-1190).
#include "context.hpp"

#include <algorithm>
#include <vector>

namespace mtpb {

__global__ void k_mask_neighbors(long E, const int *__restrict__ in, int mask,
                                 int *__restrict__ out)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < E)
        out[e] = in[e] & mask;
}

__global__ void k_split_vectors(long E, const double *__restrict__ v, double *__restrict__ rx,
                                double *__restrict__ ry, double *__restrict__ rz)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < E) {
        rx[e] = v[3 * e];
        ry[e] = v[3 * e + 1];
        rz[e] = v[3 * e + 2];
    }
}

// Per-atom virial with the MLIPCore split, written as 9 rows [q][ntotal]
// (q = 0..5: xx yy zz xy xz yz, rows 6..8 zero) so that the segment reduction
// can sum it.
__global__ void k_split_virial(int ncenter, int ntotal, const int *__restrict__ offsets,
                               const int *__restrict__ in_offsets,
                               const int *__restrict__ in_edges, const double *__restrict__ dx,
                               const double *__restrict__ dy, const double *__restrict__ dz,
                               const double *__restrict__ rx, const double *__restrict__ ry,
                               const double *__restrict__ rz, double *__restrict__ out)
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
    for (int q = in_offsets[k]; q < in_offsets[k + 1]; ++q)
        add(in_edges[q]);
#pragma unroll
    for (int q = 0; q < 6; ++q)
        out[(size_t)q * ntotal + k] = v[q];
#pragma unroll
    for (int q = 6; q < 9; ++q)
        out[(size_t)q * ntotal + k] = 0.0;
}

__global__ void k_virial_rows_to_aos(int n, const double *__restrict__ rows, double *__restrict__ out,
                                     int accumulate)
{
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n)
        return;
#pragma unroll
    for (int q = 0; q < 6; ++q) {
        const double v = rows[(size_t)q * n + k];
        out[6 * (size_t)k + q] = accumulate ? out[6 * (size_t)k + q] + v : v;
    }
}

static inline int nb_(long n, int t) { return (int)((n + t - 1) / t); }

int csr_compute_impl(mtpb_context *c, const mtpb_csr_request *r, int memory,
                     bool accumulate_virial)
{
    if (!c || !r)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    const int NC = r->center_count, NT = r->ntotal;
    if (NC < 0 || NT < NC)
        return fail(MTPB_ERR_ARGUMENT, "need 0 <= center_count <= ntotal");
    if (NT > 0 && (!r->types || !r->x))
        return fail(MTPB_ERR_ARGUMENT, "types and x are required");
    if (!r->offsets || (NC > 0 && !r->neighbors))
        return fail(MTPB_ERR_ARGUMENT, "offsets and neighbors are required");
    int rc = set_device(c);
    if (rc)
        return rc;
    const bool dev = memory == MTPB_MEMORY_DEVICE;
    cudaStream_t s = c->stream;
    c->launches = 0;
    c->have_list = false;   // the structure list is replaced by this request
    c->have_efs = false;
    // offsets and edge count
    std::vector<int> hoff(NC + 1);
    if (dev)
        CUDA_TRY(cudaMemcpy(hoff.data(), r->offsets, sizeof(int) * (NC + 1), cudaMemcpyDeviceToHost),
                 "read offsets");
    else
        std::copy(r->offsets, r->offsets + NC + 1, hoff.begin());
    if (hoff[0] != 0)
        return fail(MTPB_ERR_ARGUMENT, "offsets[0] must be 0");
    for (int i = 0; i < NC; ++i)
        if (hoff[i + 1] < hoff[i])
            return fail(MTPB_ERR_ARGUMENT, "offsets must be non-decreasing");
    const long E = hoff[NC];
    // host-side index validation (neighbour indices and types)
    {
        std::vector<int> hn(E), ht(NT);
        if (dev) {
            if (E)
                CUDA_TRY(cudaMemcpy(hn.data(), r->neighbors, sizeof(int) * E, cudaMemcpyDeviceToHost),
                         "read neighbors");
            if (NT)
                CUDA_TRY(cudaMemcpy(ht.data(), r->types, sizeof(int) * NT, cudaMemcpyDeviceToHost),
                         "read types");
        } else {
            std::copy(r->neighbors, r->neighbors + E, hn.begin());
            std::copy(r->types, r->types + NT, ht.begin());
        }
        for (long e = 0; e < E; ++e) {
            const int j = hn[e] & r->neighbor_mask;
            if (j < 0 || j >= NT)
                return fail(MTPB_ERR_ARGUMENT, "neighbor index out of range at edge " +
                                                   std::to_string(e));
        }
        for (int i = 0; i < NT; ++i)
            if (ht[i] < -1 || ht[i] >= c->model.K)
                return fail(MTPB_ERR_ARGUMENT, "type out of range at atom " + std::to_string(i));
    }
    int *d_off = c->arena.get<int>("csr_offsets", NC + 1);
    int *d_nbr = c->arena.get<int>("csr_nbr", E + 1);
    int *d_types = c->arena.get<int>("csr_types", NT + 1);
    double *d_x = c->arena.get<double>("csr_x", 3 * (size_t)NT + 3);
    double *rx = c->arena.get<double>("csr_rx", E + 1), *ry = c->arena.get<double>("csr_ry", E + 1),
           *rz = c->arena.get<double>("csr_rz", E + 1);
    double *dx = c->arena.get<double>("dx", E + 1), *dy = c->arena.get<double>("dy", E + 1),
           *dz = c->arena.get<double>("dz", E + 1);
    double *site_energy = c->arena.get<double>("site_energy", NC + 1);
    double *forces = c->arena.get<double>("forces", 3 * (size_t)NT + 3);
    double *rows = c->arena.get<double>("atom_virial", 9 * (size_t)NT + 9);
    if (!d_off || !d_nbr || !d_types || !d_x || !rx || !ry || !rz || !dx || !dy || !dz ||
        !site_energy || !forces || !rows)
        return fail(MTPB_ERR_MEMORY, "device allocation failed");
    const cudaMemcpyKind k = dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    CUDA_TRY(cudaMemcpyAsync(d_off, r->offsets, sizeof(int) * (NC + 1), k, s), "upload offsets");
    if (E) {
        int *tmp = c->arena.get<int>("csr_nbr_raw", E + 1);
        if (!tmp)
            return fail(MTPB_ERR_MEMORY, "device allocation failed");
        CUDA_TRY(cudaMemcpyAsync(tmp, r->neighbors, sizeof(int) * E, k, s), "upload neighbors");
        k_mask_neighbors<<<nb_(E, 256), 256, 0, s>>>(E, tmp, r->neighbor_mask, d_nbr);
    }
    if (NT) {
        CUDA_TRY(cudaMemcpyAsync(d_types, r->types, sizeof(int) * NT, k, s), "upload types");
        CUDA_TRY(cudaMemcpyAsync(d_x, r->x, sizeof(double) * 3 * NT, k, s), "upload x");
    }
    if (E) {
        if (r->neighbor_vectors) {
            double *v = c->arena.get<double>("csr_vec", 3 * (size_t)E + 3);
            if (!v)
                return fail(MTPB_ERR_MEMORY, "device allocation failed");
            CUDA_TRY(cudaMemcpyAsync(v, r->neighbor_vectors, sizeof(double) * 3 * E, k, s),
                     "upload vectors");
            k_split_vectors<<<nb_(E, 256), 256, 0, s>>>(E, v, rx, ry, rz);
        } else {
            CUDA_TRY(edge_vectors(NC, d_off, d_nbr, d_x, rx, ry, rz, s), "edge vectors");
        }
    }
    NbResult res;
    CUDA_TRY(build_in_edges(NT, E, d_nbr, c->arena, res, s), "in-edge lists");
    CUDA_TRY(cudaEventRecord(c->ev[0], s), "event");
    // caller lists (LAMMPS full lists with their skin) may hold pairs beyond
    // the cutoff
    rc = run_moments(c, NC, d_types, d_off, d_nbr, rx, ry, rz, site_energy, dx, dy, dz, true, E,
                     true);
    if (rc)
        return rc;
    CUDA_TRY(launch_force_gather(NC, NT, d_off, res.in_offsets, res.in_edges, dx, dy, dz, rx, ry,
                                 rz, forces, nullptr, 0, s),
             "force gather");
    c->launches++;
    // energy and virial sums (one segment list over the centres / all atoms)
    std::vector<int> sb, se;
    for (int a = 0; a < std::max(NT, 1); a += 1024) {
        sb.push_back(a);
        se.push_back(std::min(a + 1024, NT));
    }
    const int nseg = (int)sb.size();
    int *d_sb = c->arena.get<int>("csr_seg_b", nseg), *d_se = c->arena.get<int>("csr_seg_e", nseg);
    int *d_s0 = c->arena.get<int>("csr_seg_0", 2);
    double *partials = c->arena.get<double>("partials", 10 * (size_t)nseg + 10);
    double *sums = c->arena.get<double>("csr_sums", 20);
    if (!d_sb || !d_se || !d_s0 || !partials || !sums)
        return fail(MTPB_ERR_MEMORY, "device allocation failed");
    const int s0[2] = {0, nseg};
    CUDA_TRY(cudaMemcpyAsync(d_sb, sb.data(), sizeof(int) * nseg, cudaMemcpyHostToDevice, s), "seg");
    CUDA_TRY(cudaMemcpyAsync(d_se, se.data(), sizeof(int) * nseg, cudaMemcpyHostToDevice, s), "seg");
    CUDA_TRY(cudaMemcpyAsync(d_s0, s0, sizeof(int) * 2, cudaMemcpyHostToDevice, s), "seg");
    // site energies exist for centres only: pad to ntotal with zeros
    double *se_all = c->arena.get<double>("csr_se_all", NT + 1);
    if (!se_all)
        return fail(MTPB_ERR_MEMORY, "device allocation failed");
    CUDA_TRY(cudaMemsetAsync(se_all, 0, sizeof(double) * (NT + 1), s), "memset");
    if (NC)
        CUDA_TRY(cudaMemcpyAsync(se_all, site_energy, sizeof(double) * NC, cudaMemcpyDeviceToDevice, s),
                 "copy");
    const bool want_virial = r->site_virial || r->global_virial;
    if (want_virial && NT) {
        k_split_virial<<<nb_(NT, 128), 128, 0, s>>>(NC, NT, d_off, res.in_offsets, res.in_edges, dx,
                                                  dy, dz, rx, ry, rz, rows);
        c->launches++;
    }
    CUDA_TRY(launch_segment_reduce(nseg, d_sb, d_se, se_all, want_virial && NT ? rows : nullptr, NT,
                                   partials, s),
             "segment reduce");
    CUDA_TRY(launch_struct_reduce(1, d_s0, partials, sums, sums + 10, s), "reduce");
    c->launches += 2;
    CUDA_TRY(cudaEventRecord(c->ev[5], s), "event");
    c->ev_valid = true;
    // outputs
    const cudaMemcpyKind o = dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
    std::vector<double> hsum(20);
    CUDA_TRY(cudaMemcpyAsync(hsum.data(), sums, sizeof(double) * 20, cudaMemcpyDeviceToHost, s),
             "copy sums");
    std::vector<double> hf;
    if (r->force && NT) {
        if (r->accumulate_force) {
            hf.resize(3 * (size_t)NT);
            CUDA_TRY(cudaMemcpyAsync(hf.data(), forces, sizeof(double) * 3 * NT,
                                     cudaMemcpyDeviceToHost, s),
                     "copy forces");
        } else {
            CUDA_TRY(cudaMemcpyAsync(r->force, forces, sizeof(double) * 3 * NT, o, s), "copy forces");
        }
    }
    if (r->site_energy && NC)
        CUDA_TRY(cudaMemcpyAsync(r->site_energy, site_energy, sizeof(double) * NC, o, s),
                 "copy site energy");
    std::vector<double> hv;
    if (r->site_virial && NT) {
        double *aos = c->arena.get<double>("csr_vir_aos", 6 * (size_t)NT + 6);
        if (!aos)
            return fail(MTPB_ERR_MEMORY, "device allocation failed");
        k_virial_rows_to_aos<<<nb_(NT, 256), 256, 0, s>>>(NT, rows, aos, 0);
        if (accumulate_virial) {
            hv.resize(6 * (size_t)NT);
            CUDA_TRY(cudaMemcpyAsync(hv.data(), aos, sizeof(double) * 6 * NT,
                                     cudaMemcpyDeviceToHost, s),
                     "copy virial");
        } else {
            CUDA_TRY(cudaMemcpyAsync(r->site_virial, aos, sizeof(double) * 6 * NT, o, s),
                     "copy virial");
        }
    }
    CUDA_TRY(cudaStreamSynchronize(s), "CSR EFS");
    if ((rc = check_device_error(c)))
        return rc;
    if (r->force && NT && r->accumulate_force) {
        if (dev)
            return fail(MTPB_ERR_ARGUMENT, "accumulate_force needs host memory");
        for (size_t i = 0; i < hf.size(); ++i)
            r->force[i] += hf[i];
    }
    if (!hv.empty())
        for (size_t i = 0; i < hv.size(); ++i)
            r->site_virial[i] += hv[i];
    if (r->total_energy) {
        if (dev)
            CUDA_TRY(cudaMemcpy(r->total_energy, sums, sizeof(double), cudaMemcpyDeviceToDevice),
                     "copy energy");
        else
            *r->total_energy = hsum[0];
    }
    if (r->global_virial) {
        double g[6];
        for (int q = 0; q < 6; ++q)
            g[q] = hsum[10 + q];
        if (dev)
            CUDA_TRY(cudaMemcpy(r->global_virial, g, sizeof(g), cudaMemcpyHostToDevice), "copy");
        else
            std::copy(g, g + 6, r->global_virial);
    }
    // per-edge derivatives stay available for diagnostics
    c->nedges = E;
    c->have_efs = true;
    return MTPB_OK;
}

int csr_compute(mtpb_context *c, const mtpb_csr_request *r, int memory)
{
    return csr_compute_impl(c, r, memory, false);
}

// LAMMPS request: renumber so that the centres come first, run the CSR path,
// scatter results back (forces / virials added, as the pair style expects).
int lammps_compute(mtpb_context *c, const mtpb_lammps_request *r)
{
    if (!c || !r)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    const int inum = r->inum, NT = r->ntotal;
    if (inum < 0 || NT < inum || (inum > 0 && (!r->ilist || !r->numneigh || !r->firstneigh)) ||
        (NT > 0 && (!r->type || !r->x || !r->type_map)))
        return fail(MTPB_ERR_ARGUMENT, "incomplete LAMMPS request");
    std::vector<int> newid(NT, -1), oldid(NT);
    for (int c2 = 0; c2 < inum; ++c2) {
        const int a = r->ilist[c2];
        if (a < 0 || a >= NT || newid[a] >= 0)
            return fail(MTPB_ERR_ARGUMENT, "ilist has an invalid or repeated atom");
        newid[a] = c2;
        oldid[c2] = a;
    }
    int next = inum;
    for (int a = 0; a < NT; ++a)
        if (newid[a] < 0) {
            newid[a] = next;
            oldid[next++] = a;
        }
    std::vector<int> off(inum + 1, 0), nbr;
    std::vector<int> types(NT);
    std::vector<double> x(3 * (size_t)NT);
    for (int i = 0; i < NT; ++i) {
        const int a = oldid[i];
        const int t = r->type[a];
        types[i] = (t >= 0 && t < r->type_map_count) ? r->type_map[t] : -1;
        if (types[i] >= c->model.K)
            return fail(MTPB_ERR_ARGUMENT, "type_map gives a species outside the model");
        x[3 * i] = r->x[3 * a];
        x[3 * i + 1] = r->x[3 * a + 1];
        x[3 * i + 2] = r->x[3 * a + 2];
    }
    for (int c2 = 0; c2 < inum; ++c2) {
        const int a = oldid[c2];
        const int *list = r->firstneigh[a];
        for (int jj = 0; jj < r->numneigh[a]; ++jj) {
            const int j = list[jj] & r->neighbor_mask;
            if (j < 0 || j >= NT)
                return fail(MTPB_ERR_ARGUMENT, "neighbour index out of range");
            nbr.push_back(newid[j]);
        }
        off[c2 + 1] = (int)nbr.size();
    }
    std::vector<double> f(3 * (size_t)NT, 0.0), se(inum), vir(r->site_virial ? 6 * (size_t)NT : 0);
    double energy = 0, gvir[6] = {0, 0, 0, 0, 0, 0};
    mtpb_csr_request q{};
    q.center_count = inum;
    q.ntotal = NT;
    q.offsets = off.data();
    q.neighbors = nbr.data();
    q.neighbor_mask = -1;
    q.types = types.data();
    q.x = x.data();
    q.force = f.data();
    q.total_energy = &energy;
    q.site_energy = se.data();
    q.site_virial = r->site_virial ? vir.data() : nullptr;
    q.global_virial = r->virial ? gvir : nullptr;
    int rc = csr_compute_impl(c, &q, MTPB_MEMORY_HOST, false);
    if (rc)
        return rc;
    for (int i = 0; i < NT; ++i) {
        const int a = oldid[i];
        for (int d = 0; d < 3; ++d)
            r->f[3 * a + d] += f[3 * i + d];
        if (r->site_virial)
            for (int d = 0; d < 6; ++d)
                r->site_virial[6 * a + d] += vir[6 * i + d];
    }
    if (r->site_energy)
        for (int c2 = 0; c2 < inum; ++c2)
            r->site_energy[oldid[c2]] = se[c2];
    if (r->energy)
        *r->energy += energy;
    if (r->virial)
        for (int d = 0; d < 6; ++d)
            r->virial[d] += gvir[d];
    return MTPB_OK;
}

} // namespace mtpb
