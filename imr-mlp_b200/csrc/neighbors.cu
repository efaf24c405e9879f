// neighbors.cu -- GPU cell-list neighbour builder whose per-atom neighbour
// sets equal the reference's default builder bit for bit.
//
// Reference behaviour (paths relative to the reference project):
//   base/neighborhoods_base.h:113-126  wrap: frac = p * inv(cell),
//                                      frac -= floor(frac), p = frac * cell
//   base/neighborhoods_base.h:31-99    periodic images: translation =
//                                      basis * image, basis = periodic cell
//                                      rows sorted by squared length
//   base/neighborhood.cpp:103-134      for a centre i and an image point of
//                                      atom o with i <= o: r = p_o - p_i,
//                                      accept r.r < rc^2, emit (o, r) to i
//                                      and (i, -r) to o when i != o
// A centre i therefore sees neighbour o at displacement
//   (w_o + T) - w_i            when i <= o, and
//   -((w_i + (-T)) - w_o)      when i >  o,
// where w are wrapped positions and T the image translation, every operation
// rounded as written (no fused multiply-add).  Each centre computes its own
// list independently with that rule, so no pairing step is needed.
//
// The search itself is a cell list in fractional coordinates: cells at least
// rc (perpendicular) thick, a stencil of +-ceil(rc*n/width) cells, periodic
// cell indices mapped to (cell, shift).  Atom lists inside a cell are sorted
// so that the output order is deterministic.
#include "internal.hpp"
#include "neighbors.hpp"
#include "refresh.cuh"

#include <cub/cub.cuh>

namespace mtpb {

__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }

// (p0*M(0,d) + p1*M(1,d)) + p2*M(2,d)  (Eigen RowVector3d * Matrix3d)
__device__ __forceinline__ void rowvec_mat(const double p[3], const double *M, double out[3])
{
    double r[3];
#pragma unroll
    for (int d = 0; d < 3; ++d)
        r[d] = dadd(dadd(dmul(p[0], M[d]), dmul(p[1], M[3 + d])), dmul(p[2], M[6 + d]));
    out[0] = r[0];
    out[1] = r[1];
    out[2] = r[2];
}

__global__ void k_struct_ids(int nstruct, const int *__restrict__ atom_offsets, int natoms,
                             int *__restrict__ struct_of)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= natoms)
        return;
    int lo = 0, hi = nstruct - 1;
    while (lo < hi) {   // last s with atom_offsets[s] <= i
        const int mid = (lo + hi + 1) >> 1;
        if (atom_offsets[mid] <= i)
            lo = mid;
        else
            hi = mid - 1;
    }
    struct_of[i] = lo;
}

__global__ void k_wrap_bin(int natoms, const NbStruct *__restrict__ structs,
                           const int *__restrict__ struct_of, const double *__restrict__ pos,
                           double *__restrict__ wx, double *__restrict__ wy,
                           double *__restrict__ wz, int *__restrict__ cell_of,
                           int *__restrict__ cell_count)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= natoms)
        return;
    const NbStruct &st = structs[struct_of[i]];
    const double p[3] = {pos[3 * i], pos[3 * i + 1], pos[3 * i + 2]};
    double f[3];
    rowvec_mat(p, st.inv, f);
#pragma unroll
    for (int d = 0; d < 3; ++d)
        f[d] = __dsub_rn(f[d], floor(f[d]));
    double w[3];
    rowvec_mat(f, st.cell, w);
    wx[i] = w[0];
    wy[i] = w[1];
    wz[i] = w[2];
    int c[3];
#pragma unroll
    for (int d = 0; d < 3; ++d) {
        int q = (int)floor(f[d] * st.ncell[d]);
        c[d] = q < 0 ? 0 : (q >= st.ncell[d] ? st.ncell[d] - 1 : q);
    }
    const int cell = st.cell0 + (c[0] * st.ncell[1] + c[1]) * st.ncell[2] + c[2];
    cell_of[i] = cell;
    atomicAdd(cell_count + cell, 1);
}

__global__ void k_fill_cells(int natoms, const int *__restrict__ cell_of,
                             const int *__restrict__ cell_start, int *__restrict__ cell_cursor,
                             int *__restrict__ cell_atoms)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= natoms)
        return;
    const int c = cell_of[i];
    cell_atoms[cell_start[c] + atomicAdd(cell_cursor + c, 1)] = i;
}

// insertion sort of small segments (the atoms of a cell, about ten each)
__global__ void k_sort_segments(int nseg, const int *__restrict__ start, int *__restrict__ data)
{
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= nseg)
        return;
    const int b = start[s], e = start[s + 1];
    for (int i = b + 1; i < e; ++i) {
        const int v = data[i];
        int j = i - 1;
        while (j >= b && data[j] > v) {
            data[j + 1] = data[j];
            --j;
        }
        data[j + 1] = v;
    }
}

// Bitonic sort of n = 32 V keys held by one warp, key k = v * 32 + lane in
// register v of that lane; ascending.
template <int V> __device__ __forceinline__ void warp_bitonic(int (&a)[V], int lane)
{
#pragma unroll
    for (int size = 2; size <= 32 * V; size <<= 1) {
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
            if (j >= 32) {   // partner in register v ^ (j / 32) of the same lane
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    const int w = v ^ (j >> 5);
                    if (w > v) {
                        const bool up = (((v << 5) | lane) & size) == 0;
                        const int lo = min(a[v], a[w]), hi = max(a[v], a[w]);
                        a[v] = up ? lo : hi;
                        a[w] = up ? hi : lo;
                    }
                }
            } else {   // partner in lane ^ j, same register
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    const int other = __shfl_xor_sync(0xffffffffu, a[v], j);
                    const bool up = (((v << 5) | lane) & size) == 0;
                    const bool lower = (lane & j) == 0;
                    a[v] = (up == lower) ? min(a[v], other) : max(a[v], other);
                }
            }
        }
    }
}

template <int V>
__device__ __forceinline__ void warp_sort_segment(int *__restrict__ data, int b, int n, int lane)
{
    int a[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
        const int k = v * 32 + lane;
        a[v] = k < n ? data[b + k] : 0x7fffffff;
    }
    warp_bitonic<V>(a, lane);
#pragma unroll
    for (int v = 0; v < V; ++v) {
        const int k = v * 32 + lane;
        if (k < n)
            data[b + k] = a[v];
    }
}

// In-edge lists: one warp sorts the segment of one atom into increasing edge
// order (bitonic in registers up to 256 entries; a single lane's insertion
// sort beyond), so that force sums run in a fixed order.
__global__ void k_sort_in_edges(int nseg, const int *__restrict__ start, int *__restrict__ data)
{
    const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int sgm = (int)(t >> 5);
    const int lane = threadIdx.x & 31;
    if (sgm >= nseg)
        return;
    const int b = start[sgm], n = start[sgm + 1] - b;
    if (n <= 1)
        return;
    if (n <= 64)
        warp_sort_segment<2>(data, b, n, lane);
    else if (n <= 128)
        warp_sort_segment<4>(data, b, n, lane);
    else if (n <= 256)
        warp_sort_segment<8>(data, b, n, lane);
    else if (lane == 0)
        for (int i = b + 1; i < b + n; ++i) {
            const int v = data[i];
            int j = i - 1;
            while (j >= b && data[j] > v) {
                data[j + 1] = data[j];
                --j;
            }
            data[j + 1] = v;
        }
}

// Cell-ordered copy of the wrapped positions: entry q holds the position of
// cell_atoms[q], so that the candidates of one cell are read contiguously.
__global__ void k_cell_positions(int natoms, const int *__restrict__ cell_atoms,
                                 const double *__restrict__ wx, const double *__restrict__ wy,
                                 const double *__restrict__ wz, double *__restrict__ xs,
                                 double *__restrict__ ys, double *__restrict__ zs)
{
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= natoms)
        return;
    const int o = cell_atoms[q];
    xs[q] = wx[o];
    ys[q] = wy[o];
    zs[q] = wz[o];
}

// Traverses the candidate set of centre i (one thread per centre): stencil
// cells in (d0, d1, d2) order, atoms of a cell in increasing index, their
// positions read from the cell-ordered copy.  FILL selects counting or
// writing (neighbour, image code, displacement, centre).
template <bool FILL>
__global__ void k_neighbors(int natoms, const NbStruct *__restrict__ structs,
                            const int *__restrict__ struct_of, const double *__restrict__ wx,
                            const double *__restrict__ wy, const double *__restrict__ wz,
                            const double *__restrict__ xs, const double *__restrict__ ys,
                            const double *__restrict__ zs, const int *__restrict__ cell_of,
                            const int *__restrict__ cell_start, const int *__restrict__ cell_atoms,
                            int *__restrict__ counts, const int *__restrict__ offsets,
                            int *__restrict__ nbr, int *__restrict__ shift_code,
                            double *__restrict__ rx, double *__restrict__ ry,
                            double *__restrict__ rz, int *__restrict__ center)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= natoms)
        return;
    const NbStruct &st = structs[struct_of[i]];
    const double xi = wx[i], yi = wy[i], zi = wz[i];
    int rel = cell_of[i] - st.cell0;
    const int c2 = rel % st.ncell[2];
    rel /= st.ncell[2];
    const int c1 = rel % st.ncell[1];
    const int c0 = rel / st.ncell[1];
    int count = 0;
    int out = FILL ? offsets[i] : 0;
    for (int d0 = -st.stencil[0]; d0 <= st.stencil[0]; ++d0) {
        const int a0 = c0 + d0;
        const int s0 = (a0 >= 0) ? a0 / st.ncell[0] : -((-a0 + st.ncell[0] - 1) / st.ncell[0]);
        const int w0 = a0 - s0 * st.ncell[0];
        for (int d1 = -st.stencil[1]; d1 <= st.stencil[1]; ++d1) {
            const int a1 = c1 + d1;
            const int s1 = (a1 >= 0) ? a1 / st.ncell[1] : -((-a1 + st.ncell[1] - 1) / st.ncell[1]);
            const int w1 = a1 - s1 * st.ncell[1];
            for (int d2 = -st.stencil[2]; d2 <= st.stencil[2]; ++d2) {
                const int a2 = c2 + d2;
                const int s2 =
                    (a2 >= 0) ? a2 / st.ncell[2] : -((-a2 + st.ncell[2] - 1) / st.ncell[2]);
                const int w2 = a2 - s2 * st.ncell[2];
                const bool zero = (s0 == 0 && s1 == 0 && s2 == 0);
                double t[3];
                image_translation(st, s0, s1, s2, t);
                const int cell = st.cell0 + (w0 * st.ncell[1] + w1) * st.ncell[2] + w2;
                for (int q = cell_start[cell]; q < cell_start[cell + 1]; ++q) {
                    const int o = cell_atoms[q];
                    if (zero && o == i)
                        continue;
                    const double xo = xs[q], yo = ys[q], zo = zs[q];
                    double r0, r1, r2;
                    if (i <= o) {
                        const double px = zero ? xo : dadd(xo, t[0]);
                        const double py = zero ? yo : dadd(yo, t[1]);
                        const double pz = zero ? zo : dadd(zo, t[2]);
                        r0 = __dsub_rn(px, xi);
                        r1 = __dsub_rn(py, yi);
                        r2 = __dsub_rn(pz, zi);
                    } else {
                        const double px = zero ? xi : dadd(xi, -t[0]);
                        const double py = zero ? yi : dadd(yi, -t[1]);
                        const double pz = zero ? zi : dadd(zi, -t[2]);
                        r0 = -__dsub_rn(px, xo);
                        r1 = -__dsub_rn(py, yo);
                        r2 = -__dsub_rn(pz, zo);
                    }
                    const double dsq = dadd(dadd(dmul(r0, r0), dmul(r1, r1)), dmul(r2, r2));
                    if (dsq < st.cutsq) {
                        if (FILL) {   // displacements: k_refresh_edges after this pass
                            nbr[out] = o;
                            shift_code[out] = (s0 + 128) | ((s1 + 128) << 8) | ((s2 + 128) << 16);
                            center[out] = i;
                            ++out;
                        } else {
                            ++count;
                        }
                    }
                }
            }
        }
    }
    if (!FILL)
        counts[i] = count;
}

// lowest index of an atom whose species lies outside 0..K-1 (INT_MAX: none)
__global__ void k_check_types(int natoms, const int *__restrict__ types, int K,
                              int *__restrict__ bad)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < natoms && (types[i] < 0 || types[i] >= K))
        atomicMin(bad, i);
}

__global__ void k_in_count(long nedges, const int *__restrict__ nbr, int *__restrict__ in_count)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < nedges)
        atomicAdd(in_count + nbr[e], 1);
}

__global__ void k_in_fill(long nedges, const int *__restrict__ nbr,
                          const int *__restrict__ in_offsets, int *__restrict__ cursor,
                          int *__restrict__ in_edges)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < nedges) {
        const int j = nbr[e];
        in_edges[in_offsets[j] + atomicAdd(cursor + j, 1)] = (int)e;
    }
}

// r_ij = x[j] - x[i] for caller-supplied lists (LAMMPS / CSR requests)
__global__ void k_edge_vectors(int ncenter, const int *__restrict__ offsets,
                               const int *__restrict__ nbr, const double *__restrict__ x,
                               double *__restrict__ rx, double *__restrict__ ry,
                               double *__restrict__ rz)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= ncenter)
        return;
    const double xi = x[3 * i], yi = x[3 * i + 1], zi = x[3 * i + 2];
    for (int e = offsets[i]; e < offsets[i + 1]; ++e) {
        const int j = nbr[e];
        rx[e] = __dsub_rn(x[3 * j], xi);
        ry[e] = __dsub_rn(x[3 * j + 1], yi);
        rz[e] = __dsub_rn(x[3 * j + 2], zi);
    }
}

// Edge vectors for new positions with the image of every pair kept from the
// last build (MD steps between rebuilds, MTPGpuComputeRequest::reuse_topology):
// w' = w_build + (x - x_build) keeps atoms unwrapped relative to the build, and
// r follows the build's i <= o rule so that unchanged positions reproduce the
// build's displacements bit for bit.  w' is formed once per atom (k_unwrapped,
// [atom][4] so that an edge gathers one 32-byte sector per atom).
__global__ void k_unwrapped(int natoms, const double *__restrict__ wx,
                            const double *__restrict__ wy, const double *__restrict__ wz,
                            const double *__restrict__ x_build, const double *__restrict__ x,
                            double *__restrict__ p)
{
    const int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= natoms)
        return;
    const double v0 = dadd(wx[a], __dsub_rn(x[3 * a], x_build[3 * a]));
    const double v1 = dadd(wy[a], __dsub_rn(x[3 * a + 1], x_build[3 * a + 1]));
    const double v2 = dadd(wz[a], __dsub_rn(x[3 * a + 2], x_build[3 * a + 2]));
    double2 *q = reinterpret_cast<double2 *>(p + 4 * (size_t)a);
    q[0] = make_double2(v0, v1);
    q[1] = make_double2(v2, 0.0);
}

// Wrapped positions as [atom][4] rows for k_refresh_edges, which then
// reproduces the build's displacement arithmetic edge by edge.
__global__ void k_pack_positions(int natoms, const double *__restrict__ wx,
                                 const double *__restrict__ wy, const double *__restrict__ wz,
                                 double *__restrict__ p)
{
    const int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= natoms)
        return;
    double2 *q = reinterpret_cast<double2 *>(p + 4 * (size_t)a);
    q[0] = make_double2(wx[a], wy[a]);
    q[1] = make_double2(wz[a], 0.0);
}

__global__ void k_refresh_edges(long nedges, const NbStruct *__restrict__ structs,
                                const int *__restrict__ struct_of, const int *__restrict__ center,
                                const int *__restrict__ nbr, const int *__restrict__ shift,
                                const double *__restrict__ p, double *__restrict__ rx,
                                double *__restrict__ ry, double *__restrict__ rz)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= nedges)
        return;
    const int i = center[e];
    double x, y, z;
    refresh_vector(structs[struct_of[i]], i, nbr[e], shift[e], p, x, y, z);
    rx[e] = x;
    ry[e] = y;
    rz[e] = z;
}

static inline int nblk(long n, int t) { return (int)((n + t - 1) / t); }

cudaError_t exclusive_scan(const int *in, int *out, int n, DeviceArena &arena, cudaStream_t s)
{
    // out has n+1 entries: out[0] = 0, out[k+1] = sum in[0..k]
    size_t tmp = 0;
    cudaError_t err = cub::DeviceScan::InclusiveSum(nullptr, tmp, in, out + 1, n, s);
    if (err != cudaSuccess)
        return err;
    void *t = arena.get("scan_tmp", tmp + 16);
    if (!t)
        return cudaErrorMemoryAllocation;
    err = cudaMemsetAsync(out, 0, sizeof(int), s);
    if (err != cudaSuccess)
        return err;
    if (n == 0)
        return cudaSuccess;
    return cub::DeviceScan::InclusiveSum(t, tmp, in, out + 1, n, s);
}

cudaError_t build_neighbors(const NbBuildInput &in, DeviceArena &arena, NbResult &res,
                            cudaStream_t s)
{
    const int N = in.natoms;
    const int NC = in.ncenter < 0 ? N : in.ncenter;   // centres: atoms [0, NC)
    const int T = 256;
    cudaError_t err;
#define CK(x)                                                                                      \
    do {                                                                                           \
        err = (x);                                                                                 \
        if (err != cudaSuccess)                                                                    \
            return err;                                                                            \
    } while (0)
    int *struct_of = arena.get<int>("nb_struct_of", N);
    double *wx = arena.get<double>("nb_wx", N), *wy = arena.get<double>("nb_wy", N),
           *wz = arena.get<double>("nb_wz", N);
    int *cell_of = arena.get<int>("nb_cell_of", N);
    int *cell_count = arena.get<int>("nb_cell_count", in.total_cells + 1);
    int *cell_start = arena.get<int>("nb_cell_start", in.total_cells + 1);
    int *cell_cursor = arena.get<int>("nb_cell_cursor", in.total_cells + 1);
    int *cell_atoms = arena.get<int>("nb_cell_atoms", N);
    double *xs = arena.get<double>("nb_xs", N), *ys = arena.get<double>("nb_ys", N),
           *zs = arena.get<double>("nb_zs", N);
    int *counts = arena.get<int>("nb_counts", NC + 1);
    int *offsets = arena.get<int>("offsets", NC + 1);
    if (!struct_of || !wx || !wy || !wz || !cell_of || !cell_count || !cell_start ||
        !cell_cursor || !cell_atoms || !xs || !ys || !zs || !counts || !offsets)
        return cudaErrorMemoryAllocation;
    res.wx = wx;
    res.wy = wy;
    res.wz = wz;
    res.offsets = offsets;
    res.struct_of = struct_of;
    if (N == 0 || NC == 0) {
        CK(cudaMemsetAsync(offsets, 0, sizeof(int), s));
        res.nedges = 0;
        if (N == 0)
            return cudaSuccess;
    }
    int *bad_type = arena.get<int>("nb_bad_type", 1);
    if (!bad_type)
        return cudaErrorMemoryAllocation;
    CK(cudaMemsetAsync(bad_type, 0x7f, sizeof(int), s));   // 0x7f7f7f7f: above any index
    if (in.types)
        k_check_types<<<nblk(N, T), T, 0, s>>>(N, in.types, in.K, bad_type);
    CK(cudaMemsetAsync(cell_count, 0, sizeof(int) * (in.total_cells + 1), s));
    CK(cudaMemsetAsync(cell_cursor, 0, sizeof(int) * (in.total_cells + 1), s));
    k_struct_ids<<<nblk(N, T), T, 0, s>>>(in.nstruct, in.atom_offsets, N, struct_of);
    k_wrap_bin<<<nblk(N, T), T, 0, s>>>(N, in.structs, struct_of, in.positions, wx, wy, wz,
                                       cell_of, cell_count);
    CK(cudaGetLastError());
    CK(exclusive_scan(cell_count, cell_start, in.total_cells, arena, s));
    k_fill_cells<<<nblk(N, T), T, 0, s>>>(N, cell_of, cell_start, cell_cursor, cell_atoms);
    k_sort_segments<<<nblk(in.total_cells, T), T, 0, s>>>(in.total_cells, cell_start,
                                                          cell_atoms);
    k_cell_positions<<<nblk(N, T), T, 0, s>>>(N, cell_atoms, wx, wy, wz, xs, ys, zs);
    CK(cudaGetLastError());
    if (NC > 0)
        k_neighbors<false><<<nblk(NC, 128), 128, 0, s>>>(
            NC, in.structs, struct_of, wx, wy, wz, xs, ys, zs, cell_of, cell_start, cell_atoms,
            counts, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr);
    CK(cudaGetLastError());
    CK(exclusive_scan(counts, offsets, NC, arena, s));
    int E = 0, bad = 0;
    CK(cudaMemcpyAsync(&E, offsets + NC, sizeof(int), cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(&bad, bad_type, sizeof(int), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    res.nedges = E;
    res.bad_type = bad < N ? bad : -1;
    int *nbr = arena.get<int>("nbr", (size_t)E + 1);
    int *shift = arena.get<int>("shift", (size_t)E + 1);
    double *rx = arena.get<double>("rx", (size_t)E + 1);
    double *ry = arena.get<double>("ry", (size_t)E + 1);
    double *rz = arena.get<double>("rz", (size_t)E + 1);
    int *center = arena.get<int>("edge_center", (size_t)E + 1);
    if (!nbr || !shift || !rx || !ry || !rz || !center)
        return cudaErrorMemoryAllocation;
    if (NC > 0)
        k_neighbors<true><<<nblk(NC, 128), 128, 0, s>>>(
            NC, in.structs, struct_of, wx, wy, wz, xs, ys, zs, cell_of, cell_start, cell_atoms,
            nullptr, offsets, nbr, shift, rx, ry, rz, center);
    CK(cudaGetLastError());
    // displacements edge-parallel from the wrapped positions (coalesced
    // stores; the same operations as the candidate test of the fill pass)
    double *packed = arena.get<double>("nb_packed", 4 * (size_t)N + 4);
    if (!packed)
        return cudaErrorMemoryAllocation;
    if (E > 0) {
        k_pack_positions<<<nblk(N, T), T, 0, s>>>(N, wx, wy, wz, packed);
        k_refresh_edges<<<nblk(E, 256), 256, 0, s>>>(E, in.structs, struct_of, center, nbr, shift,
                                                     packed, rx, ry, rz);
        CK(cudaGetLastError());
    }
    res.center = center;
    res.nbr = nbr;
    res.shift = shift;
    res.rx = rx;
    res.ry = ry;
    res.rz = rz;
    CK(build_in_edges(N, E, nbr, arena, res, s));
    return cudaSuccess;
#undef CK
}

cudaError_t build_in_edges(int ntotal, long E, const int *nbr, DeviceArena &arena, NbResult &res,
                           cudaStream_t s)
{
    cudaError_t err;
    int *in_count = arena.get<int>("in_count", ntotal + 1);
    int *in_offsets = arena.get<int>("in_offsets", ntotal + 1);
    int *cursor = arena.get<int>("in_cursor", ntotal + 1);
    int *in_edges = arena.get<int>("in_edges", (size_t)E + 1);
    if (!in_count || !in_offsets || !cursor || !in_edges)
        return cudaErrorMemoryAllocation;
    if ((err = cudaMemsetAsync(in_count, 0, sizeof(int) * (ntotal + 1), s)) != cudaSuccess)
        return err;
    if ((err = cudaMemsetAsync(cursor, 0, sizeof(int) * (ntotal + 1), s)) != cudaSuccess)
        return err;
    if (E > 0)
        k_in_count<<<nblk(E, 256), 256, 0, s>>>(E, nbr, in_count);
    if ((err = exclusive_scan(in_count, in_offsets, ntotal, arena, s)) != cudaSuccess)
        return err;
    if (E > 0)
        k_in_fill<<<nblk(E, 256), 256, 0, s>>>(E, nbr, in_offsets, cursor, in_edges);
    if (ntotal > 0)
        k_sort_in_edges<<<nblk((long)ntotal * 32, 128), 128, 0, s>>>(ntotal, in_offsets, in_edges);
    res.in_offsets = in_offsets;
    res.in_edges = in_edges;
    return cudaGetLastError();
}

cudaError_t refresh_edges(int natoms, const NbStruct *structs, const int *struct_of,
                          const NbResult &nb, const double *x_build, const double *x,
                          double *unwrapped, double *rx, double *ry, double *rz, cudaStream_t s)
{
    if (nb.nedges == 0)
        return cudaSuccess;
    k_unwrapped<<<nblk(natoms, 256), 256, 0, s>>>(natoms, nb.wx, nb.wy, nb.wz, x_build, x,
                                                  unwrapped);
    k_refresh_edges<<<nblk(nb.nedges, 256), 256, 0, s>>>(nb.nedges, structs, struct_of,
                                                         nb.center, nb.nbr, nb.shift, unwrapped,
                                                         rx, ry, rz);
    return cudaGetLastError();
}

cudaError_t unwrap_positions(int natoms, const NbResult &nb, const double *x_build,
                             const double *x, double *unwrapped, cudaStream_t s)
{
    if (natoms == 0)
        return cudaSuccess;
    k_unwrapped<<<nblk(natoms, 256), 256, 0, s>>>(natoms, nb.wx, nb.wy, nb.wz, x_build, x,
                                                  unwrapped);
    return cudaGetLastError();
}

__global__ void k_edge_pairs(long nedges, const int *__restrict__ center,
                             const int *__restrict__ nbr, const int *__restrict__ types, int K,
                             int *__restrict__ pair)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= nedges)
        return;
    const int it = types[center[e]], jt = types[nbr[e]];
    pair[e] = (it >= 0 && jt >= 0) ? it * K + jt : -1;
}

cudaError_t edge_pairs(long nedges, const int *center, const int *nbr, const int *types, int K,
                       int *pair, cudaStream_t s)
{
    if (nedges == 0)
        return cudaSuccess;
    k_edge_pairs<<<nblk(nedges, 256), 256, 0, s>>>(nedges, center, nbr, types, K, pair);
    return cudaGetLastError();
}

cudaError_t edge_vectors(int ncenter, const int *offsets, const int *nbr, const double *x,
                         double *rx, double *ry, double *rz, cudaStream_t s)
{
    if (ncenter == 0)
        return cudaSuccess;
    k_edge_vectors<<<nblk(ncenter, 128), 128, 0, s>>>(ncenter, offsets, nbr, x, rx, ry, rz);
    return cudaGetLastError();
}

} // namespace mtpb
