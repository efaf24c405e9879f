// training.cu -- loss and coefficient gradient of a structure batch on the
// device (the reference trainer's AccumulateGard without the penalty term).
//
// Reference semantics (paths relative to the reference project):
//   loss terms and their derivatives   train/train_mtp.cpp:3839-3996 (AddLossGard)
//   weights E/N^p, F/N^p, S/N^p         train/train_mtp.cpp:2552-2568
//   per-structure normalisation         train/train_mtp.cpp:3073-3078
//   edge weights w_j, species gradient  potentials/potential_mtp.cpp:6896-6922
//   site gradient                       potentials/potential_mtp.cpp:3348-3550
//
// Order of work for one call (all on the context stream):
//   EFS pass (efs.cu) -> k_loss_struct -> k_edge_weights -> tangent basics
//   -> dual graph -> per-edge channel records -> k_radial_grad over edges
//   bucketed by species pair -> column sums -> k_assemble.
// Every reduction runs in a fixed order, so results are reproducible.
#include "radial.cuh"
#include "context.hpp"

#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>

namespace mtpb {

constexpr int LOSS_THREADS = 128;
constexpr int TERMS = 7;   // loss, E/F/S loss, squared E/N, F and S errors

struct LossParams {
    double we, wf, ws;   // weights
    double pe, pf, ps;   // powers of the atom count
    int has_e, has_f, has_s;
    int K;
};

template <int N> __device__ __forceinline__ double block_sum(double v, double *sh)
{
    sh[threadIdx.x] = v;
    __syncthreads();
#pragma unroll
    for (int s = N / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s)
            sh[threadIdx.x] += sh[threadIdx.x + s];
        __syncthreads();
    }
    const double r = sh[0];
    __syncthreads();
    return r;
}

// One block per structure: loss terms, dL/dE, dL/dS (9) and dL/dF per atom,
// dL/dE copied to every atom, species gradient.  terms[s] = {loss, energy,
// force, stress loss, (E-E*)^2/N^2, sum |F-F*|^2, sum (W-W*)^2, species[K]}.
__global__ void __launch_bounds__(LOSS_THREADS)
    k_loss_struct(const int *__restrict__ aoff, const int *__restrict__ types,
                  const double *__restrict__ energy, const double *__restrict__ forces,
                  const double *__restrict__ stress, const double *__restrict__ te,
                  const double *__restrict__ tf, const double *__restrict__ ts, LossParams lp,
                  double *__restrict__ dlde_atom, double *__restrict__ dldf,
                  double *__restrict__ dlds, double *__restrict__ terms)
{
    __shared__ double sh[LOSS_THREADS];
    __shared__ int counts[32];
    __shared__ double dlde_s;
    const int s = blockIdx.x;
    const int a0 = aoff[s], a1 = aoff[s + 1];
    const int n = a1 - a0;
    double *t = terms + (size_t)s * (TERMS + lp.K);
    for (int i = threadIdx.x; i < lp.K && i < 32; i += blockDim.x)
        counts[i] = 0;
    __syncthreads();
    if (n == 0) {
        for (int i = threadIdx.x; i < TERMS + lp.K; i += blockDim.x)
            t[i] = 0.0;
        return;
    }
    // forces (train_mtp.cpp: force term, weight / N^power)
    const double wf = lp.has_f ? lp.wf / pow((double)n, lp.pf) : 0.0;
    double ff = 0.0;
    for (int i = a0 + threadIdx.x; i < a1; i += blockDim.x) {
        double d[3];
#pragma unroll
        for (int a = 0; a < 3; ++a)
            d[a] = lp.has_f ? forces[3 * (size_t)i + a] - tf[3 * (size_t)i + a] : 0.0;
        ff += d[0] * d[0] + d[1] * d[1] + d[2] * d[2];
#pragma unroll
        for (int a = 0; a < 3; ++a)
            dldf[3 * (size_t)i + a] = 2.0 * wf * d[a];
        const int ty = types[i];
        if (ty >= 0 && ty < 32)
            atomicAdd(&counts[ty], 1);
    }
    ff = block_sum<LOSS_THREADS>(ff, sh);
    if (threadIdx.x == 0) {
        double loss = 0.0, lf = 0.0, ls = 0.0, le = 0.0, m4 = 0.0, m5 = 0.0, m6 = 0.0;
        if (lp.has_f) {
            m5 = ff;
            lf = wf * ff;
            loss += lf;
        }
        double ws = lp.has_s ? lp.ws / pow((double)n, lp.ps) : 0.0;
        double ss = 0.0;
        for (int a = 0; a < 9; ++a) {
            const double d = lp.has_s ? stress[9 * (size_t)s + a] - ts[9 * (size_t)s + a] : 0.0;
            ss += d * d;
            dlds[9 * (size_t)s + a] = 2.0 * ws * d;
        }
        if (lp.has_s) {
            m6 = ss;
            ls = ws * ss;
            loss += ls;
        }
        double dlde = 0.0;
        if (lp.has_e) {
            const double we = lp.we / pow((double)n, lp.pe);
            const double d = energy[s] - te[s];
            m4 = d * d / n / n;
            le = we * (d * d);
            loss += le;
            dlde = 2.0 * we * d;
        }
        dlde_s = dlde;
        t[0] = loss;
        t[1] = le;
        t[2] = lf;
        t[3] = ls;
        t[4] = m4;
        t[5] = m5;
        t[6] = m6;
    }
    __syncthreads();
    const double dlde = dlde_s;
    for (int i = a0 + threadIdx.x; i < a1; i += blockDim.x)
        dlde_atom[i] = dlde;
    for (int k = threadIdx.x; k < lp.K; k += blockDim.x)
        t[TERMS + k] = k < 32 ? dlde * counts[k] : 0.0;
}

// w_e = dL/dF_centre - dL/dF_neighbour - dL/dS r_e (potential_mtp.cpp:6905-6916)
__global__ void k_edge_weights(long E, const int *__restrict__ center, const int *__restrict__ nbr,
                               const int *__restrict__ struct_of, const double *__restrict__ rx,
                               const double *__restrict__ ry, const double *__restrict__ rz,
                               const double *__restrict__ dldf, const double *__restrict__ dlds,
                               double *__restrict__ wx, double *__restrict__ wy,
                               double *__restrict__ wz)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= E)
        return;
    const int i = center[e], j = nbr[e];
    const double *S = dlds + 9 * (size_t)struct_of[i];
    const double r[3] = {rx[e], ry[e], rz[e]};
    double w[3];
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        w[a] = dldf[3 * (size_t)i + a] - dldf[3 * (size_t)j + a];
#pragma unroll
        for (int b = 0; b < 3; ++b)
            w[a] -= S[a * 3 + b] * r[b];
    }
    wx[e] = w[0];
    wy[e] = w[1];
    wz[e] = w[2];
}

// Species-pair bucket of every edge; edges the site sums skip (r > cutoff,
// r = 0, type -1; potential_mtp.cpp:2842) go to bucket K*K.
__global__ void k_pair_keys(long E, int K, const int *__restrict__ center,
                            const int *__restrict__ nbr, const int *__restrict__ types,
                            const double *__restrict__ rx, const double *__restrict__ ry,
                            const double *__restrict__ rz, const PairParams *__restrict__ pairs,
                            unsigned *__restrict__ keys, int *__restrict__ ids)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= E)
        return;
    const int it = types[center[e]], jt = types[nbr[e]];
    unsigned key = (unsigned)(K * K);
    if (it >= 0 && jt >= 0) {
        const double x = rx[e], y = ry[e], z = rz[e];
        const double r = sqrt(__dadd_rn(__dadd_rn(__dmul_rn(x, x), __dmul_rn(y, y)),
                                        __dmul_rn(z, z)));
        const int p = it * K + jt;
        if (r > 0.0 && r <= pairs[p].rmax)
            key = (unsigned)p;
    }
    keys[e] = key;
    ids[e] = (int)e;
}

// bounds[p] = first sorted position of bucket p (p = 0..K*K+1)
__global__ void k_bucket_bounds(long E, int nb, const unsigned *__restrict__ sorted,
                                long *__restrict__ bounds)
{
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p > nb)
        return;
    long lo = 0, hi = E;
    while (lo < hi) {
        const long mid = (lo + hi) / 2;
        if (sorted[mid] < (unsigned)p)
            lo = mid + 1;
        else
            hi = mid;
    }
    bounds[p] = lo;
}

// Radial gradient over the edges of each species pair (sorted positions
// bounds[p] .. bounds[p+1] of perm): for output (mu, xi)
//   G[p][mu][xi] += Q_xi(r_e) U_e[mu] + Q'_xi(r_e) V_e[mu]
// with Q the Chebyshev basis of basis.cpp:148-164.  Each block takes an equal
// slice of every bucket; threads stage 256 edges, then one thread per output
// sums them.  partial[block][p][mu][xi].
constexpr int RG_THREADS = 256;

template <bool RG>   // RG: radial families other than RBChebyshev present
__global__ void __launch_bounds__(RG_THREADS)
    k_radial_grad(int KK, int nmu, int R, double scaling, const long *__restrict__ bounds,
                  const int *__restrict__ perm, const double *__restrict__ rx,
                  const double *__restrict__ ry, const double *__restrict__ rz,
                  const PairParams *__restrict__ pairs, const double *__restrict__ uv,
                  double *__restrict__ partial)
{
    extern __shared__ double rsm[];
    double *Q = rsm;                          // [256][R]
    double *Qd = Q + RG_THREADS * R;          // [256][R]
    double *U = Qd + RG_THREADS * R;          // [256][nmu]
    double *V = U + RG_THREADS * nmu;         // [256][nmu]
    const int tid = threadIdx.x;
    const int nout = nmu * R;
    const int om = tid / R, ox = tid - om * R;   // output of this thread (tid < nout)
    for (int p = 0; p < KK; ++p) {
        const long b0 = bounds[p], b1 = bounds[p + 1];
        const long per = (b1 - b0 + gridDim.x - 1) / gridDim.x;
        const long lo = b0 + per * blockIdx.x;
        const long hi = min(b1, lo + per);
        const PairParams &pp = pairs[p];
        double acc = 0.0;
        for (long base = lo; base < hi; base += RG_THREADS) {
            const long i = base + tid;
            if (i < hi) {
                const int e = perm[i];
                const double x = rx[e], y = ry[e], z = rz[e];
                const double r = sqrt(__dadd_rn(__dadd_rn(__dmul_rn(x, x), __dmul_rn(y, y)),
                                                __dmul_rn(z, z)));
                for (int xi = 0; xi < R; ++xi) {   // zero where the family vanishes
                    Q[tid * R + xi] = 0.0;
                    Qd[tid * R + xi] = 0.0;
                }
                auto emit = [&](int xi, double q, double d) {
                    Q[tid * R + xi] = q;
                    Qd[tid * R + xi] = d;
                };
                if constexpr (RG)
                    radial_basis(pp, scaling, R, r, emit);
                else
                    radial_chebyshev(pp, scaling, R, r, emit);
                const double *u = uv + (size_t)e * 2 * nmu;
                for (int m = 0; m < nmu; ++m) {
                    U[tid * nmu + m] = u[m];
                    V[tid * nmu + m] = u[nmu + m];
                }
            }
            __syncthreads();
            if (tid < nout) {
                const int cnt = (int)min((long)RG_THREADS, hi - base);
                for (int k = 0; k < cnt; ++k)
                    acc = fma(Q[k * R + ox], U[k * nmu + om],
                              fma(Qd[k * R + ox], V[k * nmu + om], acc));
            }
            __syncthreads();
        }
        if (tid < nout)
            partial[((size_t)blockIdx.x * KK + p) * nout + tid] = acc;
    }
}

// out[j] = scale * sum_i in[i][j] (one block per column, fixed order)
__global__ void k_colsum(const double *__restrict__ in, long nrows, int ncols,
                         double *__restrict__ out)
{
    __shared__ double sh[256];
    const int j = blockIdx.x;
    double s = 0.0;
    for (long i = threadIdx.x; i < nrows; i += blockDim.x)
        s += in[i * ncols + j];
    s = block_sum<256>(s, sh);
    if (threadIdx.x == 0)
        out[j] = s;
}

// grad = [radial K*K x mu x R | species K | moment S] / norm; loss and metrics.
// RBPolyB pairs were evaluated with folded coefficients c' = c T_p (api.cu
// upload_model), so their radial gradient is T_p applied to the gradient of
// c': g[mu][i] = sum_j g'[mu][j] T_p(i, j), poly[(p R + i) R + j] = T_p(i, j)
__global__ void k_assemble(int KK, int mu_total, int nmu, int R, int K, int S,
                           const double *__restrict__ rsum, const double *__restrict__ tsum,
                           const double *__restrict__ gsum, const int *__restrict__ moment_energy,
                           const PairParams *__restrict__ pairs, const double *__restrict__ poly,
                           double inv_norm, double *__restrict__ grad, double *__restrict__ lm)
{
    const int rsize = KK * mu_total * R;
    const int n = rsize + K + S;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        double g;
        if (i < rsize) {
            const int p = i / (mu_total * R), rem = i - p * mu_total * R;
            const int m = rem / R, xi = rem - m * R;
            if (m >= nmu) {
                g = 0.0;
            } else if (poly && (pairs[p].type == RB_POLYB || pairs[p].type == RB_POLYB_COS)) {
                const double *t = poly + ((size_t)p * R + xi) * R;
                const double *gp = rsum + (size_t)(p * nmu + m) * R;
                g = 0.0;
                for (int j = 0; j < R; ++j)
                    g += gp[j] * t[j];
            } else {
                g = rsum[(p * nmu + m) * R + xi];
            }
        } else if (i < rsize + K) {
            g = tsum[TERMS + (i - rsize)];
        } else {
            const int e = moment_energy[i - rsize - K];
            g = e >= 0 ? gsum[e] : 0.0;
        }
        grad[i] = g * inv_norm;
    }
    if (blockIdx.x == 0 && threadIdx.x < TERMS) {
        lm[1 + threadIdx.x] = tsum[threadIdx.x];   // metrics (un-normalised)
        if (threadIdx.x == 0)
            lm[0] = tsum[0] * inv_norm;             // loss
    }
}

// Finite check of [loss, metrics, gradient] (the reference's
// training_finite_kernel, runtime/mtp/gpu-direct/mtp_gpu_direct.cu:5395-5420):
// first_bad receives the smallest index of a NaN or infinite value (it starts
// at INT_MAX).
__global__ void k_finite_check(int n, const double *__restrict__ v, int *__restrict__ first_bad)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        if (!isfinite(v[i]))
            atomicMin(first_bad, i);
}

// ---- host orchestration ------------------------------------------------------

static int labels_on_device(mtpb_context *c, const mtpb_labels *labels, int memory,
                            const double **te, const double **tf, const double **ts)
{
    const int S = c->nstruct, N = c->natoms;
    *te = labels->energy;
    *tf = labels->forces;
    *ts = labels->stress;
    if (memory == MTPB_MEMORY_DEVICE)
        return MTPB_OK;
    struct Up {
        const double *src;
        size_t n;
        const char *name;
        const double **dst;
    } ups[3] = {{labels->energy, (size_t)S, "train_label_e", te},
                {labels->forces, 3 * (size_t)N, "train_label_f", tf},
                {labels->stress, 9 * (size_t)S, "train_label_s", ts}};
    for (const Up &u : ups) {
        if (!u.src)
            continue;
        double *d = c->arena.get<double>(u.name, u.n + 1);
        if (!d)
            return fail(MTPB_ERR_MEMORY, "device allocation for labels failed");
        CUDA_TRY(cudaMemcpyAsync(d, u.src, sizeof(double) * u.n, cudaMemcpyHostToDevice,
                                 c->stream),
                 "upload labels");
        *u.dst = d;
    }
    return MTPB_OK;
}

// species-pair buckets of the current edge list (kept until the edges change)
static int pair_buckets(mtpb_context *c)
{
    TrainingState &t = c->train;
    const long E = c->nedges;
    const int K = c->model.K, KK = K * K;
    if (t.bucket_epoch == c->edge_epoch && t.perm && t.bounds)
        return MTPB_OK;
    unsigned *keys = c->arena.get<unsigned>("train_keys", E + 1);
    unsigned *keys_sorted = c->arena.get<unsigned>("train_keys_sorted", E + 1);
    int *ids = c->arena.get<int>("train_ids", E + 1);
    int *perm = c->arena.get<int>("train_perm", E + 1);
    long *bounds = c->arena.get<long>("train_bounds", KK + 2);
    if (!keys || !keys_sorted || !ids || !perm || !bounds)
        return fail(MTPB_ERR_MEMORY, "device allocation for edge buckets failed");
    if (E > 0x7fffffffL)
        return fail(MTPB_ERR_UNSUPPORTED, "more than 2^31 edges in one training batch");
    const int threads = 256;
    const unsigned blocks = (unsigned)((E + threads - 1) / threads);
    if (E > 0) {
        k_pair_keys<<<blocks, threads, 0, c->stream>>>(E, K, c->nb.center, c->nb.nbr, c->d_types,
                                                       c->nb.rx, c->nb.ry, c->nb.rz, c->d_pairs,
                                                       keys, ids);
        CUDA_TRY(cudaGetLastError(), "pair keys");
        int bits = 1;
        while ((1 << bits) <= KK)
            ++bits;
        size_t tmp_bytes = 0;
        CUDA_TRY(cub::DeviceRadixSort::SortPairs(nullptr, tmp_bytes, keys, keys_sorted, ids, perm,
                                                 (int)E, 0, bits, c->stream),
                 "edge sort size");
        void *tmp = c->arena.get("train_sort_tmp", tmp_bytes + 16);
        if (!tmp)
            return fail(MTPB_ERR_MEMORY, "device allocation for the edge sort failed");
        CUDA_TRY(cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, keys, keys_sorted, ids, perm,
                                                 (int)E, 0, bits, c->stream),
                 "edge sort");
        c->launches += 3;
    }
    k_bucket_bounds<<<(KK + 2 + 127) / 128, 128, 0, c->stream>>>(E, KK + 1, keys_sorted, bounds);
    CUDA_TRY(cudaGetLastError(), "bucket bounds");
    c->launches++;
    t.perm = perm;
    t.bounds = bounds;
    t.bucket_epoch = c->edge_epoch;
    return MTPB_OK;
}

int upload_training_program(mtpb_context *c)
{
    TrainingState &t = c->train;
    const DagPlan &plan = c->plan;
    std::vector<DagDevRec> recs = dag_grad_records(plan);
    t.recs = c->arena.get<DagDevRec>("train_dag", recs.size() + 1);
    // moment coefficient s -> its scalar moment in the graph's energy list
    std::vector<int> pos(c->model.M, -1), me(c->model.S());
    for (size_t i = 0; i < plan.energy_moments.size(); ++i)
        pos[plan.energy_moments[i]] = (int)i;
    for (int s = 0; s < c->model.S(); ++s)
        me[s] = pos[c->model.mapping[s]];
    t.moment_energy = c->arena.get<int>("train_moment_energy", me.size() + 1);
    if (!t.recs || !t.moment_energy)
        return fail(MTPB_ERR_MEMORY, "device allocation for the gradient program failed");
    CUDA_TRY(cudaMemcpyAsync(t.recs, recs.data(), sizeof(DagDevRec) * recs.size(),
                             cudaMemcpyHostToDevice, c->stream),
             "upload gradient graph");
    CUDA_TRY(cudaMemcpyAsync(t.moment_energy, me.data(), sizeof(int) * me.size(),
                             cudaMemcpyHostToDevice, c->stream),
             "upload moment map");
    t.h_recs = std::move(recs);
    t.ready = true;
    return MTPB_OK;
}

int loss_grad_compute(mtpb_context *c, const mtpb_labels *labels, const mtpb_loss_weights *w,
                      int norm_count, int memory, double *loss, double *metrics, double *grad)
{
    if (!c || !labels || !w)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    if (memory != MTPB_MEMORY_HOST && memory != MTPB_MEMORY_DEVICE)
        return fail(MTPB_ERR_ARGUMENT, "memory must be MTPB_MEMORY_HOST or MTPB_MEMORY_DEVICE");
    if (!c->have_list)
        return fail(MTPB_ERR_STATE, "build the neighbour list first (mtpb_build_neighbors)");
    if (norm_count < 0)
        return fail(MTPB_ERR_ARGUMENT, "norm_count must be >= 0");
    if (c->natoms != c->ntotal)
        return fail(MTPB_ERR_STATE, "the loss needs every atom as a centre "
                                    "(mtpb_set_center_count(ctx, 0) before the build)");
    const ModelHost &m = c->model;
    const int K = m.K, KK = K * K, S = c->nstruct, N = c->natoms;
    const long E = c->nedges;
    const int nmu = shape_desc(c->shape).nmu;
    if (K > 32)
        return fail(MTPB_ERR_UNSUPPORTED, "more than 32 species in training");
    if (nmu * m.R > RG_THREADS)
        return fail(MTPB_ERR_UNSUPPORTED, "radial basis too large for the gradient kernel");
    int rc = set_device(c);
    if (rc)
        return rc;
    if (!c->train.ready && (rc = upload_training_program(c)))
        return rc;
    cudaEvent_t *tev = c->train.ev;
    if (!tev[0])
        for (int i = 0; i < 7; ++i)
            CUDA_TRY(cudaEventCreate(&tev[i]), "cudaEventCreate");
    c->train.ev_valid = false;
    CUDA_TRY(cudaEventRecord(tev[0], c->stream), "event");
    // EFS pass: energies, forces, virials, basic moments and their adjoints;
    // without force and stress terms (the trainer's energy_only branch,
    // train_mtp.cpp:3858-3864) the reverse pass and the tangent moments are
    // skipped: the edge weights are then zero
    const bool use_f = labels->forces != nullptr && w->weight_force > 0;
    const bool use_s = labels->stress != nullptr && w->weight_stress > 0;
    const bool energy_only = !use_f && !use_s;
    mtpb_efs_output none{nullptr, nullptr, nullptr, nullptr};
    if ((rc = efs_compute(c, MTPB_MEMORY_DEVICE, &none, !energy_only)))
        return rc;
    CUDA_TRY(cudaEventRecord(tev[1], c->stream), "event");
    const double *d_energy = c->arena.get<double>("energy", S + 1);
    const double *d_forces = c->arena.get<double>("forces", 3 * (size_t)N + 1);
    const double *d_stress = c->arena.get<double>("stress", 9 * (size_t)S + 9);
    const double *basic = c->arena.get<double>("basic", (size_t)c->nslot * c->npad + 1);
    const double *adjoint = c->arena.get<double>("adjoint", (size_t)c->nslot * c->npad + 1);
    const double *te = nullptr, *tf = nullptr, *ts = nullptr;
    if ((rc = labels_on_device(c, labels, memory, &te, &tf, &ts)))
        return rc;
    const int NT = TERMS + K;
    int *aoff = c->arena.get<int>("train_atom_offsets", S + 1);
    double *dlde_atom = c->arena.get<double>("train_dlde", N + 1);
    double *dldf = c->arena.get<double>("train_dldf", 3 * (size_t)N + 3);
    double *dlds = c->arena.get<double>("train_dlds", 9 * (size_t)S + 9);
    double *terms = c->arena.get<double>("train_terms", (size_t)NT * S + NT);
    double *wx = c->arena.get<double>("train_wx", E + 1);
    double *wy = c->arena.get<double>("train_wy", E + 1);
    double *wz = c->arena.get<double>("train_wz", E + 1);
    double *tangent = c->arena.get<double>("train_tangent", (size_t)c->nslot * c->npad + 1);
    double *adjoint2 = c->arena.get<double>("train_adjoint2", (size_t)c->nslot * c->npad + 1);
    double *uv = c->arena.get<double>("train_uv", (size_t)E * 2 * nmu + 1);
    const int ne = (int)c->plan.energy_moments.size();
    const int grid = dag_grad_grid(c->plan, N);
    double *epart = c->arena.get<double>("train_energy_part", (size_t)grid * ne + 1);
    const size_t nscr = dag_grad_scratch_doubles(c->plan);
    double *gscratch = nscr ? c->arena.get<double>("train_dag_rows", nscr) : nullptr;
    if (nscr && !gscratch)
        return fail(MTPB_ERR_MEMORY, "device allocation for the dual graph rows failed");
    int rg_grid = 0;
    {
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        rg_grid = 2 * sms;
    }
    const int nout = nmu * m.R;
    double *rpart = c->arena.get<double>("train_radial_part", (size_t)rg_grid * KK * nout + 1);
    const int ncoef = m.coeff_count();
    double *sums = c->arena.get<double>("train_sums", (size_t)KK * nout + NT + ne + 3);
    double *d_out = c->arena.get<double>("train_out", (size_t)ncoef + 8 + 1);
    int *nonfinite = c->arena.get<int>("train_nonfinite", 1);
    if (!aoff || !dlde_atom || !dldf || !dlds || !terms || !wx || !wy || !wz || !tangent ||
        !adjoint2 || !uv || !epart || !rpart || !sums || !d_out || !d_energy || !basic || !adjoint ||
        !nonfinite)
        return fail(MTPB_ERR_MEMORY, "device allocation for the gradient failed");
    double *rsum = sums, *tsum = sums + (size_t)KK * nout, *gsum = tsum + NT;
    CUDA_TRY(cudaMemcpyAsync(aoff, c->h_atom_offsets.data(), sizeof(int) * (S + 1),
                             cudaMemcpyHostToDevice, c->stream),
             "upload offsets");
    LossParams lp{w->weight_eng, w->weight_force, w->weight_stress, w->weight_eng_power,
                  w->weight_force_power, w->weight_stress_power,
                  te != nullptr && w->weight_eng > 0, tf != nullptr && w->weight_force > 0,
                  ts != nullptr && w->weight_stress > 0, K};
    NvtxRange range_loss("mtpb:train_loss_weights");
    if (S > 0) {
        k_loss_struct<<<S, LOSS_THREADS, 0, c->stream>>>(aoff, c->d_types, d_energy, d_forces,
                                                         d_stress, te, tf, ts, lp, dlde_atom,
                                                         dldf, dlds, terms);
        CUDA_TRY(cudaGetLastError(), "loss");
        c->launches++;
    }
    if (E > 0 && !energy_only) {
        k_edge_weights<<<(unsigned)((E + 255) / 256), 256, 0, c->stream>>>(
            E, c->nb.center, c->nb.nbr, c->nb.struct_of, c->nb.rx, c->nb.ry, c->nb.rz, dldf, dlds,
            wx, wy, wz);
        CUDA_TRY(cudaGetLastError(), "edge weights");
        c->launches++;
    } else if (E > 0) {
        for (double *p : {wx, wy, wz})
            CUDA_TRY(cudaMemsetAsync(p, 0, sizeof(double) * E, c->stream), "zero weights");
    }
    if ((rc = pair_buckets(c)))
        return rc;
    CUDA_TRY(cudaEventRecord(tev[2], c->stream), "event");
    EdgeArgs a = edge_args(c, N, c->d_types, c->nb.offsets, c->nb.nbr, c->nb.rx, c->nb.ry,
                           c->nb.rz);
    if (energy_only)
        CUDA_TRY(cudaMemsetAsync(tangent, 0, sizeof(double) * (size_t)c->nslot * c->npad,
                                 c->stream),
                 "zero tangent");
    else {
        NvtxRange range("mtpb:train_tangent_moments");
        CUDA_TRY(launch_moments_tangent(c->shape, a, wx, wy, wz, tangent, c->stream), "tangent");
    }
    CUDA_TRY(cudaEventRecord(tev[3], c->stream), "event");
    NvtxRange range_dual("mtpb:train_dual_graph_edge_grad");
    CUDA_TRY(launch_dag_grad(c->plan, c->train.recs, c->d_phase_row0, grid, c->nslot, N, c->npad,
                             basic, tangent, dlde_atom, adjoint2, epart, gscratch, c->d_err,
                             c->stream),
             "dual graph");
    CUDA_TRY(cudaEventRecord(tev[4], c->stream), "event");
    CUDA_TRY(launch_edge_grad(c->shape, a, wx, wy, wz, adjoint, adjoint2, uv, c->stream),
             "edge gradient");
    CUDA_TRY(cudaEventRecord(tev[5], c->stream), "event");
    c->launches += (energy_only ? 0 : grad_kernel_launches(c->shape, false)) + 1 +
                   grad_kernel_launches(c->shape, true);
    const size_t rg_smem = sizeof(double) * RG_THREADS * (2 * m.R + 2 * nmu);
    auto rg_kern = a.rb_generic ? k_radial_grad<true> : k_radial_grad<false>;
    CUDA_TRY(cudaFuncSetAttribute(rg_kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)rg_smem),
             "radial gradient attribute");
    rg_kern<<<rg_grid, RG_THREADS, rg_smem, c->stream>>>(
        KK, nmu, m.R, m.scaling, c->train.bounds, c->train.perm, c->nb.rx, c->nb.ry, c->nb.rz,
        c->d_pairs, uv, rpart);
    CUDA_TRY(cudaGetLastError(), "radial gradient");
    k_colsum<<<KK * nout, 256, 0, c->stream>>>(rpart, rg_grid, KK * nout, rsum);
    k_colsum<<<NT, 256, 0, c->stream>>>(terms, S, NT, tsum);
    if (ne > 0)
        k_colsum<<<ne, 256, 0, c->stream>>>(epart, grid, ne, gsum);
    const int cnt = norm_count > 0 ? norm_count : S;
    const double inv_norm = cnt > 0 ? 1.0 / cnt : 1.0;
    double *d_grad = d_out + 8;
    k_assemble<<<(ncoef + 255) / 256, 256, 0, c->stream>>>(
        KK, m.mu, nmu, m.R, K, m.S(), rsum, tsum, gsum, c->train.moment_energy, c->d_pairs,
        c->d_poly, inv_norm, d_grad, d_out);
    CUDA_TRY(cudaGetLastError(), "assemble");
    CUDA_TRY(cudaMemsetAsync(nonfinite, 0x7f, sizeof(int), c->stream), "clear finite check");
    k_finite_check<<<(ncoef + 8 + 255) / 256, 256, 0, c->stream>>>(ncoef + 8, d_out, nonfinite);
    CUDA_TRY(cudaGetLastError(), "finite check");
    c->train.nonfinite = nonfinite;
    c->launches += ne > 0 ? 6 : 5;
    const cudaMemcpyKind kind =
        memory == MTPB_MEMORY_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
    if (loss)
        CUDA_TRY(cudaMemcpyAsync(loss, d_out, sizeof(double), kind, c->stream), "copy loss");
    if (metrics)
        CUDA_TRY(cudaMemcpyAsync(metrics, d_out + 1, sizeof(double) * TERMS, kind, c->stream),
                 "copy metrics");
    if (grad)
        CUDA_TRY(cudaMemcpyAsync(grad, d_grad, sizeof(double) * ncoef, kind, c->stream),
                 "copy gradient");
    CUDA_TRY(cudaEventRecord(tev[6], c->stream), "event");
    c->train.ev_valid = true;
    if (memory == MTPB_MEMORY_HOST) {
        CUDA_TRY(cudaStreamSynchronize(c->stream), "gradient");
        if ((rc = check_device_error(c)))
            return rc;
        long bad = -1;
        return training_values_status(c, &bad);
    }
    return MTPB_OK;
}

int training_values_status(mtpb_context *c, long *first_bad)
{
    *first_bad = -1;
    if (!c->train.nonfinite)
        return fail(MTPB_ERR_STATE, "no mtpb_loss_grad call to check");
    int rc = set_device(c);
    if (rc)
        return rc;
    int bad = 0;
    CUDA_TRY(cudaMemcpyAsync(&bad, c->train.nonfinite, sizeof(int), cudaMemcpyDeviceToHost,
                             c->stream),
             "read finite check");
    CUDA_TRY(cudaStreamSynchronize(c->stream), "finite check");
    if (bad == 0x7f7f7f7f)
        return MTPB_OK;
    *first_bad = bad;
    std::string where = bad == 0 ? "the loss"
                        : bad <= TERMS ? "metric " + std::to_string(bad - 1)
                                       : "gradient component " + std::to_string(bad - 1 - TERMS);
    return fail(MTPB_ERR_NONFINITE, "non-finite training value: " + where +
                                        " (a label, weight or coefficient is NaN or infinite, "
                                        "or the loss overflowed)");
}

} // namespace mtpb
