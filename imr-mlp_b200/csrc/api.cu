// api.cu -- C ABI implementation (include/mtpb200.h): context lifetime,
// validation, uploads and the EFS pipeline.
#include "context.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <new>
#include <string>
#include <vector>

using namespace mtpb;

namespace mtpb {
static thread_local std::string g_last_error;

int fail(int status, const std::string &msg)
{
    g_last_error = msg;
    return status;
}

int cuda_fail(cudaError_t e, const char *where)
{
    g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
    return e == cudaErrorMemoryAllocation ? MTPB_ERR_MEMORY : MTPB_ERR_CUDA;
}
} // namespace mtpb



namespace mtpb {

int set_device(mtpb_context *c)
{
    CUDA_TRY(cudaSetDevice(c->device), "cudaSetDevice");
    return MTPB_OK;
}

static bool copy_model(const mtpb_model_view *v, ModelHost &m, std::string *err)
{
    if (!v) {
        *err = "model view is NULL";
        return false;
    }
    if (v->species_count <= 0 || v->radial_func_count <= 0 || v->rb_size <= 0 ||
        v->alpha_index_basic_count <= 0 || v->alpha_index_times_count < 0 ||
        v->alpha_scalar_moments < 0 || v->alpha_moments_count <= 0) {
        *err = "model counts must be positive";
        return false;
    }
    if (!v->min_dist || !v->max_dist || !v->alpha_index_basic || !v->alpha_moment_mapping ||
        !v->radial_coeffs || !v->species_coeffs || !v->moment_coeffs ||
        (v->alpha_index_times_count > 0 && !v->alpha_index_times)) {
        *err = "model view has a NULL array";
        return false;
    }
    m.K = v->species_count;
    m.mu = v->radial_func_count;
    m.R = v->rb_size;
    m.split = v->radial_basis_split ? 1 : 0;
    m.M = v->alpha_moments_count;
    m.scaling = v->scaling;
    const int pairs = m.split ? m.K * m.K : 1;
    m.min_dist.assign(v->min_dist, v->min_dist + pairs);
    m.max_dist.assign(v->max_dist, v->max_dist + pairs);
    m.basic.assign(v->alpha_index_basic, v->alpha_index_basic + 4 * v->alpha_index_basic_count);
    if (v->alpha_index_times_count > 0)
        m.times.assign(v->alpha_index_times, v->alpha_index_times + 4 * v->alpha_index_times_count);
    m.mapping.assign(v->alpha_moment_mapping, v->alpha_moment_mapping + v->alpha_scalar_moments);
    m.radial.assign(v->radial_coeffs, v->radial_coeffs + m.K * m.K * m.mu * m.R);
    m.species.assign(v->species_coeffs, v->species_coeffs + m.K);
    m.moment.assign(v->moment_coeffs, v->moment_coeffs + v->alpha_scalar_moments);
    m.family.clear();
    if (v->radial_family) {
        const int nf = m.split ? m.K * m.K : 1;
        for (int p = 0; p < nf; ++p) {
            const mtpb_radial_family &f = v->radial_family[p];
            RadialFamily h;
            h.type = f.type;
            h.cutoff = f.cutoff_type;
            h.shift = f.shift_type;
            h.flipped = f.one_minus_chebyshev ? 1 : 0;
            h.b = f.b;
            h.r1 = f.r1;
            h.r2 = f.r2;
            h.lambda = f.lambda;
            h.scale_lambda = f.scale_lambda;
            if (f.type == MTPB_RB_POLYB || f.type == MTPB_RB_POLYB_COS) {
                if (!f.poly_matrix || !f.poly_norm) {
                    *err = "RBPolyB / RBPolyBCos need poly_matrix and poly_norm";
                    return false;
                }
                h.poly_matrix.assign(f.poly_matrix, f.poly_matrix + (size_t)m.R * m.R);
                h.poly_norm.assign(f.poly_norm, f.poly_norm + m.R);
            }
            m.family.push_back(h);
        }
    }
    return true;
}

// Graph kernel geometry: 16 atoms per block with the rows in shared memory
// when they fit, else 8 atoms, else rows in an L2-resident global slice per
// persistent block (one block per SM).  MTPB_DAG_ATOMS=8|16 forces the
// shared-memory width where it fits.
static int dag_configure(mtpb_context *c)
{
    DagPlan &p = c->plan;
    int optin = 0, sms = 0;
    CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c->device),
             "device attribute");
    CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->device),
             "device attribute");
    // static shared arrays of the graph kernels: at most 64 x 16 energy
    // partials (8 KB), the mbarriers and the phase table
    const size_t limit = (size_t)optin - 10 * 1024;
    auto fits = [&](int atoms) {
        return dag_ring_bytes(atoms) + (size_t)p.nrows * atoms * sizeof(double) <= limit;
    };
    p.global_rows = false;
    p.grid = sms;
    if (c->dag_atoms_env && fits(c->dag_atoms_env))
        p.atoms = c->dag_atoms_env;
    else if (fits(16))
        p.atoms = 16;
    else if (fits(8))
        p.atoms = 8;
    else {
        p.atoms = 16;
        p.global_rows = true;
    }
    p.grad_global_rows = dag_grad_smem_bytes(p, false) > limit;
    if (c->force_global_rows) {   // MTPB_DAG_GLOBAL_ROWS=1: test the large-graph mode
        p.atoms = 16;
        p.global_rows = true;
        p.grad_global_rows = true;
    }
    p.grad_grid = sms;
    return MTPB_OK;
}

static int upload_model(mtpb_context *c)
{
    int rc = MTPB_OK;
    const ModelHost &m = c->model;
    const int KK = m.K * m.K;
    std::vector<PairParams> pp(KK);
    for (int p = 0; p < KK; ++p) {
        const double rmin = m.pair_min(p), rmax = m.pair_max(p);
        const RadialFamily f = m.pair_family(p);
        PairParams &q = pp[p];
        q = PairParams{};
        // the constants the reference bases compute once (basis.cpp setup(),
        // cutoff.cpp / xtrans.cpp constructors)
        q.pu = rmax + rmin;
        q.su = rmax - rmin;
        q.mult = 2.0 / (rmax - rmin);
        q.rmax = rmax;
        q.rmin = rmin;
        q.inv_range = 1.0 / (rmax - rmin);
        q.irpi = M_PI / rmax;
        q.cfreq = M_PI / (rmax - rmin);
        q.slope = 2.0 / (rmax - rmin);
        q.b = f.b;
        q.r1 = f.r1;
        q.r2 = f.r2;
        q.lambda = f.lambda;
        q.scale_lambda = f.scale_lambda;
        q.den = f.lambda != 0.0 ? std::expm1(f.lambda) : 0.0;
        q.sden = f.scale_lambda != 0.0 ? std::tanh(f.scale_lambda) : 0.0;
        q.type = f.type;
        q.cutoff = f.type == RB_POLYB_COS ? CUT_COSINE_LEFT : f.cutoff;
        q.shift = f.shift;
        q.flipped = f.flipped;
    }
    // RBPolyB / RBPolyBCos (runtime/mtp/radial_basis.h:223-290):
    // Q_i = fc sum_j M(i, j) N_j s (max - r)^(j + first).  The device evaluates
    // the powers and the matrix and normalisations are folded into the
    // coefficients, c'[mu][j] = N_j sum_i c[mu][i] M(i, j), so that
    // f_mu = sum_j c'[mu][j] s (max - r)^(j + first) fc; the same sums in
    // another order (checked against the reference loader's matrix in the
    // tests).  T_p(i, j) = N_j M(i, j) maps gradients back (training.cu).
    std::vector<double> radial_dev = m.radial;
    std::vector<double> poly_t;
    for (int p = 0; p < KK; ++p) {
        const RadialFamily f = m.pair_family(p);
        if (f.type != RB_POLYB && f.type != RB_POLYB_COS)
            continue;
        const int R = m.R;
        if (poly_t.empty())
            poly_t.assign((size_t)KK * R * R, 0.0);
        for (int i = 0; i < R; ++i)
            for (int j = 0; j < R; ++j)
                poly_t[((size_t)p * R + i) * R + j] = f.poly_norm[j] * f.poly_matrix[i + (size_t)j * R];
        for (int mu = 0; mu < m.mu; ++mu) {
            const double *cin = &m.radial[((size_t)p * m.mu + mu) * R];
            double *cout = &radial_dev[((size_t)p * m.mu + mu) * R];
            for (int j = 0; j < R; ++j) {
                double acc = 0.0;
                for (int i = 0; i < R; ++i)
                    acc += cin[i] * f.poly_matrix[i + (size_t)j * R];
                cout[j] = f.poly_norm[j] * acc;
            }
        }
    }
    c->d_poly = nullptr;
    if (!poly_t.empty()) {
        c->d_poly = c->arena.get<double>("model_poly", poly_t.size());
        if (!c->d_poly)
            return fail(MTPB_ERR_MEMORY, "device allocation for the model failed");
        CUDA_TRY(cudaMemcpyAsync(c->d_poly, poly_t.data(), sizeof(double) * poly_t.size(),
                                 cudaMemcpyHostToDevice, c->stream),
                 "upload PolyB matrices");
    }
    c->d_radial = c->arena.get<double>("model_radial", m.radial.size());
    c->d_species = c->arena.get<double>("model_species", m.K);
    c->d_pairs = c->arena.get<PairParams>("model_pairs", KK);
    c->d_recs = c->arena.get<DagDevRec>("model_dag", c->plan.recs.size());
    std::vector<int> row0(c->plan.phase_rows.size() + 1, 0);
    for (size_t i = 0; i < c->plan.phase_rows.size(); ++i)
        row0[i + 1] = row0[i] + c->plan.phase_rows[i];
    c->d_phase_row0 = c->arena.get<int>("model_dag_row0", row0.size());
    if (!c->d_err) {
        c->d_err = c->arena.get<int>("err_flag", 4);
        if (!c->d_err)
            return fail(MTPB_ERR_MEMORY, "device allocation failed");
        CUDA_TRY(cudaMemsetAsync(c->d_err, 0, sizeof(int), c->stream), "memset");
    }
    if (!c->d_radial || !c->d_species || !c->d_pairs || !c->d_recs || !c->d_phase_row0)
        return fail(MTPB_ERR_MEMORY, "device allocation for the model failed");
    CUDA_TRY(cudaMemcpyAsync(c->d_radial, radial_dev.data(), sizeof(double) * radial_dev.size(),
                             cudaMemcpyHostToDevice, c->stream),
             "upload radial");
    CUDA_TRY(cudaMemcpyAsync(c->d_species, m.species.data(), sizeof(double) * m.K,
                             cudaMemcpyHostToDevice, c->stream),
             "upload species");
    CUDA_TRY(cudaMemcpyAsync(c->d_pairs, pp.data(), sizeof(PairParams) * KK,
                             cudaMemcpyHostToDevice, c->stream),
             "upload pairs");
    if ((rc = dag_configure(c)))
        return rc;
    c->h_recs = dag_device_records(c->plan);
    CUDA_TRY(cudaMemcpyAsync(c->d_recs, c->h_recs.data(), sizeof(DagDevRec) * c->h_recs.size(),
                             cudaMemcpyHostToDevice, c->stream),
             "upload graph");
    CUDA_TRY(cudaMemcpyAsync(c->d_phase_row0, row0.data(), sizeof(int) * row0.size(),
                             cudaMemcpyHostToDevice, c->stream),
             "upload graph phases");
    CUDA_TRY(cudaStreamSynchronize(c->stream), "model upload");
    c->train.ready = false;   // the gradient program follows the new records
    return MTPB_OK;
}

EdgeArgs edge_args(const mtpb_context *c, int ncenter, const int *types, const int *offsets,
                   const int *nbr, const double *rx, const double *ry, const double *rz)
{
    EdgeArgs a{};
    a.natoms = ncenter;
    a.npad = c->npad;
    a.types = types;
    a.offsets = offsets;
    a.nbr = nbr;
    a.rx = rx;
    a.ry = ry;
    a.rz = rz;
    // species pairs per edge exist for the lists built by mtpb_build_neighbors
    a.pair = (nbr == c->nb.nbr && c->nb.pair) ? c->nb.pair : nullptr;
    a.group_maxdeg = c->d_group_maxdeg;
    a.K = c->model.K;
    a.R = c->model.R;
    a.mu_total = c->model.mu;
    a.scaling = c->model.scaling;
    a.radial = c->d_radial;
    a.pairs = c->d_pairs;
    a.rb_generic = 0;
    for (const RadialFamily &f : c->model.family)
        a.rb_generic |= f.type != RB_CHEBYSHEV;
    return a;
}

// forward moments -> graph -> reverse moments for ncenter centres.
int run_moments(mtpb_context *c, int ncenter, const int *types, const int *offsets,
                const int *nbr, const double *rx, const double *ry, const double *rz,
                double *site_energy, double *dx, double *dy, double *dz, bool reverse,
                long nedges, bool beyond_cutoff, const EdgeRefresh *refresh)
{
    c->npad = ((ncenter + 31) / 32) * 32;
    c->d_group_maxdeg = c->arena.get<int>("group_maxdeg", c->npad / 32 + 1);
    double *basic = c->arena.get<double>("basic", (size_t)c->nslot * c->npad + 1);
    double *adjoint = c->arena.get<double>("adjoint", (size_t)c->nslot * c->npad + 1);
    if (!c->d_group_maxdeg || !basic || !adjoint)
        return fail(MTPB_ERR_MEMORY, "device allocation for moments failed");
    CUDA_TRY(launch_group_maxdeg(ncenter, offsets, c->d_group_maxdeg, c->stream), "group_maxdeg");
    c->launches++;
    EdgeArgs a = edge_args(c, ncenter, types, offsets, nbr, rx, ry, rz);
    // lists that hold pairs beyond the cutoff (a skin, a caller's list) are
    // staged through their active edges; the training kernels keep the full
    // list and its degree table
    if (refresh && !(beyond_cutoff && nedges > 0 && ncenter > 0))
        return fail(MTPB_ERR_STATE, "edge refresh without an active-edge pass");
    if (beyond_cutoff && nedges > 0 && ncenter > 0) {
        ActiveEdges act;
        act.active = c->arena.get<int>("active_edges", nedges + 1);
        act.nact = c->arena.get<int>("active_count", ncenter + 1);
        act.group_maxdeg = c->arena.get<int>("group_maxdeg_active", c->npad / 32 + 1);
        act.cx = c->arena.get<double>("active_rx", nedges + 1);
        act.cy = c->arena.get<double>("active_ry", nedges + 1);
        act.cz = c->arena.get<double>("active_rz", nedges + 1);
        act.cnbr = c->arena.get<int>("active_nbr", nedges + 1);
        act.cpair = c->arena.get<int>("active_pair", nedges + 1);
        if (!act.active || !act.nact || !act.group_maxdeg || !act.cx || !act.cy || !act.cz ||
            !act.cnbr || !act.cpair)
            return fail(MTPB_ERR_MEMORY, "device allocation for the active edges failed");
        NvtxRange range("mtpb:active_edges");
        CUDA_TRY(launch_active_edges(a, act, refresh, reverse ? dx : nullptr,
                                     reverse ? dy : nullptr, reverse ? dz : nullptr, c->stream),
                 "active edges");
        c->launches += 2;
        // the moment kernels stage the compacted active edges
        a.active = act.active;
        a.nact = act.nact;
        a.group_maxdeg = act.group_maxdeg;
        a.nbr = act.cnbr;
        a.rx = act.cx;
        a.ry = act.cy;
        a.rz = act.cz;
        a.pair = act.cpair;
    }
    CUDA_TRY(cudaEventRecord(c->ev[1], c->stream), "event");
    {
        NvtxRange range("mtpb:moments_fwd");
        CUDA_TRY(launch_moments_fwd(c->shape, a, basic, c->stream), "moments forward");
    }
    c->launches += moment_kernel_parts(c->shape, false);
    CUDA_TRY(cudaEventRecord(c->ev[2], c->stream), "event");
    double *gscratch = nullptr;
    if (c->plan.global_rows) {
        gscratch = c->arena.get<double>("dag_rows", (size_t)c->plan.grid * c->plan.nrows *
                                                        c->plan.atoms);
        if (!gscratch)
            return fail(MTPB_ERR_MEMORY, "device allocation for graph rows failed");
    }
    {
        NvtxRange range("mtpb:moment_graph");
        CUDA_TRY(launch_dag(c->plan, c->d_recs, c->d_phase_row0, c->nslot, ncenter, c->npad,
                            types, c->d_species, basic, adjoint, site_energy, gscratch, c->d_err,
                            c->stream),
                 "moment graph");
    }
    c->launches++;
    CUDA_TRY(cudaEventRecord(c->ev[3], c->stream), "event");
    if (reverse) {   // energy-only calls stop at the site energies and adjoints
        NvtxRange range("mtpb:moments_rev");
        CUDA_TRY(launch_moments_rev(c->shape, a, adjoint, dx, dy, dz, c->stream),
                 "moments reverse");
        c->launches += moment_kernel_parts(c->shape, true);
    }
    CUDA_TRY(cudaEventRecord(c->ev[4], c->stream), "event");
    return MTPB_OK;
}

int check_device_error(mtpb_context *c)
{
    int flag = 0;
    CUDA_TRY(cudaMemcpy(&flag, c->d_err, sizeof(int), cudaMemcpyDeviceToHost), "read error flag");
    if (flag) {
        CUDA_TRY(cudaMemset(c->d_err, 0, sizeof(int)), "clear error flag");
        return fail(MTPB_ERR_CUDA, "a device-side wait gave up (record stream did not arrive); "
                                   "results of this call are invalid");
    }
    return MTPB_OK;
}

static int check_structures(const mtpb_context *c, const mtpb_structures *in)
{
    if (!in)
        return fail(MTPB_ERR_ARGUMENT, "structures is NULL");
    if (in->n_structures < 0)
        return fail(MTPB_ERR_ARGUMENT, "n_structures must be >= 0");
    if (in->n_structures > 0 && (!in->atom_offsets || !in->cells))
        return fail(MTPB_ERR_ARGUMENT, "atom_offsets and cells are required");
    return MTPB_OK;
}

} // namespace mtpb

// ============================================================================
extern "C" {

const char *mtpb_last_error(void) { return mtpb::g_last_error.c_str(); }

int mtpb_abi_version(void) { return MTPB_ABI_VERSION; }

int mtpb_device_count(int *count)
{
    if (!count)
        return fail(MTPB_ERR_ARGUMENT, "count is NULL");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *count = 0;
        return cuda_fail(e, "cudaGetDeviceCount");
    }
    *count = n;
    return MTPB_OK;
}

int mtpb_create(int device, const mtpb_model_view *view, mtpb_context **out)
{
    if (!out)
        return fail(MTPB_ERR_ARGUMENT, "ctx output pointer is NULL");
    *out = nullptr;
    mtpb_context *c = nullptr;
    try {
        c = new mtpb_context();
    } catch (const std::bad_alloc &) {
        return fail(MTPB_ERR_MEMORY, "host allocation failed");
    }
    std::string err;
    int rc = MTPB_OK;
    do {
        if (!copy_model(view, c->model, &err) || !validate_model(c->model, &err)) {
            rc = fail(MTPB_ERR_ARGUMENT, err);
            break;
        }
        if (const char *v = std::getenv("MTPB_DAG_ATOMS"))
            c->dag_atoms_env = std::atoi(v) == 16 ? 16 : 8;
        if (const char *v = std::getenv("MTPB_DAG_GLOBAL_ROWS"))
            c->force_global_rows = std::atoi(v) == 1;
        c->shape = select_shape(c->model, &err);
        if (c->shape < 0) {
            rc = fail(MTPB_ERR_UNSUPPORTED, err);
            break;
        }
        c->nslot = shape_desc(c->shape).nslot;
        if (!build_slot_map(c->model, c->shape, c->slot_of_basic, &err) ||
            !build_dag_plan(c->model, c->shape, c->slot_of_basic, c->plan, &err)) {
            rc = fail(MTPB_ERR_UNSUPPORTED, err);
            break;
        }
        int ndev = 0;
        cudaError_t e = cudaGetDeviceCount(&ndev);
        if (e != cudaSuccess || ndev == 0) {
            cudaGetLastError();
            rc = fail(MTPB_ERR_CUDA, std::string("no CUDA device available: ") +
                                         cudaGetErrorString(e));
            break;
        }
        if (device < 0 || device >= ndev) {
            rc = fail(MTPB_ERR_ARGUMENT, "device index out of range");
            break;
        }
        c->device = device;
        if ((rc = set_device(c)) != MTPB_OK)
            break;
        cudaDeviceProp prop;
        if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) {
            rc = cuda_fail(e, "cudaGetDeviceProperties");
            break;
        }
        if (prop.major < 10) {
            rc = fail(MTPB_ERR_UNSUPPORTED, "this library is built for sm_100a (B200) devices");
            break;
        }
        if ((e = cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking)) !=
            cudaSuccess) {
            rc = cuda_fail(e, "cudaStreamCreate");
            break;
        }
        c->stream = c->own_stream;
        for (auto &ev : c->ev)
            if ((e = cudaEventCreate(&ev)) != cudaSuccess) {
                rc = cuda_fail(e, "cudaEventCreate");
                break;
            }
        if (rc != MTPB_OK)
            break;
        if ((e = cudaEventCreateWithFlags(&c->stage_ev, cudaEventDisableTiming)) !=
            cudaSuccess) {
            rc = cuda_fail(e, "cudaEventCreate");
            break;
        }
        rc = upload_model(c);
    } while (false);
    if (rc != MTPB_OK) {
        mtpb_destroy(c);
        return rc;
    }
    *out = c;
    return MTPB_OK;
}

int mtpb_destroy(mtpb_context *c)
{
    if (!c)
        return MTPB_OK;
    if (c->stream) {
        cudaSetDevice(c->device);
        cudaStreamSynchronize(c->stream);
    }
    c->arena.release();
    for (auto &ev : c->ev)
        if (ev)
            cudaEventDestroy(ev);
    for (auto &ev : c->train.ev)
        if (ev)
            cudaEventDestroy(ev);
    if (c->stage_ev)
        cudaEventDestroy(c->stage_ev);
    if (c->h_stage)
        cudaFreeHost(c->h_stage);
    if (c->own_stream)
        cudaStreamDestroy(c->own_stream);
    delete c;
    return MTPB_OK;
}

int mtpb_update_coefficients(mtpb_context *c, const double *radial, const double *species,
                             const double *moment)
{
    if (!c || !radial || !species || !moment)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    ModelHost m = c->model;
    std::copy(radial, radial + m.radial.size(), m.radial.begin());
    std::copy(species, species + m.K, m.species.begin());
    std::copy(moment, moment + m.S(), m.moment.begin());
    std::string err;
    if (!validate_model(m, &err))
        return fail(MTPB_ERR_ARGUMENT, err);
    DagPlan plan;
    if (!build_dag_plan(m, c->shape, c->slot_of_basic, plan, &err))
        return fail(MTPB_ERR_UNSUPPORTED, err);
    int rc = set_device(c);
    if (rc)
        return rc;
    CUDA_TRY(cudaStreamSynchronize(c->stream), "sync");
    c->model = std::move(m);
    c->plan = std::move(plan);
    c->have_efs = false;
    return upload_model(c);
}

int mtpb_set_stream(mtpb_context *c, void *stream)
{
    if (!c)
        return fail(MTPB_ERR_ARGUMENT, "ctx is NULL");
    int rc = set_device(c);
    if (rc)
        return rc;
    CUDA_TRY(cudaStreamSynchronize(c->stream), "sync");
    c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own_stream;
    return MTPB_OK;
}

int mtpb_cutoff(const mtpb_context *c, double *cutoff)
{
    if (!c || !cutoff)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    *cutoff = c->model.cutoff();
    return MTPB_OK;
}

int mtpb_set_skin(mtpb_context *c, double skin)
{
    if (!c || !(skin >= 0) || !std::isfinite(skin))
        return fail(MTPB_ERR_ARGUMENT, "skin must be a finite non-negative number");
    c->skin = skin;
    c->have_list = false;
    return MTPB_OK;
}

int mtpb_set_center_count(mtpb_context *c, int center_count)
{
    if (!c || center_count < 0)
        return fail(MTPB_ERR_ARGUMENT, "center_count must be >= 0");
    c->center_count_req = center_count;
    c->have_list = false;
    return MTPB_OK;
}

int mtpb_build_neighbors(mtpb_context *c, const mtpb_structures *in, int memory)
{
    mtpb::NvtxRange range("mtpb:build_neighbors");
    if (!c)
        return fail(MTPB_ERR_ARGUMENT, "ctx is NULL");
    int rc = check_structures(c, in);
    if (rc)
        return rc;
    if ((rc = set_device(c)))
        return rc;
    const int S = in->n_structures;
    const bool dev = memory == MTPB_MEMORY_DEVICE;
    c->have_list = false;
    c->have_efs = false;
    // host copies of the (small) per-structure arrays
    c->h_atom_offsets.assign(S + 1, 0);
    c->h_cells.assign(9 * (size_t)S, 0.0);
    std::vector<int> pbc(3 * (size_t)S, 1);
    if (S > 0) {
        if (dev) {
            CUDA_TRY(cudaMemcpy(c->h_atom_offsets.data(), in->atom_offsets, sizeof(int) * (S + 1),
                                cudaMemcpyDeviceToHost),
                     "read atom_offsets");
            CUDA_TRY(cudaMemcpy(c->h_cells.data(), in->cells, sizeof(double) * 9 * S,
                                cudaMemcpyDeviceToHost),
                     "read cells");
            if (in->pbc)
                CUDA_TRY(cudaMemcpy(pbc.data(), in->pbc, sizeof(int) * 3 * S,
                                    cudaMemcpyDeviceToHost),
                         "read pbc");
        } else {
            std::copy(in->atom_offsets, in->atom_offsets + S + 1, c->h_atom_offsets.begin());
            std::copy(in->cells, in->cells + 9 * (size_t)S, c->h_cells.begin());
            if (in->pbc)
                std::copy(in->pbc, in->pbc + 3 * (size_t)S, pbc.begin());
        }
    }
    if (c->h_atom_offsets[0] != 0)
        return fail(MTPB_ERR_ARGUMENT, "atom_offsets[0] must be 0");
    for (int s = 0; s < S; ++s)
        if (c->h_atom_offsets[s + 1] < c->h_atom_offsets[s])
            return fail(MTPB_ERR_ARGUMENT, "atom_offsets must be non-decreasing");
    const int N = c->h_atom_offsets[S];
    if (N > 0 && (!in->positions || !in->types))
        return fail(MTPB_ERR_ARGUMENT, "positions and types are required");
    const double cut = c->model.cutoff() + c->skin;
    std::vector<NbStruct> ns(S);
    int cells = 0;
    for (int s = 0; s < S; ++s) {
        std::string err;
        if (!prepare_struct(&c->h_cells[9 * (size_t)s], &pbc[3 * (size_t)s], cut, ns[s], &err))
            return fail(MTPB_ERR_UNSUPPORTED, "structure " + std::to_string(s) + ": " + err);
        ns[s].cell0 = cells;
        const long nc = (long)ns[s].ncell[0] * ns[s].ncell[1] * ns[s].ncell[2];
        if (cells + nc > (1L << 30))
            return fail(MTPB_ERR_UNSUPPORTED, "too many neighbour cells");
        cells += (int)nc;
    }
    // device inputs
    int *d_aoff = c->arena.get<int>("in_atom_offsets", S + 1);
    NbStruct *d_ns = c->arena.get<NbStruct>("in_nbstructs", S + 1);
    if (!d_aoff || !d_ns)
        return fail(MTPB_ERR_MEMORY, "device allocation failed");
    CUDA_TRY(cudaMemcpyAsync(d_aoff, c->h_atom_offsets.data(), sizeof(int) * (S + 1),
                             cudaMemcpyHostToDevice, c->stream),
             "upload offsets");
    if (S > 0)
        CUDA_TRY(cudaMemcpyAsync(d_ns, ns.data(), sizeof(NbStruct) * S, cudaMemcpyHostToDevice,
                                 c->stream),
                 "upload structs");
    const double *d_pos = in->positions;
    const int *d_types = in->types;
    if (!dev && N > 0) {
        double *p = c->arena.get<double>("in_positions", 3 * (size_t)N);
        int *t = c->arena.get<int>("in_types", N);
        if (!p || !t)
            return fail(MTPB_ERR_MEMORY, "device allocation failed");
        CUDA_TRY(cudaMemcpyAsync(p, in->positions, sizeof(double) * 3 * N, cudaMemcpyHostToDevice,
                                 c->stream),
                 "upload positions");
        CUDA_TRY(cudaMemcpyAsync(t, in->types, sizeof(int) * N, cudaMemcpyHostToDevice, c->stream),
                 "upload types");
        d_pos = p;
        d_types = t;
    } else if (dev && N > 0) {
        // keep a private copy of the types: the caller's buffer is borrowed
        int *t = c->arena.get<int>("in_types", N);
        if (!t)
            return fail(MTPB_ERR_MEMORY, "device allocation failed");
        CUDA_TRY(cudaMemcpyAsync(t, in->types, sizeof(int) * N, cudaMemcpyDeviceToDevice,
                                 c->stream),
                 "copy types");
        d_types = t;
    }
    const int NC = c->center_count_req > 0 ? c->center_count_req : N;
    if (NC > N)
        return fail(MTPB_ERR_ARGUMENT, "center count " + std::to_string(NC) +
                                           " exceeds the batch's " + std::to_string(N) +
                                           " atoms");
    NbBuildInput bi;
    bi.nstruct = S;
    bi.natoms = N;
    bi.ncenter = NC;
    bi.total_cells = cells;
    bi.atom_offsets = d_aoff;
    bi.structs = d_ns;
    bi.positions = d_pos;
    bi.types = d_types;   // species range checked on the device, read with the edge count
    bi.K = c->model.K;
    CUDA_TRY(cudaEventRecord(c->ev[0], c->stream), "event");
    NbResult res;
    cudaError_t e = build_neighbors(bi, c->arena, res, c->stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "neighbour build");
    if (res.bad_type >= 0)
        return fail(MTPB_ERR_ARGUMENT, "atom " + std::to_string(res.bad_type) +
                                           " has a species index outside 0..K-1");
    {   // species pair of every edge, read by the moment kernels' prefetch
        int *pair = c->arena.get<int>("edge_pair", (size_t)res.nedges + 1);
        if (!pair)
            return fail(MTPB_ERR_MEMORY, "device allocation failed");
        CUDA_TRY(edge_pairs(res.nedges, res.center, res.nbr, d_types, c->model.K, pair,
                            c->stream),
                 "edge pairs");
        res.pair = pair;
    }
    c->nb = res;
    c->nedges = res.nedges;
    c->d_ns = d_ns;
    c->d_x_build = c->arena.get<double>("x_build", 3 * (size_t)N + 3);
    if (!c->d_x_build)
        return fail(MTPB_ERR_MEMORY, "device allocation failed");
    if (N)
        CUDA_TRY(cudaMemcpyAsync(c->d_x_build, d_pos, sizeof(double) * 3 * N,
                                 cudaMemcpyDeviceToDevice, c->stream),
                 "keep positions");
    c->natoms = NC;   // centres: atoms [0, NC)
    c->ntotal = N;
    c->nstruct = S;
    c->d_types = d_types;
    c->d_offsets = res.offsets;
    // reduction segments: <= 1024 centres of one structure each
    std::vector<int> sb, se, s0(S + 1, 0);
    for (int s = 0; s < S; ++s) {
        s0[s] = (int)sb.size();
        const int a0 = std::min(c->h_atom_offsets[s], NC);
        const int a1 = std::min(c->h_atom_offsets[s + 1], NC);
        if (a0 == a1) {
            sb.push_back(a0);
            se.push_back(a1);
        }
        for (int a = a0; a < a1; a += 1024) {
            sb.push_back(a);
            se.push_back(std::min(a + 1024, a1));
        }
    }
    s0[S] = (int)sb.size();
    c->nseg = (int)sb.size();
    // one upload of the three tables through pinned staging (no stream sync:
    // the staging buffer is rewritten only after its last copy has finished)
    const size_t nseg_tab = sb.size(), ntab = 2 * nseg_tab + (size_t)S + 1;
    int *d_tab = c->arena.get<int>("seg_tables", ntab + 1);
    if (!d_tab)
        return fail(MTPB_ERR_MEMORY, "device allocation failed");
    if (c->stage_pending)
        CUDA_TRY(cudaEventSynchronize(c->stage_ev), "staging buffer");
    c->stage_pending = false;
    if (c->h_stage_cap < ntab) {
        if (c->h_stage)
            cudaFreeHost(c->h_stage);
        c->h_stage = nullptr;
        c->h_stage_cap = 0;
        CUDA_TRY(cudaHostAlloc(reinterpret_cast<void **>(&c->h_stage), sizeof(int) * (ntab + 1024),
                               cudaHostAllocDefault),
                 "pinned staging");
        c->h_stage_cap = ntab + 1024;
    }
    std::copy(sb.begin(), sb.end(), c->h_stage);
    std::copy(se.begin(), se.end(), c->h_stage + nseg_tab);
    std::copy(s0.begin(), s0.end(), c->h_stage + 2 * nseg_tab);
    CUDA_TRY(cudaMemcpyAsync(d_tab, c->h_stage, sizeof(int) * ntab, cudaMemcpyHostToDevice,
                             c->stream),
             "upload segments");
    CUDA_TRY(cudaEventRecord(c->stage_ev, c->stream), "event");
    c->stage_pending = true;
    c->d_seg_begin = d_tab;
    c->d_seg_end = d_tab + nseg_tab;
    c->d_struct_seg0 = d_tab + 2 * nseg_tab;
    c->have_list = true;
    c->edge_epoch++;
    c->nb_built_this_call = true;
    c->refresh_pending = false;
    // struct ids, wrap/bin, 3 scans (2 kernels each), cell fill, sort and
    // position gather, count, fill, position packing and displacements,
    // in-edge count, fill and sort, edge species pairs
    c->pending_launches = 20;
    return MTPB_OK;
}

int mtpb_neighbor_count(const mtpb_context *c, long *n)
{
    if (!c || !n)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    if (!c->have_list)
        return fail(MTPB_ERR_STATE, "no neighbour list has been built");
    *n = c->nedges;
    return MTPB_OK;
}

int mtpb_get_neighbors(const mtpb_context *c, int *offsets, int *nbr, double *rij, int *shift)
{
    if (!c)
        return fail(MTPB_ERR_ARGUMENT, "ctx is NULL");
    if (!c->have_list)
        return fail(MTPB_ERR_STATE, "no neighbour list has been built");
    CUDA_TRY(cudaSetDevice(c->device), "cudaSetDevice");
    CUDA_TRY(cudaStreamSynchronize(c->stream), "sync");   // the build is stream-ordered
    const long E = c->nedges;
    if (offsets)
        CUDA_TRY(cudaMemcpy(offsets, c->nb.offsets, sizeof(int) * (c->natoms + 1),
                            cudaMemcpyDeviceToHost),
                 "copy offsets");
    if (nbr && E)
        CUDA_TRY(cudaMemcpy(nbr, c->nb.nbr, sizeof(int) * E, cudaMemcpyDeviceToHost), "copy nbr");
    if (shift && E)
        CUDA_TRY(cudaMemcpy(shift, c->nb.shift, sizeof(int) * E, cudaMemcpyDeviceToHost),
                 "copy shift");
    if (rij && E) {
        std::vector<double> x(E), y(E), z(E);
        CUDA_TRY(cudaMemcpy(x.data(), c->nb.rx, sizeof(double) * E, cudaMemcpyDeviceToHost), "rx");
        CUDA_TRY(cudaMemcpy(y.data(), c->nb.ry, sizeof(double) * E, cudaMemcpyDeviceToHost), "ry");
        CUDA_TRY(cudaMemcpy(z.data(), c->nb.rz, sizeof(double) * E, cudaMemcpyDeviceToHost), "rz");
        for (long e = 0; e < E; ++e) {
            rij[3 * e] = x[e];
            rij[3 * e + 1] = y[e];
            rij[3 * e + 2] = z[e];
        }
    }
    return MTPB_OK;
}

} // extern "C"

int mtpb::efs_compute(mtpb_context *c, int memory, const mtpb_efs_output *out,
                      bool forces_needed)
{
    if (!c)
        return fail(MTPB_ERR_ARGUMENT, "ctx is NULL");
    if (!c->have_list)
        return fail(MTPB_ERR_STATE, "build the neighbour list first (mtpb_build_neighbors)");
    int rc = set_device(c);
    if (rc)
        return rc;
    const bool dev = memory == MTPB_MEMORY_DEVICE;
    const int N = c->natoms, NT = c->ntotal, S = c->nstruct;   // centres, all atoms
    const long E = c->nedges;
    c->launches = c->nb_built_this_call ? c->pending_launches : 0;
    c->pending_launches = 0;
    if (!c->nb_built_this_call)
        CUDA_TRY(cudaEventRecord(c->ev[0], c->stream), "event");
    double *site_energy = c->arena.get<double>("site_energy", N + 1);
    double *dx = c->arena.get<double>("dx", E + 1), *dy = c->arena.get<double>("dy", E + 1),
           *dz = c->arena.get<double>("dz", E + 1);
    double *forces = (dev && out && out->forces) ? out->forces
                                                 : c->arena.get<double>("forces", 3 * (size_t)NT + 1);
    double *avir = c->arena.get<double>("atom_virial", 9 * (size_t)N + 1);
    double *partials = c->arena.get<double>("partials", 10 * (size_t)c->nseg + 10);
    double *energy = (dev && out && out->energy) ? out->energy
                                                 : c->arena.get<double>("energy", S + 1);
    double *stress = (dev && out && out->stress) ? out->stress
                                                 : c->arena.get<double>("stress", 9 * (size_t)S + 9);
    if (!site_energy || !dx || !dy || !dz || !forces || !avir || !partials || !energy || !stress)
        return fail(MTPB_ERR_MEMORY, "device allocation failed");
    // with a skin the list holds pairs up to r_c + skin; a pending refresh
    // of its vectors runs in the active-edge pass
    const EdgeRefresh *refresh = c->refresh_pending ? &c->refresh : nullptr;
    c->refresh_pending = false;
    rc = run_moments(c, N, c->d_types, c->nb.offsets, c->nb.nbr, c->nb.rx, c->nb.ry, c->nb.rz,
                     site_energy, dx, dy, dz, forces_needed, E, c->skin > 0.0, refresh);
    if (rc)
        return rc;
    NvtxRange range_gather("mtpb:force_gather_reduce");
    if (forces_needed) {
        CUDA_TRY(launch_force_gather(N, NT, c->nb.offsets, c->nb.in_offsets, c->nb.in_edges, dx,
                                     dy, dz, c->nb.rx, c->nb.ry, c->nb.rz, forces, avir, 0,
                                     c->stream),
                 "force gather");
        c->launches++;
    }
    CUDA_TRY(launch_segment_reduce(c->nseg, c->d_seg_begin, c->d_seg_end, site_energy,
                                   forces_needed ? avir : nullptr, N, partials, c->stream),
             "segment reduce");
    CUDA_TRY(launch_struct_reduce(S, c->d_struct_seg0, partials, energy, stress, c->stream),
             "structure reduce");
    c->launches += 2;
    CUDA_TRY(cudaEventRecord(c->ev[5], c->stream), "event");
    c->ev_valid = true;
    c->nb_built_this_call = false;
    if (out) {
        const cudaMemcpyKind k = dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
        if (out->energy && !dev)
            CUDA_TRY(cudaMemcpyAsync(out->energy, energy, sizeof(double) * S, k, c->stream), "copy");
        if (out->forces && !dev)
            CUDA_TRY(cudaMemcpyAsync(out->forces, forces, sizeof(double) * 3 * NT, k, c->stream),
                     "copy");
        if (out->stress && !dev)
            CUDA_TRY(cudaMemcpyAsync(out->stress, stress, sizeof(double) * 9 * S, k, c->stream),
                     "copy");
        if (out->site_energy && N)
            CUDA_TRY(cudaMemcpyAsync(out->site_energy, site_energy, sizeof(double) * N, k,
                                     c->stream),
                     "copy");
    }
    if (!dev) {
        CUDA_TRY(cudaStreamSynchronize(c->stream), "EFS");
        if ((rc = check_device_error(c)))
            return rc;
    } else {
        CUDA_TRY(cudaGetLastError(), "EFS");
    }
    c->have_efs = true;
    c->have_dedr = forces_needed;
    return MTPB_OK;
}

extern "C" {

int mtpb_efs_compute(mtpb_context *c, int memory, const mtpb_efs_output *out)
{
    // an output without forces and stress asks for energies only (the
    // energy-only branch of calc_efs and the trainer): no reverse pass
    const bool forces = !out || out->forces || out->stress;
    return efs_compute(c, memory, out, forces);
}

int mtpb_efs_structures(mtpb_context *c, const mtpb_structures *in, int memory,
                        int reuse_neighbors, const mtpb_efs_output *out)
{
    if (!c)
        return fail(MTPB_ERR_ARGUMENT, "ctx is NULL");
    int rc = check_structures(c, in);
    if (rc)
        return rc;
    bool reuse = reuse_neighbors && c->have_list && in->n_structures == c->nstruct;
    if (reuse) {
        // the batch layout must be unchanged; cells are those of the build
        // host arrays are checked; for device arrays the caller guarantees an
        // unchanged batch layout (no device-to-host read on the reuse path)
        if (memory != MTPB_MEMORY_DEVICE) {
            std::vector<int> off(in->atom_offsets, in->atom_offsets + in->n_structures + 1);
            reuse = off == c->h_atom_offsets;
        }
    }
    if (!reuse) {
        rc = mtpb_build_neighbors(c, in, memory);
        if (rc)
            return rc;
    } else {
        if ((rc = set_device(c)))
            return rc;
        const int N = c->ntotal;
        const double *x = in->positions;
        if (memory != MTPB_MEMORY_DEVICE && N) {
            double *p = c->arena.get<double>("in_positions", 3 * (size_t)N);
            if (!p)
                return fail(MTPB_ERR_MEMORY, "device allocation failed");
            CUDA_TRY(cudaMemcpyAsync(p, in->positions, sizeof(double) * 3 * N,
                                     cudaMemcpyHostToDevice, c->stream),
                     "upload positions");
            x = p;
        }
        double *unwrapped = c->arena.get<double>("refresh_unwrapped", 4 * (size_t)N + 4);
        if (!unwrapped)
            return fail(MTPB_ERR_MEMORY, "device allocation failed");
        CUDA_TRY(cudaEventRecord(c->ev[0], c->stream), "event");
        // with a skin the compute's active-edge pass recomputes the vectors
        // while it tests them (one pass over the list instead of two)
        const bool fused = c->skin > 0.0 && c->nedges > 0 && c->natoms > 0;
        {
            NvtxRange range("mtpb:refresh_edges");
            if (fused)
                CUDA_TRY(unwrap_positions(N, c->nb, c->d_x_build, x, unwrapped, c->stream),
                         "unwrap positions");
            else
                CUDA_TRY(refresh_edges(N, c->d_ns, c->nb.struct_of, c->nb, c->d_x_build, x,
                                       unwrapped, const_cast<double *>(c->nb.rx),
                                       const_cast<double *>(c->nb.ry),
                                       const_cast<double *>(c->nb.rz), c->stream),
                         "refresh edge vectors");
        }
        if (fused) {
            c->refresh = EdgeRefresh{c->d_ns, c->nb.struct_of, c->nb.shift, unwrapped,
                                     const_cast<double *>(c->nb.rx),
                                     const_cast<double *>(c->nb.ry),
                                     const_cast<double *>(c->nb.rz)};
            c->refresh_pending = true;
        }
        c->edge_epoch++;
        c->nb_built_this_call = true;   // ev[0] marks the refresh
        c->pending_launches = c->nedges ? (fused ? 1 : 2) : 0;
    }
    return mtpb_efs_compute(c, memory, out);
}

int mtpb_check_device_status(mtpb_context *c)
{
    if (!c)
        return fail(MTPB_ERR_ARGUMENT, "ctx is NULL");
    int rc = set_device(c);
    if (rc)
        return rc;
    if (!c->d_err)
        return MTPB_OK;   // no graph kernel has run on this context
    CUDA_TRY(cudaStreamSynchronize(c->stream), "synchronise");
    return check_device_error(c);
}

int mtpb_debug_flag_device_error(mtpb_context *c)
{
    if (!c)
        return fail(MTPB_ERR_ARGUMENT, "ctx is NULL");
    int rc = set_device(c);
    if (rc)
        return rc;
    if (!c->d_err)
        return fail(MTPB_ERR_STATE, "load a model first");
    const int one = 1;
    CUDA_TRY(cudaMemcpyAsync(c->d_err, &one, sizeof(int), cudaMemcpyHostToDevice, c->stream),
             "set flag");
    CUDA_TRY(cudaStreamSynchronize(c->stream), "synchronise");
    return MTPB_OK;
}

int mtpb_last_timings(const mtpb_context *c, double *ms)
{
    if (!c || !ms)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    if (!c->ev_valid)
        return fail(MTPB_ERR_STATE, "no compute call has been timed");
    CUDA_TRY(cudaSetDevice(c->device), "cudaSetDevice");
    CUDA_TRY(cudaEventSynchronize(c->ev[5]), "event sync");
    float t[5];
    for (int i = 0; i < 5; ++i) {
        CUDA_TRY(cudaEventElapsedTime(&t[i], c->ev[i], c->ev[i + 1]), "elapsed");
        ms[i] = t[i];
    }
    return MTPB_OK;
}

int mtpb_last_train_timings(const mtpb_context *c, double *ms)
{
    if (!c || !ms)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    if (!c->train.ev_valid)
        return fail(MTPB_ERR_STATE, "no mtpb_loss_grad call has been timed");
    CUDA_TRY(cudaSetDevice(c->device), "cudaSetDevice");
    CUDA_TRY(cudaEventSynchronize(c->train.ev[6]), "event sync");
    for (int i = 0; i < 6; ++i) {
        float t = 0.f;
        CUDA_TRY(cudaEventElapsedTime(&t, c->train.ev[i], c->train.ev[i + 1]), "elapsed");
        ms[i] = t;
    }
    return MTPB_OK;
}

int mtpb_last_launch_count(const mtpb_context *c, int *launches)
{
    if (!c || !launches)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    *launches = c->launches;
    return MTPB_OK;
}

int mtpb_get_site_moments(const mtpb_context *c, double *basic, double *adjoint)
{
    if (!c)
        return fail(MTPB_ERR_ARGUMENT, "ctx is NULL");
    if (!c->have_efs)
        return fail(MTPB_ERR_STATE, "no EFS result available");
    CUDA_TRY(cudaSetDevice(c->device), "cudaSetDevice");
    CUDA_TRY(cudaStreamSynchronize(c->stream), "sync");
    const int nb = c->model.nb();
    const int N = c->natoms;
    auto fetch = [&](const char *name, double *dst) -> int {
        double *src = const_cast<DeviceArena &>(c->arena).get<double>(name, 1);
        std::vector<double> all((size_t)c->nslot * c->npad);
        CUDA_TRY(cudaMemcpy(all.data(), src, sizeof(double) * all.size(), cudaMemcpyDeviceToHost),
                 "copy moments");
        for (int i = 0; i < N; ++i)
            for (int b = 0; b < nb; ++b)
                dst[(size_t)i * nb + b] = all[(size_t)c->slot_of_basic[b] * c->npad + i];
        return MTPB_OK;
    };
    int rc;
    if (basic && (rc = fetch("basic", basic)))
        return rc;
    if (adjoint && (rc = fetch("adjoint", adjoint)))
        return rc;
    return MTPB_OK;
}

int mtpb_get_edge_derivatives(const mtpb_context *c, double *dedr)
{
    if (!c || !dedr)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    if (!c->have_efs || !c->have_dedr)
        return fail(MTPB_ERR_STATE, "no EFS result available");
    CUDA_TRY(cudaSetDevice(c->device), "cudaSetDevice");
    CUDA_TRY(cudaStreamSynchronize(c->stream), "sync");
    const long E = c->nedges;
    DeviceArena &ar = const_cast<DeviceArena &>(c->arena);
    std::vector<double> x(E), y(E), z(E);
    if (E) {
        CUDA_TRY(cudaMemcpy(x.data(), ar.get<double>("dx", 1), sizeof(double) * E,
                            cudaMemcpyDeviceToHost),
                 "dx");
        CUDA_TRY(cudaMemcpy(y.data(), ar.get<double>("dy", 1), sizeof(double) * E,
                            cudaMemcpyDeviceToHost),
                 "dy");
        CUDA_TRY(cudaMemcpy(z.data(), ar.get<double>("dz", 1), sizeof(double) * E,
                            cudaMemcpyDeviceToHost),
                 "dz");
    }
    for (long e = 0; e < E; ++e) {
        dedr[3 * e] = x[e];
        dedr[3 * e + 1] = y[e];
        dedr[3 * e + 2] = z[e];
    }
    return MTPB_OK;
}

int mtpb_graph_program(const mtpb_model_view *view, int *nslot, int *slot_of_basic, int *nrows,
                       int *one_row, int *zero_row, int *n_fwd, int *n_rev, int *phase_rows,
                       long *n_records, unsigned int *records)
{
    ModelHost m;
    std::string err;
    if (!copy_model(view, m, &err) || !validate_model(m, &err))
        return fail(MTPB_ERR_ARGUMENT, err);
    const int shape = select_shape(m, &err);
    if (shape < 0)
        return fail(MTPB_ERR_UNSUPPORTED, err);
    std::vector<int> sob;
    DagPlan plan;
    if (!build_slot_map(m, shape, sob, &err) || !build_dag_plan(m, shape, sob, plan, &err))
        return fail(MTPB_ERR_UNSUPPORTED, err);
    if (nslot)
        *nslot = shape_desc(shape).nslot;
    if (slot_of_basic)
        std::copy(sob.begin(), sob.end(), slot_of_basic);
    if (nrows)
        *nrows = plan.nrows;
    if (one_row)
        *one_row = plan.one_row;
    if (zero_row)
        *zero_row = plan.zero_row;
    if (n_fwd)
        *n_fwd = plan.n_fwd;
    if (n_rev)
        *n_rev = plan.n_rev;
    if (phase_rows)
        std::copy(plan.phase_rows.begin(), plan.phase_rows.end(), phase_rows);
    if (n_records)
        *n_records = (long)plan.recs.size();
    if (records)
        std::memcpy(records, plan.recs.data(), sizeof(DagRec) * plan.recs.size());
    return MTPB_OK;
}

int mtpb_efs_csr(mtpb_context *c, const mtpb_csr_request *req, int memory)
{
    mtpb::NvtxRange range("mtpb:efs_csr");
    return csr_compute(c, req, memory);
}

int mtpb_efs_lammps(mtpb_context *c, const mtpb_lammps_request *req)
{
    return lammps_compute(c, req);
}

int mtpb_loss_grad(mtpb_context *c, const mtpb_labels *labels, const mtpb_loss_weights *w,
                   int norm_count, int memory, double *loss, double *metrics, double *grad)
{
    return loss_grad_compute(c, labels, w, norm_count, memory, loss, metrics, grad);
}

int mtpb_check_training_values(mtpb_context *c, long *first_nonfinite)
{
    if (!c || !first_nonfinite)
        return fail(MTPB_ERR_ARGUMENT, "NULL argument");
    return training_values_status(c, first_nonfinite);
}

} // extern "C"
