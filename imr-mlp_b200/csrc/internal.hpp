// internal.hpp -- structures shared by the host planner and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace mtpb {

// NVTX range over one stage of a call (the kernels it launches), named
// "mtpb:<stage>" in profiler timelines; with no tool attached a push/pop is a
// check of a function pointer (NVTX v3 is header-only).  The reference wraps
// its kernels the same way (runtime/mtp/gpu-direct/mtp_gpu_direct.cu:46-65).
struct NvtxRange {
    explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange &) = delete;
    NvtxRange &operator=(const NvtxRange &) = delete;
};


// Identifies one instantiated basis shape (see shapes.cuh).
enum ShapeId : int {
    SHAPE_S1 = 0,
    SHAPE_S2,
    SHAPE_L16,
    SHAPE_L20,
    SHAPE_L24,
    SHAPE_PS,
    SHAPE_COUNT
};

struct ShapeDesc {
    int nmu;
    int numax[8];
    int nslot;
};

// Host query of the instantiated shapes and their slot map.
const ShapeDesc &shape_desc(int id);
int shape_slot(int id, int mu, int a, int b, int c);

// Radial parameters of one ordered species pair (RBasis_Chebyshev::setup,
// basis/basis.cpp:119-126): pu = rmax + rmin, su = rmax - rmin,
// mult = 2 / (rmax - rmin), rmax is also the pair cutoff.
// Radial family of a pair (mtpb_radial_family of include/mtpb200.h).
enum RadialType { RB_CHEBYSHEV = 0, RB_CHEBY_COS = 1, RB_CHEBY_POLY5 = 2, RB_CONFIGURABLE = 3,
                  RB_CHEBY_POLY4 = 4, RB_POLYB = 5, RB_POLYB_COS = 6 };
enum RadialCutoffType { CUT_QUADRATIC = 0, CUT_COSINE = 1, CUT_POLY5 = 2,
                        CUT_NORMALIZED_QUADRATIC = 3, CUT_COSINE_LEFT = 4,
                        CUT_COSINE_UNSCALED = 5, CUT_COSINE_SQUARED = 6, CUT_SINE_SQUARED = 7,
                        CUT_POLY3 = 8, CUT_POLY4 = 9, CUT_SMOOTHSTEP5 = 10, CUT_SMOOTHSTEP7 = 11 };
enum RadialShiftType { SHIFT_LINEAR = 0, SHIFT_EXPONENTIAL = 1, SHIFT_EXPONENTIAL_LEFT = 2,
                       SHIFT_I2 = 3, SHIFT_EXPONENTIAL_TANH = 4 };
struct RadialFamily {
    int type = RB_CHEBYSHEV, cutoff = CUT_QUADRATIC, shift = SHIFT_LINEAR, flipped = 0;
    double b = 0.0, r1 = 0.0, r2 = 0.0, lambda = 0.0, scale_lambda = 0.0;
    // RBPolyB / RBPolyBCos: orthogonalisation matrix [R*R] (column-major) and
    // power normalisations [R], as the reference's loader computes them
    std::vector<double> poly_matrix, poly_norm;
};

// Device parameters of a pair's radial basis (filled by upload_model, api.cu):
// the Chebyshev coordinate ksi = (2r - pu) / su with dksi/dr = mult, the
// interval, and the family's envelope / shift parameters with the constants the
// reference computes once per basis (expm1(lambda), tanh(scale_lambda)).
struct PairParams {
    double pu, su, mult, rmax;
    double rmin, inv_range, irpi, b;
    double r1, r2, lambda, scale_lambda;
    double den, sden, slope, cfreq;   // cfreq: pi / (max - min) of the cosine cutoff
    int type, cutoff, shift, flipped;
};
constexpr int PAIR_PARAM_DOUBLES = (int)(sizeof(PairParams) / sizeof(double));

// Record of the moment-graph program (see k_dag in efs.cu): 16 bytes,
// {s1 | s2 << 16, out | flags << 16, c (double)}.
struct alignas(16) DagRec {
    unsigned int s12;
    unsigned int outf;
    double c;
};
enum DagFlags : unsigned {
    DAG_END = 2,     // store acc to row `out` (or the global adjoint slot), then acc = 0
    DAG_GLOBAL = 4,  // reverse: `out` is a kernel slot of the global adjoint array
    DAG_ENERGY = 8,  // forward: E += c * acc before any store (its product is zero)
};
inline DagRec make_rec(int s1, int s2, int out, unsigned flags, double c)
{
    DagRec r;
    r.s12 = (unsigned)s1 | ((unsigned)s2 << 16);
    r.outf = (unsigned)(out < 0 ? 0 : out) | (flags << 16);
    r.c = c;
    return r;
}

// Record streams per graph block: 32 or 64 (16 warps, the planner's choice
// unless the 64-stream program pads more than 10% extra record slots;
// build_dag_plan in plan.cpp).
constexpr int DAG_STREAMS = 32;
constexpr int DAG_STREAMS_LARGE = 64;
constexpr int DAG_STREAMS_MAX = 64;
constexpr int DAG_MAX_PHASES = 64;   // phase table size of the graph kernels
// record rows per ring slot (the ring stays 32 KB for both stream counts)
constexpr int dag_chunk_rows(int streams) { return streams > 32 ? 16 : 32; }

// Device form of a record (16 bytes): the two operand row indices (16 bits
// each), a word that is zero for plain product records and otherwise holds
// flags << 28 | out, and the coefficient.
struct alignas(16) DagDevRec {
    unsigned rows;   // s1 | s2 << 16
    unsigned outf;
    double c;
};

struct DagPlan {
    int nrows = 0;           // rows (one double per atom each)
    int one_row = 0;         // row holding 1.0
    int zero_row = 0;        // row holding 0.0
    int scratch_row = 0;     // row receiving stores that nothing reads
    std::vector<int> phase_rows;   // record rows per phase (fwd phases, then reverse)
    int n_fwd = 0, n_rev = 0;
    int streams = DAG_STREAMS;     // record streams (DAG_STREAMS or DAG_STREAMS_LARGE)
    std::vector<DagRec> recs;      // [sum rows][streams]
    // training: index into energy_moments of the scalar moment an ENERGY
    // record closes (-1 for every other record), parallel to recs
    std::vector<int> rec_energy;
    std::vector<int> energy_moments;   // moment ids with a scalar coefficient
    // execution geometry, chosen when the plan is uploaded (dag_configure)
    int atoms = 16;            // atoms per graph block (8 or 16)
    bool global_rows = false;  // rows in global scratch (graph too large for shared memory)
    int grid = 0;              // persistent blocks with global rows (one per SM)
    bool grad_global_rows = false;   // the same choice for the dual graph (grad.cu)
    int grad_grid = 0;
};

// Edge-kernel parameters (device pointers).
struct EdgeArgs {
    int natoms;          // centres
    int npad;            // row stride of the moment/adjoint arrays
    const int *types;    // [ntotal] species of every atom referenced
    const int *offsets;  // [natoms+1]
    const int *nbr;      // [E]
    const double *rx, *ry, *rz;  // [E]
    const int *pair;             // [E] species pair it*K+jt (-1: a type is -1), or NULL
    const int *group_maxdeg;     // [ceil(natoms/32)]
    // optional active edges (inside the pair cutoff): centre i has nact[i]
    // of them, compacted in list order to slots offsets[i] .. offsets[i] +
    // nact[i] - 1 of nbr, rx, ry, rz and pair, and active[offsets[i] + k] is
    // the list index of its k-th (where the per-edge derivatives go); NULL
    // stages every edge of the list
    const int *active;
    const int *nact;
    int K, R, mu_total;
    double scaling;
    const double *radial;          // [K*K][mu_total][R]
    const PairParams *pairs;       // [K*K]
    int rb_generic;                // some pair's radial family is not RBChebyshev
};

// launchers (efs.cu); moment_kernel_parts = launches per call
int moment_kernel_parts(int shape, bool rev);
int grad_kernel_launches(int shape, bool edge);
cudaError_t launch_moments_fwd(int shape, const EdgeArgs &a, double *basic, cudaStream_t s);
// Active edges of a neighbour list whose edges may reach beyond the pair
// cutoff (a skin or a caller's list): active/nact as in EdgeArgs, the active
// edges' vectors, neighbours and species pairs compacted into cx, cy, cz,
// cnbr, cpair, the largest active count of every 32-centre group in
// group_maxdeg, and zero per-edge derivatives dx/dy/dz (may be NULL) for the
// inactive edges.
struct ActiveEdges {
    int *active, *nact, *group_maxdeg;
    double *cx, *cy, *cz;
    int *cnbr, *cpair;
};
// Edge vectors of a stored list recomputed from moved positions (refresh.cuh):
// the structures and structure ids of the build, the packed shift of every
// edge, the positions as [atom][4] rows relative to the build's images, and
// the list's vector arrays, overwritten.
struct NbStruct;
struct EdgeRefresh {
    const NbStruct *structs;
    const int *struct_of;
    const int *shift;
    const double *unwrapped;
    double *rx, *ry, *rz;
};
// refresh (may be NULL): the vectors are recomputed first, in the same pass
cudaError_t launch_active_edges(const EdgeArgs &a, const ActiveEdges &out,
                                const EdgeRefresh *refresh, double *dx, double *dy, double *dz,
                                cudaStream_t s);
cudaError_t launch_moments_rev(int shape, const EdgeArgs &a, const double *adjoint, double *dx,
                               double *dy, double *dz, cudaStream_t s);
size_t dag_ring_bytes(int atoms);
std::vector<DagDevRec> dag_device_records(const DagPlan &plan);
cudaError_t launch_dag(const DagPlan &plan, const DagDevRec *recs, const int *phase_row0,
                       int nslot, int natoms, int npad, const int *types,
                       const double *species_coeffs, const double *basic, double *adjoint,
                       double *site_energy, double *gscratch, int *err_flag, cudaStream_t s);
cudaError_t launch_group_maxdeg(int natoms, const int *offsets, int *group_maxdeg,
                                cudaStream_t s);
cudaError_t launch_force_gather(int natoms, int ntotal, const int *offsets, const int *in_offsets,
                                const int *in_edges, const double *dx, const double *dy,
                                const double *dz, const double *rx, const double *ry,
                                const double *rz, double *forces, double *atom_virial,
                                int accumulate, cudaStream_t s);
cudaError_t launch_segment_reduce(int nseg, const int *seg_begin, const int *seg_end,
                                  const double *site_energy, const double *atom_virial,
                                  int natoms, double *partials, cudaStream_t s);
cudaError_t launch_struct_reduce(int nstruct, const int *struct_seg0, const double *partials,
                                 double *energy, double *virial, cudaStream_t s);

// training gradient kernels (grad.cu)
cudaError_t launch_moments_tangent(int shape, const EdgeArgs &a, const double *wx,
                                   const double *wy, const double *wz, double *tangent,
                                   cudaStream_t s);
cudaError_t launch_edge_grad(int shape, const EdgeArgs &a, const double *wx, const double *wy,
                             const double *wz, const double *adjoint, const double *adjoint2,
                             double *uv, cudaStream_t s);
std::vector<DagDevRec> dag_grad_records(const DagPlan &plan);
size_t dag_grad_smem_bytes(const DagPlan &plan, bool global_rows);
size_t dag_grad_scratch_doubles(const DagPlan &plan);
int dag_grad_grid(const DagPlan &plan, int natoms);
cudaError_t launch_dag_grad(const DagPlan &plan, const DagDevRec *recs, const int *phase_row0,
                            int grid, int nslot, int natoms, int npad, const double *basic,
                            const double *tangent, const double *dlde_atom, double *adjoint2,
                            double *energy_partials, double *gscratch, int *err_flag,
                            cudaStream_t s);

} // namespace mtpb
