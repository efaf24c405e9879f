/*
 * mtpb200.h -- C ABI of the B200 MTP energy/force/stress and
 * coefficient-gradient path.
 *
 * Every entry point returns MTPB_OK (0) or a nonzero status; the message of
 * the last failure on the calling thread is available from
 * mtpb_last_error().  No entry point throws, aborts or exits.  All pointers
 * are borrowed for the duration of the call only.  One context belongs to one
 * CUDA device and must not be used by two threads at once.
 *
 * Array pointers carry host memory unless a call takes a `memory` argument
 * equal to MTPB_MEMORY_DEVICE, in which case every array of that call is
 * device memory on the context's device.  Host-memory calls have finished
 * with every array when they return.  Device-memory calls are ordered on the
 * context's stream (mtpb_set_stream): their device arrays are read and
 * written by work queued on that stream and must stay valid until it has
 * run; the per-structure tables of mtpb_build_neighbors (atom_offsets, cells,
 * pbc) are read back to the host at the start of the call and must already
 * hold their values.
 *
 * Each declaration names the reference interface it replaces (paths relative
 * to the reference project root).
 */
#ifndef MTPB200_H
#define MTPB200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define MTPB_ABI_VERSION 3

enum mtpb_status {
    MTPB_OK = 0,
    MTPB_ERR_ARGUMENT = 1,     /* invalid argument or inconsistent sizes */
    MTPB_ERR_UNSUPPORTED = 2,  /* model or geometry outside what the kernels implement */
    MTPB_ERR_CUDA = 3,         /* CUDA runtime error (message holds the CUDA text) */
    MTPB_ERR_MEMORY = 4,       /* device allocation failed */
    MTPB_ERR_STATE = 5,        /* call order violated (e.g. no neighbour list yet) */
    MTPB_ERR_NONFINITE = 6     /* a loss, metric or gradient value is NaN or infinite */
};

enum mtpb_memory { MTPB_MEMORY_HOST = 0, MTPB_MEMORY_DEVICE = 1 };

typedef struct mtpb_context mtpb_context;

/* Radial basis families (basis/basis.cpp; numbering of RadialBasis,
 * RadialCutoff and RadialTransform in runtime/mtp/gpu-direct/mtp_gpu_direct.h:
 * 152-186).  Every family is a Chebyshev series in a coordinate x(r) times an
 * envelope fc(r), scaled by the model's scaling:
 *   RBChebyshev        x = (2r - min - max)/(max - min), fc = (r - max)^2
 *   RBChebyCos         same x, fc = (1 + cos(pi r / max)) / 2
 *   RBChebyshevPoly4   same x, fc = (1-t)^3 (1 + (3+b) t), t = (r-min)/(max-min)
 *   RBChebyshevPoly5   same x, fc = (1-t)^4 (1 + (4+b) t)
 *   RBChebyshevConfigurable  x from shift_type, fc from cutoff_type, optionally
 *                      the 1 - T_(i+1) polynomials (basis.cpp:937-1013,
 *                      cutoff.cpp, xtrans.cpp)
 *   RBPolyB / RBPolyBCos  Q_i = fc sum_j M(i,j) N_j s (max - r)^(j + first),
 *                      first 3 with fc = 1 / first 2 with fc = (1 + cos(pi r / max))/2
 *                      (runtime/mtp/radial_basis.h:223-290); M and N are the
 *                      orthogonalisation matrix and normalisations of the
 *                      reference's loader (radial_basis_t::polynomial_matrix,
 *                      polynomial_normalizations), passed in poly_matrix / poly_norm:
 *                      M is ill-conditioned (1e13 at R = 8), so it is taken as data
 *                      rather than recomputed.
 * Poly4, Poly5 and the configurable family are zero below min_dist. */
enum mtpb_radial_type {
    MTPB_RB_CHEBYSHEV = 0,
    MTPB_RB_CHEBY_COS = 1,
    MTPB_RB_CHEBY_POLY5 = 2,
    MTPB_RB_CHEBY_CONFIGURABLE = 3,
    MTPB_RB_CHEBY_POLY4 = 4,
    MTPB_RB_POLYB = 5,
    MTPB_RB_POLYB_COS = 6
};
enum mtpb_radial_cutoff {   /* cutoff_type of RBChebyshevConfigurable */
    MTPB_CUT_QUADRATIC = 0, MTPB_CUT_COSINE = 1, MTPB_CUT_POLY5 = 2,
    MTPB_CUT_NORMALIZED_QUADRATIC = 3, MTPB_CUT_COSINE_LEFT = 4, MTPB_CUT_COSINE_UNSCALED = 5,
    MTPB_CUT_COSINE_SQUARED = 6, MTPB_CUT_SINE_SQUARED = 7, MTPB_CUT_POLY3 = 8,
    MTPB_CUT_POLY4 = 9, MTPB_CUT_SMOOTHSTEP5 = 10, MTPB_CUT_SMOOTHSTEP7 = 11
};
enum mtpb_radial_shift {   /* shift_type of RBChebyshevConfigurable */
    MTPB_SHIFT_LINEAR = 0, MTPB_SHIFT_EXPONENTIAL = 1, MTPB_SHIFT_EXPONENTIAL_LEFT = 2,
    MTPB_SHIFT_I2 = 3, MTPB_SHIFT_EXPONENTIAL_TANH = 4
};
typedef struct mtpb_radial_family {
    int type;                  /* mtpb_radial_type */
    int cutoff_type;           /* configurable only */
    int shift_type;            /* configurable only */
    int one_minus_chebyshev;   /* configurable only: basis_function_type */
    double b;                  /* rb_b (Poly4, Poly5) or cutoff_b (poly3/4/5 cutoffs) */
    double r1, r2;             /* cutoff_r1, cutoff_r2 (smoothstep7) */
    double lambda;             /* shift_lambda */
    double scale_lambda;       /* shift_scale_lambda */
    const double *poly_matrix; /* RBPolyB / RBPolyBCos: M [R*R], column-major; else NULL */
    const double *poly_norm;   /* RBPolyB / RBPolyBCos: N [R]; else NULL */
} mtpb_radial_family;

/* Linear MTP.  Field meaning follows MTPGpuPotentialView
 * (runtime/mtp/gpu-direct/mtp_gpu_direct.h:270-325) and the .mtp layout read
 * by PotMTP::Load (potentials/potential_mtp.cpp:119-576):
 * radial_coeffs[(ti*K + tj)*mu*R + m*R + xi], alpha_index_basic[i] =
 * {mu, a, b, c}, alpha_index_times[t] = {l1, l2, coefficient, target}. */
typedef struct mtpb_model_view {
    int species_count;
    int radial_func_count;
    int rb_size;
    int radial_basis_split;     /* 0: one basis; 1: one basis per ordered pair */
    const double *min_dist;     /* [1] or [K*K] */
    const double *max_dist;     /* [1] or [K*K]; also the pair cutoff */
    double scaling;
    int alpha_moments_count;
    int alpha_index_basic_count;
    int alpha_index_times_count;
    int alpha_scalar_moments;
    const int *alpha_index_basic;     /* [nb][4] */
    const int *alpha_index_times;     /* [T][4] */
    const int *alpha_moment_mapping;  /* [S] */
    const double *radial_coeffs;      /* [K*K*mu*R] */
    const double *species_coeffs;     /* [K] */
    const double *moment_coeffs;      /* [S] */
    const mtpb_radial_family *radial_family;  /* NULL: RBChebyshev; else [1] or [K*K] */
} mtpb_model_view;

/* A batch of periodic structures (the Atoms + Neighborhoods inputs of
 * PotMTP::getEFS, potentials/potential_mtp.cpp:1892-1933, and of the CSR batch
 * built by MTPGpuBatch::build_impl, potentials/mtp_gpu_adapter.cpp:1011-1180). */
typedef struct mtpb_structures {
    int n_structures;
    const int *atom_offsets;   /* [S+1]: atoms of structure s are [off[s], off[s+1]) */
    const double *cells;       /* [S][9]: row-major, rows are lattice vectors (Atoms::cell_) */
    const int *pbc;            /* [S][3] periodic flags; NULL means fully periodic */
    const double *positions;   /* [N][3] Cartesian, Angstrom */
    const int *types;          /* [N] species index 0..K-1 (Atoms::chemmap_) */
} mtpb_structures;

/* Outputs of a structure batch; any pointer may be NULL. */
typedef struct mtpb_efs_output {
    double *energy;       /* [S] eV */
    double *forces;       /* [N][3] eV/Angstrom (Atoms::forces_) */
    double *stress;       /* [S][9] virial in eV, row-major (Atoms::stress_) */
    double *site_energy;  /* [N] eV (Atoms::site_energies_) */
} mtpb_efs_output;

/* ---- library and context ------------------------------------------------ */

/* Message of the last failed call on this thread ("" if none). */
const char *mtpb_last_error(void);
int mtpb_abi_version(void);
/* Replaces MTPGpuDirect::available_device_count (mtp_gpu_direct.h:803). */
int mtpb_device_count(int *count);

/* Replaces MTPGpuDirect::set_device + initialize (mtp_gpu_direct.h:801-813):
 * selects the device, validates the moment graph, uploads coefficients and
 * prepares the kernels for the model's basis shape. */
int mtpb_create(int device, const mtpb_model_view *model, mtpb_context **ctx);
int mtpb_destroy(mtpb_context *ctx);

/* Replaces MTPGpuDirect::update_coefficients (mtp_gpu_direct.h:814-816).
 * Host arrays in the native order: radial [K*K*mu*R], species [K], moment [S]. */
int mtpb_update_coefficients(mtpb_context *ctx, const double *radial, const double *species,
                             const double *moment);

/* Runs all later work of the context on `stream` (a cudaStream_t of the
 * context's device; NULL returns to the context's own stream).  The caller
 * keeps the stream alive while the context uses it. */
int mtpb_set_stream(mtpb_context *ctx, void *stream);

/* Model cutoff (largest pair max_dist), in Angstrom. */
int mtpb_cutoff(const mtpb_context *ctx, double *cutoff);

/* Extra neighbour-list radius beyond the cutoff (default 0).  With a skin the
 * list can be reused while atoms move less than skin/2; pairs beyond the
 * model cutoff are skipped by the kernels (potential_mtp.cpp:2842). */
int mtpb_set_skin(mtpb_context *ctx, double skin);

/* ---- structures: neighbour build + EFS ---------------------------------- */

/* Centres of the structures path: subsequent builds evaluate the site terms of
 * the first center_count atoms of the batch only (0 = every atom), with
 * neighbours drawn from all atoms.  Forces are then partial sums for all atoms
 * (the ghost contributions of MTPGpuBatchRequest, mtp_gpu_direct.h:451-517),
 * energies and virials cover the centres.  Used by domain decompositions that
 * reduce the partial forces across ranks; mtpb_loss_grad needs all atoms. */
int mtpb_set_center_count(mtpb_context *ctx, int center_count);

/* Builds the neighbour lists of all structures on the GPU (replaces
 * Neighborhoods(atoms, cutoff), base/neighborhood.cpp:149-157) and keeps them
 * in the context.  Per-atom neighbour sets equal the reference builder's bit
 * for bit (neighbour index and displacement vector). */
int mtpb_build_neighbors(mtpb_context *ctx, const mtpb_structures *in, int memory);

/* Number of directed edges of the list built last. */
int mtpb_neighbor_count(const mtpb_context *ctx, long *n_edges);

/* Copies the list built last into host arrays: offsets[N+1], nbr[E]
 * (structure-local atom index is nbr - atom_offsets[s]; nbr is global),
 * rij[E][3] (Neighborhood::pos_), shift[E] (packed periodic image, may be NULL). */
int mtpb_get_neighbors(const mtpb_context *ctx, int *offsets, int *nbr, double *rij, int *shift);

/* Energy, forces, virial (and site energies) of the structures whose
 * neighbour list was built last; replaces PotMTP::getEFS(Atoms&,
 * AnyNeighborhoods&) (potential_mtp.cpp:1899-1933).  Positions are taken from
 * that build.  Outputs are `memory`-side arrays.  An output with neither
 * forces nor stress asks for energies only (PotMTP::CalcE, the trainer's
 * energy_only branch): the reverse pass is skipped. */
int mtpb_efs_compute(mtpb_context *ctx, int memory, const mtpb_efs_output *out);

/* Convenience: build + compute in one call (PotMTP::getEFS(Atoms&),
 * potential_mtp.cpp:1892-1897, batched like calc_efs, apps/calc_efs.cpp:336-380).
 * reuse_neighbors != 0 keeps the previous list when the batch layout is
 * unchanged (MTPGpuComputeRequest::reuse_topology): the new positions are
 * uploaded and every edge vector is recomputed from its stored periodic image
 * (the atoms must stay within the skin of the last build).  For host arrays the
 * layout is checked; for device arrays the caller guarantees it. */
int mtpb_efs_structures(mtpb_context *ctx, const mtpb_structures *in, int memory,
                        int reuse_neighbors, const mtpb_efs_output *out);

/* ---- caller-supplied neighbour lists ------------------------------------ */

/* CSR request with explicit lists (MTPGpuBatchRequest,
 * mtp_gpu_direct.h:455-517).  Centres are atoms 0..center_count-1; atoms
 * center_count..ntotal-1 are ghosts that only appear as neighbours.
 * neighbor_vectors[E][3] (optional) gives r_ij directly; otherwise
 * r_ij = x[j] - x[i].  force[ntotal][3] receives (or, with
 * accumulate_force, adds) -dE/dx; site_virial[ntotal][6] (xx yy zz xy xz yz)
 * splits each pair term 0.5/0.25 onto both atoms as MLIPCore::compute does
 * (runtime/mtp/mlip.cpp:1164-1190); global_virial[6] is the sum. */
typedef struct mtpb_csr_request {
    int center_count;
    int ntotal;
    const int *offsets;           /* [center_count+1] */
    const int *neighbors;         /* [E] atom indices (masked with neighbor_mask) */
    int neighbor_mask;            /* e.g. 0x3fffffff for LAMMPS lists; -1 keeps all bits */
    const double *neighbor_vectors;  /* [E][3] or NULL */
    const int *types;             /* [ntotal] species index, -1 skips the atom */
    const double *x;              /* [ntotal][3] */
    double *force;                /* [ntotal][3] or NULL */
    int accumulate_force;
    double *total_energy;         /* [1] or NULL */
    double *site_energy;          /* [center_count] or NULL */
    double *site_virial;          /* [ntotal][6] or NULL */
    double *global_virial;        /* [6] or NULL */
} mtpb_csr_request;

/* Replaces MTPGpuDirect::compute_batch (mtp_gpu_direct.h:870) for the FP64
 * linear model. */
int mtpb_efs_csr(mtpb_context *ctx, const mtpb_csr_request *req, int memory);

/* The CSR request of mtpb_efs_csr for small systems, without any device
 * allocation: for callers that cannot call cudaMalloc while they run, such as
 * an MD engine or plug-in host that has already reserved the GPU's memory for
 * its own pool, or a real-time loop that must never enter the allocator.  It
 * has no counterpart in the reference.
 *
 * All arrays of `req` are device memory on the context's device; the context
 * must exist already (mtpb_create allocates the model's device data once).
 * Per-call scratch lives in one fixed device array inside the library (about
 * 9.6 MB, resident on every GPU that loads the library until exit), which
 * limits a call to 1024 centres, 4096 atoms including ghosts, 65536 edges and
 * models with at most 320 basic-moment slots (level 20 and below); larger
 * requests fail with MTPB_ERR_ARGUMENT / MTPB_ERR_UNSUPPORTED.  The first call
 * on a device looks up the array's device address; make that first call before
 * any stream capture.  Every call uses the same array, so calls that overlap on
 * the GPU (from two threads or two contexts on one device) race; the call
 * returns after its work has completed. */
int mtpb_efs_csr_noalloc(mtpb_context *ctx, const mtpb_csr_request *req);

/* LAMMPS pair-style request (MTPGpuComputeRequest, mtp_gpu_direct.h:326-450;
 * PairMLIPGpuDirect::compute, LAMMPS/USER-MLIP/pair_MLIP_gpu_direct.cpp:540-640):
 * full neighbour list, newton on, forces added to f for local and ghost
 * atoms.  type[i] is the LAMMPS type; type_map[type] gives the model species
 * or -1 to skip the atom. */
typedef struct mtpb_lammps_request {
    int inum;
    const int *ilist;               /* [inum] */
    const int *numneigh;            /* indexed by atom */
    const int *const *firstneigh;   /* indexed by atom */
    int neighbor_mask;
    int ntotal;                     /* local + ghost atoms */
    const int *type;                /* [ntotal] */
    const int *type_map;            /* [type_map_count] */
    int type_map_count;
    const double *x;                /* [ntotal][3] contiguous */
    double *f;                      /* [ntotal][3] accumulated */
    double *energy;                 /* [1] accumulated, or NULL */
    double *site_energy;            /* [ntotal] or NULL (written for centres) */
    double *site_virial;            /* [ntotal][6] accumulated, or NULL */
    double *virial;                 /* [6] accumulated, or NULL */
} mtpb_lammps_request;

/* Host arrays only. */
int mtpb_efs_lammps(mtpb_context *ctx, const mtpb_lammps_request *req);

/* ---- training: loss and coefficient gradient ---------------------------- */

/* Trainer_MTP loss settings (train/train_mtp.h:205-216). */
typedef struct mtpb_loss_weights {
    double weight_eng, weight_force, weight_stress;
    double weight_eng_power, weight_force_power, weight_stress_power;
} mtpb_loss_weights;

/* Labels of a structure batch (Atoms::energy_, forces_, stress_); a NULL
 * array disables that term for all structures. */
typedef struct mtpb_labels {
    const double *energy;   /* [S] */
    const double *forces;   /* [N][3] */
    const double *stress;   /* [S][9] virial, eV */
} mtpb_labels;

/* Loss and gradient of the structures whose neighbour list was built last
 * (Trainer_MTP::AccumulateGard without the penalty term,
 * train/train_mtp.cpp:3039-3094 with AddLossGard :3839-3996 and
 * PotMTP::AccumulateEFSCombinationGard, potential_mtp.cpp:6896-6922).
 * loss and grad are divided by the number of structures in `norm_count`
 * (pass the global count when shards are reduced across ranks, or 0 for the
 * local count).  metrics[7] = {total, energy, force, stress loss, squared
 * per-atom energy error, squared force error, squared stress error}
 * (un-normalised).  grad[K*K*mu*R + K + S] in the native order.  Labels and
 * outputs are `memory`-side arrays. */
int mtpb_loss_grad(mtpb_context *ctx, const mtpb_labels *labels, const mtpb_loss_weights *w,
                   int norm_count, int memory, double *loss, double *metrics, double *grad);

/* Finite check of the last mtpb_loss_grad call's loss, metrics and gradient,
 * made on the device by that call (the reference's check_training_values /
 * training_finite_kernel, runtime/mtp/gpu-direct/mtp_gpu_direct.cu:5395-5420).
 * Host-memory calls of mtpb_loss_grad run this check themselves and return
 * MTPB_ERR_NONFINITE; device-memory calls do not synchronise, so their caller
 * asks here (this call synchronises the context stream).  first_nonfinite
 * receives -1 when every value is finite, else the smallest index into
 * [loss, metrics[7], grad[...]] of a NaN or infinite value, and the call
 * returns MTPB_ERR_NONFINITE. */
int mtpb_check_training_values(mtpb_context *ctx, long *first_nonfinite);

/* Status of the device-side waits of the calls made since the last check.
 * The graph kernels give up a wait on their record stream after a bounded
 * number of polls and set a device flag instead of hanging (the reference
 * reports a failed kernel through its CUDA error checks).  Host-memory calls
 * read the flag themselves and return MTPB_ERR_CUDA; device-memory calls do
 * not synchronise, so their caller asks here: this call synchronises the
 * context stream and returns MTPB_ERR_CUDA, clearing the flag, when a wait
 * gave up (the results of the calls since the last check are then invalid),
 * else MTPB_OK. */
int mtpb_check_device_status(mtpb_context *ctx);

/* Test hook: sets the device flag as a wait that gave up would, without
 * running any kernel, so that a caller's handling of MTPB_ERR_CUDA can be
 * exercised. */
int mtpb_debug_flag_device_error(mtpb_context *ctx);

/* ---- diagnostics ---------------------------------------------------------- */

/* Device-side timing of the last mtpb_efs_compute/mtpb_efs_structures call,
 * milliseconds: [0] neighbour build (0 when reused), [1] forward moments,
 * [2] moment graph, [3] reverse moments, [4] force gather and reductions. */
int mtpb_last_timings(const mtpb_context *ctx, double *ms5);

/* Device-side timing of the last mtpb_loss_grad call, milliseconds: [0] EFS
 * pass, [1] loss terms, edge weights and species-pair buckets, [2] tangent
 * moments, [3] dual moment graph, [4] per-edge channel records, [5] radial
 * gradient, reductions and assembly.  No reference counterpart (diagnostic). */
int mtpb_last_train_timings(const mtpb_context *ctx, double *ms6);

/* Kernel launches issued by the last compute call. */
int mtpb_last_launch_count(const mtpb_context *ctx, int *launches);

/* Basic moments and their energy adjoints of the last EFS call, [N][nb] in
 * the model's basic ordering (host arrays, either may be NULL). */
int mtpb_get_site_moments(const mtpb_context *ctx, double *basic, double *adjoint);

/* Host-only inspection of the moment-graph program that the device executes
 * for a model (no device needed).  Outputs (each may be NULL): nslot = basic
 * moment slots of the selected kernel shape; slot_of_basic[nb]; nrows = graph
 * rows; one_row / zero_row; n_fwd / n_rev phase counts; phase_rows[n_fwd+n_rev];
 * n_records; records[n_records][4] as 32-bit words {s1 | s2 << 16,
 * out | flags << 16, low and high words of the coefficient}.  Call with
 * records == NULL first to size the buffer. */
int mtpb_graph_program(const mtpb_model_view *model, int *nslot, int *slot_of_basic, int *nrows,
                       int *one_row, int *zero_row, int *n_fwd, int *n_rev, int *phase_rows,
                       long *n_records, unsigned int *records);

/* Per-edge site energy derivatives dE_i/dr_ij of the last EFS call, [E][3]
 * in neighbour-list order (PotMTP::CalcSiteEFS buff_site_energy_ders). */
int mtpb_get_edge_derivatives(const mtpb_context *ctx, double *dedr);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* MTPB200_H */
