/*
 * mtp_oracle.h -- CPU restatement of the reference MTP hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * implementation in imr-mlp_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and the cpu_baseline leg of bench.py load it.  The product library never
 * links, loads or calls it, and there is no CPU fallback built on it.
 *
 * Everything here restates, in plain C and in the reference's operation
 * order, the functions named in each comment (paths are relative to the
 * reference project root):
 *   - neighbour lists:  base/neighborhoods_base.h:31-126 (images, wrapping),
 *                       base/neighborhood.cpp:77-140 (pair filter and the
 *                       two-direction emission)
 *   - radial basis:     basis/basis.cpp:148-164 (RBasis_Chebyshev::calc_der),
 *                       :265-280 (RBChebyCos), :644-673 (RBChebyshevPoly4),
 *                       :776-806 (RBChebyshevPoly5), :937-1013
 *                       (RBChebyshevConfigurable with basis/cutoff.cpp and
 *                       basis/xtrans.cpp)
 *   - site EFS:         potentials/potential_mtp.cpp:2813-2925, 2959-2984,
 *                       3292-3305, 2938-2957 and the scatter in 1899-1933
 *   - parameter grad:   potentials/potential_mtp.cpp:3348-3550, 3312-3318,
 *                       6896-6922
 *   - loss:             train/train_mtp.cpp:2552-2568, 3839-3996, 3039-3094
 *
 * Parity of this restatement is pinned against the reference itself: the
 * neighbour lists and the MLIPCore EFS compiled from the reference sources
 * (oracle/ref_shim.cpp, built into oracle/_ref), central finite differences
 * for the gradient, and the golden fixtures under tests/golden.
 */
#ifndef MTP_ORACLE_H
#define MTP_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* Radial basis family of a pair (same layout and numbering as
 * mtpb_radial_family in include/mtpb200.h): type 0 RBChebyshev, 1 RBChebyCos,
 * 2 RBChebyshevPoly5, 3 RBChebyshevConfigurable, 4 RBChebyshevPoly4. */
typedef struct oracle_radial_family {
    int type, cutoff_type, shift_type, one_minus_chebyshev;
    double b, r1, r2, lambda, scale_lambda;
    const double *poly_matrix;   /* RBPolyB / RBPolyBCos: [R*R] column-major */
    const double *poly_norm;     /* RBPolyB / RBPolyBCos: [R] */
} oracle_radial_family;

/* Flat model description.  Same field order as mtpb_model_view in
 * include/mtpb200.h so one Python-side builder can fill both. */
typedef struct oracle_model {
    int species_count;        /* K */
    int radial_func_count;    /* mu count */
    int rb_size;              /* R */
    int radial_basis_split;   /* 0: one basis, 1: one basis per ordered pair */
    const double *min_dist;   /* [1] or [K*K] */
    const double *max_dist;   /* [1] or [K*K] */
    double scaling;
    int alpha_moments_count;
    int alpha_index_basic_count;
    int alpha_index_times_count;
    int alpha_scalar_moments;
    const int *alpha_index_basic;    /* [nb][4] = {mu, a, b, c} */
    const int *alpha_index_times;    /* [T][4]  = {l1, l2, c, id} */
    const int *alpha_moment_mapping; /* [S] */
    const double *radial_coeffs;     /* [K*K][mu][R] */
    const double *species_coeffs;    /* [K] */
    const double *moment_coeffs;     /* [S] */
    const oracle_radial_family *radial_family; /* NULL: RBChebyshev; [1] or [K*K] */
} oracle_model;

/* Neighbour lists of one structure with the reference's default builder
 * semantics.  cell is row-major with lattice vectors as rows; pbc[3] flags
 * periodic axes.  Returns the number of directed edges (or -1 on error).
 * When offsets/nbr/rij are non-NULL they receive a CSR list: offsets[n+1],
 * nbr[E] (original atom index), rij[3E] (displacement, bit-exact with the
 * reference).  Each atom's list is sorted by (nbr, rij) so that two lists can
 * be compared as sets with a plain element-wise comparison. */
long oracle_neighbors(const double *cell, const int *pbc, int n, const double *pos,
                      double cutoff, int *offsets, int *nbr, double *rij);

/* Wrapped positions as computed by NeighborhoodsBase::load_positions. */
void oracle_wrap_positions(const double *cell, const int *pbc, int n, const double *pos,
                           double *wrapped);

/* Energy, forces and virial of one structure (PotMTP::getEFS).  types are
 * species indices (0..K-1).  offsets/nbr/rij describe the neighbour lists.
 * stress[9] is row-major, eV (Atoms::stress_ convention). site_energy may be
 * NULL. Returns 0 on success. */
int oracle_efs(const oracle_model *m, int n, const int *types, const int *offsets,
               const int *nbr, const double *rij, double *energy, double *site_energy,
               double *forces, double *stress);

/* Per-site energy derivatives dE_i/dr_ij (buff_site_energy_ders) for every
 * edge, row-major [E][3].  Used by the edge-level parity tests. */
int oracle_site_derivatives(const oracle_model *m, int n, const int *types,
                            const int *offsets, const int *nbr, const double *rij,
                            double *site_energy, double *dedr);

/* Basic moments and adjoints (dE/db) of every site, [n][nb] each, in the
 * model's basic ordering.  Either output may be NULL. */
int oracle_site_moments(const oracle_model *m, int n, const int *types, const int *offsets,
                        const int *nbr, const double *rij, double *basic, double *adjoint);

/* Training loss settings (Trainer_MTP defaults: weight_eng 1, weight_force
 * 0.01, weight_stress 0.0001, powers 1, 0, 1). */
typedef struct oracle_loss_weights {
    double weight_eng, weight_force, weight_stress;
    double weight_eng_power, weight_force_power, weight_stress_power;
} oracle_loss_weights;

/* Loss and coefficient gradient of a set of structures (Trainer_MTP::
 * AccumulateGard without the penalty term): for each structure the EFS,
 * residuals and loss adjoints (AddLossGard), then
 * AccumulateEFSCombinationGard; finally loss and gradient are divided by the
 * number of structures.  Atoms of structure s are atom_offsets[s] ..
 * atom_offsets[s+1]-1 in the global arrays; the neighbour CSR uses global atom
 * indices and never crosses structures.  has_forces/has_stress/has_energy are
 * per-structure flags (NULL = all present).  metrics[7] receives the
 * un-normalised [total, energy, force, stress, sq per-atom energy error,
 * sq force error, sq stress error] sums; grad receives
 * [radial K*K*mu*R][species K][moment S], normalised. */
int oracle_loss_grad(const oracle_model *m, const oracle_loss_weights *w, int n_struct,
                     const int *atom_offsets, const int *types, const int *offsets,
                     const int *nbr, const double *rij, const double *target_energy,
                     const double *target_forces, const double *target_stress,
                     const int *has_energy, const int *has_forces, const int *has_stress,
                     double *loss, double *metrics, double *grad);

/* Forward + reverse of one structure into per-structure outputs, batched over
 * structures (OpenMP over structures when available).  Outputs energy[s],
 * forces[3N], stress[9 s]. */
int oracle_efs_batch(const oracle_model *m, int n_struct, const int *atom_offsets,
                     const int *types, const int *offsets, const int *nbr, const double *rij,
                     double *energy, double *forces, double *stress, int threads);

#ifdef __cplusplus
}
#endif
#endif
