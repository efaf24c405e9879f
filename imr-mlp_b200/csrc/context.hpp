// context.hpp -- the context object behind the C ABI and the helpers
// shared by the API translation units.
#pragma once

#include "internal.hpp"
#include "neighbors.hpp"
#include "plan.hpp"

#include "../../include/mtpb200.h"

#include <cuda_runtime.h>

#include <string>
#include <vector>

struct mtpb_context;

namespace mtpb {

// Device-resident state of the training evaluator (training.cu).
struct TrainingState {
    bool ready = false;               // gradient program uploaded for the model
    DagDevRec *recs = nullptr;        // dual-graph records (grad.cu layout)
    std::vector<DagDevRec> h_recs;
    int *moment_energy = nullptr;     // moment coefficient -> energy-moment index
    long bucket_epoch = -1;           // edge_epoch the pair buckets belong to
    int *perm = nullptr;              // edges sorted by species pair
    long *bounds = nullptr;           // bucket start positions [K*K+2]
    cudaEvent_t ev[7] = {};           // timing events of the last call
    bool ev_valid = false;
    int *nonfinite = nullptr;         // finite check of the last call's outputs
};
int upload_training_program(mtpb_context *c);
// Reads the finite check of the last mtpb_loss_grad call (synchronises the
// context stream); first_bad = -1 when every value was finite.
int training_values_status(mtpb_context *c, long *first_bad);

int fail(int status, const std::string &msg);
int cuda_fail(cudaError_t e, const char *where);

} // namespace mtpb

#define CUDA_TRY(expr, where)                                                                      \
    do {                                                                                           \
        cudaError_t _e = (expr);                                                                   \
        if (_e != cudaSuccess)                                                                     \
            return ::mtpb::cuda_fail(_e, where);                                                           \
    } while (0)

struct mtpb_context {
    int device = 0;
    cudaStream_t stream = nullptr;      // stream in use
    cudaStream_t own_stream = nullptr;  // stream created by the context
    mtpb::ModelHost model;
    int shape = -1;
    int nslot = 0;
    std::vector<int> slot_of_basic;
    mtpb::DagPlan plan;
    std::vector<mtpb::DagDevRec> h_recs;   // plan records in the kernel's layout
    mtpb::DeviceArena arena;
    double skin = 0.0;
    // device model data
    double *d_radial = nullptr, *d_species = nullptr;
    // RBPolyB pairs: T_p(i, j) = N_j M_p(i, j), [K*K][R][R], which maps the
    // gradient of the folded coefficients back to the model's (NULL: none)
    double *d_poly = nullptr;
    mtpb::PairParams *d_pairs = nullptr;
    mtpb::DagDevRec *d_recs = nullptr;
    int *d_phase_row0 = nullptr;
    int *d_err = nullptr;   // device error flag (bounded waits that gave up)
    // current batch (structures path)
    int nstruct = 0, natoms = 0, ntotal = 0;   // natoms = centres, ntotal = all atoms
    int center_count_req = 0;                  // mtpb_set_center_count (0 = all atoms)
    long nedges = 0;
    bool have_list = false;
    std::vector<int> h_atom_offsets;
    std::vector<double> h_cells;
    mtpb::NbResult nb;
    const int *d_types = nullptr;
    double *d_x_build = nullptr;          // positions of the last build
    const mtpb::NbStruct *d_ns = nullptr;  // structures of the last build
    const int *d_offsets = nullptr;
    int *d_group_maxdeg = nullptr;
    int *d_seg_begin = nullptr, *d_seg_end = nullptr, *d_struct_seg0 = nullptr;
    int nseg = 0;
    int npad = 0;
    // timings
    cudaEvent_t ev[6] = {};
    bool ev_valid = false;
    bool nb_built_this_call = false;
    int launches = 0;
    int pending_launches = 0;   // neighbour build / refresh launches of this call
    bool have_efs = false;
    bool have_dedr = false;   // the last EFS call ran the reverse pass
    long edge_epoch = 0;     // advanced whenever the edge list or its vectors change
    // a reuse step with a skin leaves the edge vectors to the active-edge pass
    // of the next compute (one shot)
    mtpb::EdgeRefresh refresh{};
    bool refresh_pending = false;
    int dag_atoms_env = 0;   // MTPB_DAG_ATOMS override of the graph block width
    bool force_global_rows = false;   // MTPB_DAG_GLOBAL_ROWS=1
    // pinned staging of the per-build segment tables; stage_ev marks the end of
    // its last upload
    int *h_stage = nullptr;
    size_t h_stage_cap = 0;
    cudaEvent_t stage_ev = nullptr;
    bool stage_pending = false;
    mtpb::TrainingState train;
};


namespace mtpb {
int set_device(mtpb_context *c);
// Reads and clears the device error flag (call after a stream sync).
int check_device_error(mtpb_context *c);
EdgeArgs edge_args(const mtpb_context *c, int ncenter, const int *types, const int *offsets,
                   const int *nbr, const double *rx, const double *ry, const double *rz);
// beyond_cutoff: the list may hold pairs beyond the model cutoff (a skin or a
// caller's list), which are then skipped through an active-edge list
// refresh (may be NULL, needs beyond_cutoff): the list's edge vectors are
// recomputed by the active-edge pass
int run_moments(mtpb_context *c, int ncenter, const int *types, const int *offsets,
                const int *nbr, const double *rx, const double *ry, const double *rz,
                double *site_energy, double *dx, double *dy, double *dz, bool reverse,
                long nedges, bool beyond_cutoff, const EdgeRefresh *refresh = nullptr);
int efs_compute(mtpb_context *c, int memory, const mtpb_efs_output *out, bool forces_needed);
int csr_compute(mtpb_context *c, const mtpb_csr_request *req, int memory);
int lammps_compute(mtpb_context *c, const mtpb_lammps_request *req);
int loss_grad_compute(mtpb_context *c, const mtpb_labels *labels, const mtpb_loss_weights *w,
                      int norm_count, int memory, double *loss, double *metrics, double *grad);
} // namespace mtpb
