// ref_gpu_shim.cpp -- C entry points over the reference's own GPU trainer core.
//
// TEST INFRASTRUCTURE ONLY.  Compiled together with the unmodified reference
// sources runtime/mtp/gpu-direct/mtp_gpu_direct.cu, sog_gpu.cu,
// runtime/mtp/mlip.cpp and radial_basis_setup.cpp, read in place from the
// reference checkout (recipe: oracle/Makefile target `refgpu`; output
// oracle/_ref/librefgpu.so, git-ignored).  It calls only the reference's public
// API and pins the coefficient gradient of this repository against the
// reference's own implementation of it:
//   - MLIPCore::setup_from_text                  runtime/mtp/mlip.h:203-215
//   - MTPGpuDirect::set_device / initialize_from_mlip
//                                                runtime/mtp/gpu-direct/mtp_gpu_direct.h:801-813
//   - MTPGpuDirect::compute_batch (MTPGpuBatchRequest, :455-517), filled as
//     Potentials::MTPGpuBatch::request() does (potentials/mtp_gpu_adapter.cpp:1285-1307)
//   - MTPGpuDirect::prepare_loss (MTPGpuLossRequest, :561-579) with the
//     per-structure / per-atom weights of train/train_mtp_gpu.cpp:252-292
//   - MTPGpuDirect::accumulate_gradient (MTPGpuGradientRequest, :523-555) on
//     the prepared adjoints, as MTPGpuBatch::accumulate_prepared_gradient
//     (mtp_gpu_adapter.cpp:2173-2193)
// Every reduction runs in the reference's deterministic mode.
#include "runtime/mtp/gpu-direct/mtp_gpu_direct.h"
#include "runtime/mtp/mlip.h"

#include <exception>
#include <numeric>
#include <string>
#include <vector>

namespace
{
thread_local std::string g_error;

struct Handle
{
    MLIPCore::mlip *model = nullptr;
    MLIPCore::GpuDirect::MTPGpuDirect gpu;
    int gradient_count = 0;
};
} // namespace

extern "C" {

const char *refgpu_last_error()
{
    return g_error.c_str();
}

// Loads a .mtp text (species map identity over `species` types) and
// initialises the reference GPU evaluator on `device`.  gradient_count
// receives K*K*mu*R + K + S (the native PotMTP parameter order).
void *refgpu_create(const char *mtp_text, int species, int device, int *gradient_count)
{
    try
    {
        auto *h = new Handle;
        std::vector<int> tmap(species);
        std::iota(tmap.begin(), tmap.end(), 0);
        double cutoff = 0.0;
        h->model = MLIPCore::setup_from_text(std::string(mtp_text), tmap.data(), &cutoff,
                                             static_cast<std::size_t>(species));
        std::string err;
        if (!h->gpu.set_device(device, &err) || !h->gpu.initialize_from_mlip(*h->model, &err))
        {
            g_error = err;
            MLIPCore::destroy_mlip(h->model);
            delete h;
            return nullptr;
        }
        const auto *m = h->model;
        h->gradient_count = m->species_count * m->species_count * m->radial_func_count *
                                m->rb_size +
                            m->species_count + m->alpha_scalar_moments;
        if (gradient_count)
            *gradient_count = h->gradient_count;
        return h;
    }
    catch (const std::exception &ex)
    {
        g_error = ex.what();
        return nullptr;
    }
}

void refgpu_destroy(void *handle)
{
    auto *h = static_cast<Handle *>(handle);
    if (!h)
        return;
    MLIPCore::destroy_mlip(h->model);
    delete h;
}

// One training evaluation of a batch of complete structures: forward EFS,
// supervised loss with adjoints on the device, coefficient gradient.
//   structure_offsets[S+1]; per atom: offsets[N+1], neighbors[E] (atom index
//   within the batch), vectors[E*3] (r_ij), types[N], x[N*3];
//   labels: target_energy[S], energy_weight[S], target_force[N*3],
//   force_weight[N], target_stress[S*9], stress_weight[S].
// Outputs: metrics[7] (MTPGpuLossRequest order), gradient[gradient_count]
// (un-normalised sum over structures), and optionally force[N*3],
// site_energy[N], site_virial[N*6] of the forward pass.
int refgpu_loss_grad(void *handle, int n_struct, const int *structure_offsets, const int *offsets,
                     const int *neighbors, const double *vectors, const int *types,
                     const double *x, const double *target_energy, const double *energy_weight,
                     const double *target_force, const double *force_weight,
                     const double *target_stress, const double *stress_weight, double *metrics,
                     double *gradient, double *force, double *site_energy, double *site_virial)
{
    try
    {
        auto *h = static_cast<Handle *>(handle);
        const int n = structure_offsets[n_struct];
        std::vector<int> centers(n), center_structure(n);
        std::iota(centers.begin(), centers.end(), 0);
        for (int s = 0; s < n_struct; ++s)
            for (int i = structure_offsets[s]; i < structure_offsets[s + 1]; ++i)
                center_structure[i] = s;
        std::vector<double> f(3 * static_cast<std::size_t>(n)), se(n),
            sv(6 * static_cast<std::size_t>(n));
        double energy = 0.0;
        MLIPCore::GpuDirect::MTPGpuBatchRequest req;
        req.centers = centers.data();
        req.offsets = offsets;
        req.neighbors = offsets[n] ? neighbors : nullptr;
        req.neighbor_vectors = offsets[n] ? vectors : nullptr;
        req.center_count = n;
        req.nlocal = n;
        req.ntotal = n;
        req.type = types;
        req.x = x;
        req.force = f.data();
        req.site_energy = se.data();
        req.site_virial = sv.data();
        req.total_energy = &energy;
        req.accumulate_force = false;
        req.deterministic_reduction = true;
        std::string err;
        if (!h->gpu.compute_batch(req, &err))
        {
            g_error = "compute_batch: " + err;
            return -1;
        }
        if (force)
            std::copy(f.begin(), f.end(), force);
        if (site_energy)
            std::copy(se.begin(), se.end(), site_energy);
        if (site_virial)
            std::copy(sv.begin(), sv.end(), site_virial);
        MLIPCore::GpuDirect::MTPGpuLossRequest loss;
        loss.structure_count = n_struct;
        loss.structure_offsets = structure_offsets;
        loss.center_structure = center_structure.data();
        loss.target_energy = target_energy;
        loss.energy_weight = energy_weight;
        loss.target_force = target_force;
        loss.force_weight = force_weight;
        loss.target_stress = target_stress;
        loss.stress_weight = stress_weight;
        loss.metrics = metrics;
        loss.deterministic_reduction = true;
        if (!h->gpu.prepare_loss(loss, &err))
        {
            g_error = "prepare_loss: " + err;
            return -1;
        }
        MLIPCore::GpuDirect::MTPGpuGradientRequest grad;
        grad.structure_count = n_struct;
        grad.gradient = gradient;
        grad.gradient_count = h->gradient_count;
        grad.accumulate_gradient = false;
        grad.adjoints_on_device = true;
        grad.deterministic_reduction = true;
        if (!h->gpu.accumulate_gradient(grad, &err))
        {
            g_error = "accumulate_gradient: " + err;
            return -1;
        }
        return 0;
    }
    catch (const std::exception &ex)
    {
        g_error = ex.what();
        return -1;
    }
}

} // extern "C"
