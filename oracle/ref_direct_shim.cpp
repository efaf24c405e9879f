// ref_direct_shim.cpp -- C entry points over the reference-side binding.
//
// TEST INFRASTRUCTURE ONLY.  Compiles the binding a maintainer of the
// reference would add (imr-mlp_b200/bindings/mtpb_direct.hpp, class
// MTPB200Direct) against the reference's own headers, together with the
// unmodified reference sources runtime/mtp/mlip.cpp and
// radial_basis_setup.cpp (read in place from the reference checkout), and
// links the product library libmtpb200.so.  Recipe: oracle/Makefile target
// `refdirect`; output oracle/_ref/librefdirect.so (git-ignored).  The GPU
// tests compare what comes back through the binding with MLIPCore::compute.
#include "mtpb_direct.hpp"

#include <exception>
#include <string>
#include <vector>

namespace
{
thread_local std::string g_error;

struct Handle
{
    MLIPCore::mlip *model = nullptr;
    mtpb::MTPB200Direct gpu;
};
} // namespace

extern "C" {

const char *refdirect_last_error()
{
    return g_error.c_str();
}

// .mtp text loaded by MLIPCore::setup_from_text (type i -> species i), then
// MTPB200Direct::set_device + initialize_from_mlip.
void *refdirect_create(const char *mtp_text, int species, int device)
{
    try
    {
        auto *h = new Handle;
        std::vector<int> tmap(species);
        for (int i = 0; i < species; ++i)
            tmap[i] = i;
        double cutoff = 0.0;
        h->model = MLIPCore::setup_from_text(std::string(mtp_text), tmap.data(), &cutoff,
                                             static_cast<std::size_t>(species));
        if (!h->gpu.set_device(device, &g_error) || !h->gpu.initialize_from_mlip(*h->model, &g_error))
        {
            MLIPCore::destroy_mlip(h->model);
            delete h;
            return nullptr;
        }
        return h;
    }
    catch (const std::exception &ex)
    {
        g_error = ex.what();
        return nullptr;
    }
}

void refdirect_destroy(void *handle)
{
    auto *h = static_cast<Handle *>(handle);
    if (!h)
        return;
    MLIPCore::destroy_mlip(h->model);
    delete h;
}

// MTPGpuDirect::compute_batch request filled as Potentials::MTPGpuBatch::
// request() does (potentials/mtp_gpu_adapter.cpp:1285-1307), host arrays.
int refdirect_compute_batch(void *handle, int center_count, int ntotal, const int *offsets,
                            const int *neighbors, const double *vectors, const int *type,
                            const double *x, double *force, double *energy, double *site_energy,
                            double *site_virial, double *global_virial)
{
    auto *h = static_cast<Handle *>(handle);
    std::vector<int> centers(center_count);
    for (int i = 0; i < center_count; ++i)
        centers[i] = i;
    MLIPCore::GpuDirect::MTPGpuBatchRequest r;
    r.centers = centers.data();
    r.offsets = offsets;
    r.neighbors = neighbors;
    r.neighbor_vectors = vectors;
    r.center_count = center_count;
    r.nlocal = center_count;
    r.ntotal = ntotal;
    r.type = type;
    r.x = x;
    r.force = force;
    r.total_energy = energy;
    r.site_energy = site_energy;
    r.site_virial = site_virial;
    r.global_virial = global_virial;
    r.accumulate_force = false;
    return h->gpu.compute_batch(r, &g_error) ? 0 : -1;
}

// MTPGpuDirect::compute_lammps request (LAMMPS row pointers over contiguous
// x / force / site_virial storage); neighbours of atom i are
// flat[off[i] .. off[i] + numneigh[i]).
int refdirect_compute_lammps(void *handle, int inum, const int *ilist, int ntotal, const int *type,
                             double *x, const int *numneigh, const int *off, const int *flat,
                             int mask, double *energy, double *site_energy, double *force,
                             double *site_virial, double *global_virial)
{
    auto *h = static_cast<Handle *>(handle);
    std::vector<double *> xr(ntotal), fr(ntotal), vr(ntotal);
    std::vector<int *> nr(ntotal);
    for (int i = 0; i < ntotal; ++i)
    {
        xr[i] = x + 3 * static_cast<std::size_t>(i);
        fr[i] = force + 3 * static_cast<std::size_t>(i);
        vr[i] = site_virial ? site_virial + 6 * static_cast<std::size_t>(i) : nullptr;
        nr[i] = const_cast<int *>(flat) + off[i];
    }
    MLIPCore::GpuDirect::MTPGpuComputeRequest r;
    r.ilist = ilist;
    r.numneigh = numneigh;
    r.firstneigh = nr.data();
    r.inum = inum;
    r.nlocal = inum;
    r.ntotal = ntotal;
    r.type = type;
    r.x = xr.data();
    r.force = fr.data();
    r.total_energy = energy;
    r.site_energy = site_energy;
    r.site_virial = site_virial ? vr.data() : nullptr;
    r.global_virial = global_virial;
    r.neighbor_index_mask = mask;
    return h->gpu.compute_lammps(r, &g_error) ? 0 : -1;
}

} // extern "C"
