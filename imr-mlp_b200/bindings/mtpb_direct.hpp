// mtpb_direct.hpp -- reference-side C++ binding of the B200 path.
//
// A drop-in for MLIPCore::GpuDirect::MTPGpuDirect
// (runtime/mtp/gpu-direct/mtp_gpu_direct.h:789-926) for the linear FP64 MTP:
// the same method names, the same borrowed request structs (MTPGpuBatchRequest
// :455-517 for compute_batch, MTPGpuComputeRequest :326-450 for
// compute_lammps) and the same error convention (bool return, message in an
// optional std::string, no exceptions).  A maintainer of the reference
// includes this header where MTPGpuDirect is used today and links
// libmtpb200.so; only the C ABI of include/mtpb200.h is called.
//
// Include paths: the reference project root (runtime/mtp/mlip.h and the
// gpu-direct request types) and this project's include/ directory.
//
// Model upload follows MTPGpuDirect::initialize_from_mlip
// (mtp_gpu_direct.cu:6814-6870): the alpha index tables, the scalar mapping,
// the coefficients and, per ordered species pair, the radial basis descriptor
// (mlip::radial_basis_t, runtime/mtp/mlip.h:166-186), whose rb / cutoff /
// transform enums share the numbering of mtpb_radial_family; RBPolyB pairs
// hand over the loader's orthogonalisation matrix and normalisations.  Atom types of
// both requests go through the model's type mapping (mlip::mapping_data(), as
// MLIPCore::compute does, mlip.cpp:910-964).
#pragma once

#include "mtpb200.h"
#include "runtime/mtp/gpu-direct/mtp_gpu_direct.h"
#include "runtime/mtp/mlip.h"

#include <cstddef>
#include <string>
#include <vector>

namespace mtpb {

class MTPB200Direct {
  public:
    MTPB200Direct() = default;
    ~MTPB200Direct()
    {
        if (ctx_)
            mtpb_destroy(ctx_);
    }
    MTPB200Direct(const MTPB200Direct &) = delete;
    MTPB200Direct &operator=(const MTPB200Direct &) = delete;

    static bool available_device_count(int *count, std::string *error = nullptr)
    {
        return check(mtpb_device_count(count), error);
    }

    bool set_device(int device_id, std::string *error = nullptr)
    {
        if (device_id < 0)
            return fail("device id must be >= 0", error);
        device_ = device_id;
        return true;
    }

    bool initialize_from_mlip(const MLIPCore::mlip &p, std::string *error = nullptr)
    {
        const int np = p.pair_radial_basis_count;
        std::vector<double> rmin, rmax;
        std::vector<mtpb_radial_family> fam;
        if (np) {
            if (np != p.species_count * p.species_count)
                return fail("pair radial bases must cover every ordered species pair", error);
            for (int k = 0; k < np; ++k) {
                const auto &b = p.pair_radial_bases[k];
                if (b.scaling != p.scaling)
                    return fail("per-pair radial scaling differs from the model scaling", error);
                if (b.size != p.rb_size)
                    return fail("per-pair radial basis size differs from rb_size", error);
                rmin.push_back(b.min_dist);
                rmax.push_back(b.max_dist);
                fam.push_back(family(b.rb, b.cutoff, b.transform, b.one_minus_chebyshev,
                                     b.cutoff_parameter, b.cutoff_r1, b.cutoff_r2,
                                     b.transform_parameter, b.transform_scale_parameter));
                // RBPolyB / RBPolyBCos: the loader's own orthogonalisation
                // matrix (ill-conditioned: it is data, not recomputed)
                if (b.rb == MLIPCore::mlip::RB_POLYB || b.rb == MLIPCore::mlip::RB_POLYBCOS) {
                    if (b.polynomial_matrix.size() != (size_t)p.rb_size * p.rb_size ||
                        b.polynomial_normalizations.size() != (size_t)p.rb_size)
                        return fail("RBPolyB pair without its polynomial data", error);
                    fam.back().poly_matrix = b.polynomial_matrix.data();
                    fam.back().poly_norm = b.polynomial_normalizations.data();
                }
            }
        } else {
            rmin.push_back(p.min_dist);
            rmax.push_back(p.max_dist);
            fam.push_back(family(p.rb, MLIPCore::mlip::RB_CUTOFF_QUADRATIC,
                                 MLIPCore::mlip::RB_TRANSFORM_LINEAR, false, 0.0, 0.0, 0.0, 0.0,
                                 0.0));
        }
        for (const auto &f : fam)
            if (f.type > MTPB_RB_POLYB_COS || (!np && f.type >= MTPB_RB_POLYB))
                return fail("radial basis family not implemented on the B200 path "
                            "(the legacy families)",
                            error);
        mtpb_model_view v{};
        v.species_count = p.species_count;
        v.radial_func_count = p.radial_func_count;
        v.rb_size = p.rb_size;
        v.radial_basis_split = np ? 1 : 0;
        v.min_dist = rmin.data();
        v.max_dist = rmax.data();
        v.scaling = p.scaling;
        v.alpha_moments_count = p.alpha_moments_count;
        v.alpha_index_basic_count = p.alpha_index_basic_count;
        v.alpha_index_times_count = p.alpha_index_times_count;
        v.alpha_scalar_moments = p.alpha_scalar_moments;
        basic_.resize(4 * (std::size_t)p.alpha_index_basic_count);
        for (int i = 0; i < p.alpha_index_basic_count; ++i) {
            const auto &a = p.alpha_index_basic[i];
            basic_[4 * i] = a.mu;
            basic_[4 * i + 1] = a.b1;
            basic_[4 * i + 2] = a.b2;
            basic_[4 * i + 3] = a.b3;
        }
        times_.resize(4 * (std::size_t)p.alpha_index_times_count);
        for (int i = 0; i < p.alpha_index_times_count; ++i) {
            const auto &t = p.alpha_index_times[i];
            times_[4 * i] = t.l1;
            times_[4 * i + 1] = t.l2;
            times_[4 * i + 2] = t.c;
            times_[4 * i + 3] = t.id;
        }
        v.alpha_index_basic = basic_.data();
        v.alpha_index_times = times_.data();
        v.alpha_moment_mapping = p.alpha_moment_mapping;
        v.radial_coeffs = p.radial_coeffs;
        v.species_coeffs = p.species_coeffs;
        v.moment_coeffs = p.moment_coeffs;
        // the plain RBChebyshev single basis needs no descriptor
        const bool plain = !np && fam[0].type == MTPB_RB_CHEBYSHEV;
        v.radial_family = plain ? nullptr : fam.data();
        if (ctx_) {
            mtpb_destroy(ctx_);
            ctx_ = nullptr;
        }
        if (!check(mtpb_create(device_, &v, &ctx_), error))
            return false;
        const int *map = p.mapping_data();
        type_map_.assign(map, map + p.mapping_size());
        return true;
    }

    bool update_coefficients(const double *radial, const double *species, const double *moment,
                             std::string *error = nullptr)
    {
        if (!ready(error))
            return false;
        return check(mtpb_update_coefficients(ctx_, radial, species, moment), error);
    }

    // MTPGpuBatchRequest with host arrays: centres are atoms 0..center_count-1
    // in order (the adapter's centers list, potentials/mtp_gpu_adapter.cpp:
    // 1121-1123), neighbour_vectors optional.
    bool compute_batch(const MLIPCore::GpuDirect::MTPGpuBatchRequest &r,
                       std::string *error = nullptr)
    {
        if (!ready(error))
            return false;
        if (r.device_input || r.device_moments.present() || r.sog_grid ||
            r.center_energy_weights || r.device_center_energy_weights)
            return fail("only the linear host-array batch request is implemented", error);
        if (r.centers)
            for (int i = 0; i < r.center_count; ++i)
                if (r.centers[i] != i)
                    return fail("centers must be 0..center_count-1 in order", error);
        if (r.ntotal > 0 && !r.type)
            return fail("type is required", error);
        species_.resize((std::size_t)r.ntotal);
        for (int i = 0; i < r.ntotal; ++i) {
            const int t = r.type[i];
            species_[i] = (t >= 0 && t < (int)type_map_.size()) ? type_map_[t] : -1;
        }
        mtpb_csr_request q{};
        q.center_count = r.center_count;
        q.ntotal = r.ntotal;
        q.offsets = r.offsets;
        q.neighbors = r.neighbors;
        q.neighbor_mask = -1;
        q.neighbor_vectors = r.neighbor_vectors;
        q.types = species_.data();
        q.x = r.x;
        q.force = r.compute_forces ? r.force : nullptr;
        q.accumulate_force = r.accumulate_force ? 1 : 0;
        q.total_energy = r.compute_global_energy ? r.total_energy : nullptr;
        q.site_energy = r.compute_site_energy ? r.site_energy : nullptr;
        q.site_virial = r.compute_forces ? r.site_virial : nullptr;
        q.global_virial = r.compute_forces ? r.global_virial : nullptr;
        return check(mtpb_efs_csr(ctx_, &q, MTPB_MEMORY_HOST), error);
    }

    // MTPGpuComputeRequest (LAMMPS pair style): full list, newton on, forces
    // added to force[][] for local and ghost atoms; x, force and site_virial
    // rows contiguous from row zero (the request's own contract).
    bool compute_lammps(const MLIPCore::GpuDirect::MTPGpuComputeRequest &r,
                        std::string *error = nullptr)
    {
        if (!ready(error))
            return false;
        if (r.device_input || r.device_moments.present() || r.sog_grid ||
            r.center_energy_weights || r.device_center_energy_weights || r.neighbor_vectors)
            return fail("only the linear host-array LAMMPS request is implemented", error);
        if (!r.accumulate_force)
            return fail("the LAMMPS request adds forces (accumulate_force must be true)", error);
        mtpb_lammps_request q{};
        q.inum = r.inum;
        q.ilist = r.ilist;
        q.numneigh = r.numneigh;
        q.firstneigh = r.firstneigh;
        q.neighbor_mask = r.neighbor_index_mask;
        q.ntotal = r.ntotal;
        q.type = r.type;
        q.type_map = type_map_.data();
        q.type_map_count = (int)type_map_.size();
        q.x = r.ntotal ? r.x[0] : nullptr;
        q.f = r.ntotal ? r.force[0] : nullptr;
        // mtpb_efs_lammps adds the energy and virial into the caller's values;
        // MTPGpuComputeRequest overwrites them
        double e = 0.0, w[6] = {0, 0, 0, 0, 0, 0};
        q.energy = r.total_energy ? &e : nullptr;
        q.site_energy = r.site_energy;
        q.site_virial = (r.site_virial && r.ntotal) ? r.site_virial[0] : nullptr;
        q.virial = r.global_virial ? w : nullptr;
        if (!check(mtpb_efs_lammps(ctx_, &q), error))
            return false;
        if (r.total_energy)
            *r.total_energy = e;
        if (r.global_virial)
            for (int k = 0; k < 6; ++k)
                r.global_virial[k] = w[k];
        return true;
    }

    mtpb_context *context() const { return ctx_; }

  private:
    template <class Rb, class Cut, class Tr>
    static mtpb_radial_family family(Rb rb, Cut cut, Tr tr, bool one_minus, double b, double r1,
                                     double r2, double lambda, double scale_lambda)
    {
        mtpb_radial_family f{};
        f.type = (int)rb;
        f.cutoff_type = (int)cut;
        f.shift_type = (int)tr;
        f.one_minus_chebyshev = one_minus ? 1 : 0;
        f.b = b;
        f.r1 = r1;
        f.r2 = r2;
        f.lambda = lambda;
        f.scale_lambda = scale_lambda;
        return f;
    }
    static bool fail(const char *msg, std::string *error)
    {
        if (error)
            *error = msg;
        return false;
    }
    static bool check(int rc, std::string *error)
    {
        if (rc == MTPB_OK)
            return true;
        if (error)
            *error = mtpb_last_error();
        return false;
    }
    bool ready(std::string *error) const
    {
        return ctx_ ? true : fail("initialize_from_mlip has not succeeded", error);
    }

    int device_ = 0;
    mtpb_context *ctx_ = nullptr;
    std::vector<int> basic_, times_, species_, type_map_;
};

} // namespace mtpb
