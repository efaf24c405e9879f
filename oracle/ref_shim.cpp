// ref_shim.cpp -- C entry points over the reference's own CPU code.
//
// TEST INFRASTRUCTURE ONLY.  This file is compiled together with unmodified
// reference sources read in place from the reference checkout (the recipe is
// oracle/Makefile; the output goes to oracle/_ref/, which is git-ignored).
// Nothing here is copied from the reference: it only calls its public API:
//   - Neighborhoods(const Atoms&, double)  base/neighborhood.h:27-42, built
//     with -DBOXED_NEBH (the reference's default Makefile define)
//   - MLIPCore::setup_from_text / create_mlip_buffer / compute
//     runtime/mtp/mlip.h:203-215 (the LAMMPS USER-MLIP CPU core)
//   - MLIPCore::Cpu::Executor is not needed: compute() is the same arithmetic.
#include "base/neighborhood.h"
#include "base/structures.h"
#include "runtime/mtp/mlip.h"

#include <algorithm>
#include <cstring>
#include <omp.h>
#include <exception>
#include <string>
#include <vector>

namespace
{
thread_local std::string g_error;
}

extern "C" {

const char *ref_last_error()
{
    return g_error.c_str();
}

// Builds the reference neighbour lists of one structure.  First call with
// nbr == nullptr to get the edge count; second call fills offsets[n+1],
// nbr[E] and rij[3E] in the reference's own per-atom order.
long ref_neighbors(const double *cell, const int *pbc, int n, const double *pos, double cutoff,
                   int *offsets, int *nbr, double *rij)
{
    try
    {
        Atoms atom;
        for (int i = 0; i < 3; ++i)
            for (int j = 0; j < 3; ++j)
                atom.cell_(i, j) = cell[3 * i + j];
        for (int a = 0; a < 3; ++a)
            atom.pbc_[a] = pbc[a] != 0;
        atom.pos_.resize(n);
        atom.chemmap_.assign(n, 0);
        for (int i = 0; i < n; ++i)
            atom.pos_[i] = Eigen::RowVector3d(pos[3 * i], pos[3 * i + 1], pos[3 * i + 2]);
        Neighborhoods nbhs(atom, cutoff);
        long total = 0;
        for (int i = 0; i < nbhs.size(); ++i)
            total += nbhs[i].nbhcount_;
        if (offsets)
        {
            long e = 0;
            for (int i = 0; i < n; ++i)
            {
                offsets[i] = static_cast<int>(e);
                if (i < nbhs.size())
                {
                    const Neighborhood &nb = nbhs[i];
                    for (int k = 0; k < nb.nbhcount_; ++k, ++e)
                    {
                        if (nbr)
                            nbr[e] = nb.indices_[k];
                        if (rij)
                            for (int a = 0; a < 3; ++a)
                                rij[3 * e + a] = nb.pos_[k][a];
                    }
                }
            }
            offsets[n] = static_cast<int>(e);
        }
        return total;
    }
    catch (const std::exception &ex)
    {
        g_error = ex.what();
        return -1;
    }
}

// MLIPCore model handle from .mtp text.  type_map[t] maps caller atom types
// to model species (LAMMPS style); cutoff receives the model cutoff.
void *ref_mlip_setup(const char *text, const int *type_map, int type_count, double *cutoff)
{
    try
    {
        return MLIPCore::setup_from_text(std::string(text), type_map, cutoff,
                                         static_cast<std::size_t>(type_count));
    }
    catch (const std::exception &ex)
    {
        g_error = ex.what();
        return nullptr;
    }
}

// PolyB / PolyBCos data of one ordered species pair as MLIPCore's loader
// computed it (runtime/mtp/radial_basis_setup.cpp): the column-major
// orthogonalisation matrix [size*size] and the power normalisations [size].
// Returns the basis size, 0 when the pair's basis is not a PolyB family, -1 on
// a bad pair index.  Either output may be null.
int ref_mlip_polyb(void *handle, int pair, double *matrix, double *normalizations)
{
    auto *p = static_cast<MLIPCore::mlip *>(handle);
    if (pair < 0 || pair >= p->pair_radial_basis_count)
        return -1;
    const auto &b = p->pair_radial_bases[pair];
    if (b.rb != MLIPCore::mlip::RB_POLYB && b.rb != MLIPCore::mlip::RB_POLYBCOS)
        return 0;
    if (matrix)
        std::copy(b.polynomial_matrix.begin(), b.polynomial_matrix.end(), matrix);
    if (normalizations)
        std::copy(b.polynomial_normalizations.begin(), b.polynomial_normalizations.end(),
                  normalizations);
    return b.size;
}

// The .mtp text MLIPCore's loader derives from a model file (a GPM bundle or
// an .mtp file; runtime/mtp/mlip.cpp:350-423).  Returns the text length and
// copies at most cap bytes (with a terminating zero) into buf; -1 on error.
long ref_read_model_text(const char *path, char *buf, long cap)
{
    try
    {
        const std::string text = MLIPCore::read_model_text(path);
        if (buf && cap > 0)
        {
            const long n = std::min<long>(cap - 1, (long)text.size());
            std::memcpy(buf, text.data(), (size_t)n);
            buf[n] = 0;
        }
        return (long)text.size();
    }
    catch (const std::exception &ex)
    {
        g_error = ex.what();
        return -1;
    }
}

void ref_mlip_destroy(void *handle)
{
    if (handle)
        MLIPCore::destroy_mlip(static_cast<MLIPCore::mlip *>(handle));
}

// MLIPCore::compute over LAMMPS-style arrays.  x holds ntotal positions
// (local atoms first, then ghosts); centers are ilist[0..inum); neighbours of
// atom i are firstneigh_flat[firstneigh_off[i] .. + numneigh[i]).  Forces are
// accumulated into f[3*ntotal]; site_virial[6*ntotal] may be null.
int ref_mlip_compute(void *handle, int inum, const int *ilist, int ntotal, const int *type,
                     const double *x, const int *numneigh, const int *firstneigh_off,
                     const int *firstneigh_flat, double *energy, double *site_energy, double *f,
                     double *site_virial)
{
    try
    {
        auto *p = static_cast<MLIPCore::mlip *>(handle);
        std::vector<double *> xptr(ntotal), fptr(ntotal), vptr(ntotal);
        std::vector<int *> nptr(ntotal);
        std::vector<double> xcopy(x, x + 3 * static_cast<std::size_t>(ntotal));
        for (int i = 0; i < ntotal; ++i)
        {
            xptr[i] = xcopy.data() + 3 * i;
            fptr[i] = f + 3 * i;
            if (site_virial)
                vptr[i] = site_virial + 6 * i;
            nptr[i] = const_cast<int *>(firstneigh_flat) + firstneigh_off[i];
        }
        MLIPCore::mlip_buffers *buf = MLIPCore::create_mlip_buffer(p);
        double en = 0;
        MLIPCore::compute(p, buf, ilist, numneigh, inum, type, xptr.data(), nptr.data(), &en,
                          site_energy, site_virial ? vptr.data() : nullptr, fptr.data());
        MLIPCore::destroy_mlip_buffer(buf);
        *energy = en;
        return 0;
    }
    catch (const std::exception &ex)
    {
        g_error = ex.what();
        return -1;
    }
}

// MLIPCore::compute driven by OpenMP over centres: each thread owns one
// mlip_buffers workspace and private force / virial arrays (the thread-safety
// contract of the standalone core, runtime/mtp/cpu/mtp_cpu.h:38-40), merged
// serially afterwards as PotMTP::getEFSOMP does (potential_mtp.cpp:2476-2485).
int ref_mlip_compute_omp(void *handle, int threads, int inum, const int *ilist, int ntotal,
                         const int *type, const double *x, const int *numneigh,
                         const int *firstneigh_off, const int *firstneigh_flat, double *energy,
                         double *f)
{
    try
    {
        auto *p = static_cast<MLIPCore::mlip *>(handle);
        if (threads <= 0)
            threads = omp_get_max_threads();
        std::vector<double> xcopy(x, x + 3 * static_cast<std::size_t>(ntotal));
        std::vector<double *> xptr(ntotal);
        std::vector<int *> nptr(ntotal);
        for (int i = 0; i < ntotal; ++i)
        {
            xptr[i] = xcopy.data() + 3 * i;
            nptr[i] = const_cast<int *>(firstneigh_flat) + firstneigh_off[i];
        }
        std::vector<std::vector<double>> fbuf(threads);
        std::vector<double> ebuf(threads, 0.0);
        int failed = 0;
#pragma omp parallel num_threads(threads) reduction(| : failed)
        {
            const int t = omp_get_thread_num();
            const int nt = omp_get_num_threads();
            const int b = (int)((long)inum * t / nt), e = (int)((long)inum * (t + 1) / nt);
            try
            {
                fbuf[t].assign(3 * static_cast<std::size_t>(ntotal), 0.0);
                std::vector<double *> fptr(ntotal);
                for (int i = 0; i < ntotal; ++i)
                    fptr[i] = fbuf[t].data() + 3 * i;
                MLIPCore::mlip_buffers *buf = MLIPCore::create_mlip_buffer(p);
                double en = 0;
                MLIPCore::compute(p, buf, ilist + b, numneigh, e - b, type, xptr.data(),
                                  nptr.data(), &en, nullptr, nullptr, fptr.data());
                MLIPCore::destroy_mlip_buffer(buf);
                ebuf[t] = en;
            }
            catch (...)
            {
                failed |= 1;
            }
        }
        if (failed)
        {
            g_error = "MLIPCore::compute failed in a worker thread";
            return -1;
        }
        double en = 0;
        for (int t = 0; t < threads; ++t)
        {
            en += ebuf[t];
            if (fbuf[t].empty())
                continue;
            for (std::size_t k = 0; k < fbuf[t].size(); ++k)
                f[k] += fbuf[t][k];
        }
        *energy = en;
        return 0;
    }
    catch (const std::exception &ex)
    {
        g_error = ex.what();
        return -1;
    }
}

// MLIPCore::compute driven by OpenMP over centres for problems where every
// neighbour of every centre is its own ghost row (the explicit-image form the
// Python wrapper builds): each row of f, site_energy and site_virial is then
// written by the one thread that owns its centre, so all threads share the
// output arrays.  f[3*ntotal] and site_virial[6*ntotal] (may be null) are
// accumulated, site_energy[ntotal] (may be null) written for the centres; the
// energy is the sum of the per-thread energies in thread order.
int ref_mlip_efs_omp(void *handle, int threads, int inum, const int *ilist, int ntotal,
                     const int *type, const double *x, const int *numneigh,
                     const int *firstneigh_off, const int *firstneigh_flat, double *energy,
                     double *f, double *site_energy, double *site_virial)
{
    try
    {
        auto *p = static_cast<MLIPCore::mlip *>(handle);
        if (threads <= 0)
            threads = omp_get_max_threads();
        std::vector<double *> xptr(ntotal), fptr(ntotal), vptr(site_virial ? ntotal : 0);
        std::vector<int *> nptr(ntotal);
        for (int i = 0; i < ntotal; ++i)
        {
            xptr[i] = const_cast<double *>(x) + 3 * static_cast<std::size_t>(i);
            fptr[i] = f + 3 * static_cast<std::size_t>(i);
            if (site_virial)
                vptr[i] = site_virial + 6 * static_cast<std::size_t>(i);
            nptr[i] = const_cast<int *>(firstneigh_flat) + firstneigh_off[i];
        }
        std::vector<double> ebuf(threads, 0.0);
        int failed = 0;
#pragma omp parallel num_threads(threads) reduction(| : failed)
        {
            const int t = omp_get_thread_num();
            const int nt = omp_get_num_threads();
            const int b = (int)((long)inum * t / nt), e = (int)((long)inum * (t + 1) / nt);
            try
            {
                MLIPCore::mlip_buffers *buf = MLIPCore::create_mlip_buffer(p);
                double en = 0;
                MLIPCore::compute(p, buf, ilist + b, numneigh, e - b, type, xptr.data(),
                                  nptr.data(), &en, site_energy,
                                  site_virial ? vptr.data() : nullptr, fptr.data());
                MLIPCore::destroy_mlip_buffer(buf);
                ebuf[t] = en;
            }
            catch (...)
            {
                failed |= 1;
            }
        }
        if (failed)
        {
            g_error = "MLIPCore::compute failed in a worker thread";
            return -1;
        }
        double en = 0;
        for (int t = 0; t < threads; ++t)
            en += ebuf[t];
        *energy = en;
        return 0;
    }
    catch (const std::exception &ex)
    {
        g_error = ex.what();
        return -1;
    }
}

} // extern "C"
