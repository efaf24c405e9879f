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

#include <cstring>
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

} // extern "C"
