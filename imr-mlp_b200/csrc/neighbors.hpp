// neighbors.hpp -- device arena and the neighbour-builder interface.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <map>
#include <string>

namespace mtpb {

// Grow-only named device buffers owned by one context.  get() returns a
// buffer of at least the requested size; contents are not preserved when it
// grows.  All buffers live on the context's device.
class DeviceArena {
  public:
    ~DeviceArena() { release(); }
    void *get(const std::string &name, size_t bytes)
    {
        auto it = bufs_.find(name);
        if (it != bufs_.end() && it->second.bytes >= bytes)
            return it->second.ptr;
        if (it != bufs_.end()) {
            cudaFree(it->second.ptr);
            bytes_total_ -= it->second.bytes;
            bufs_.erase(it);
        }
        size_t want = bytes < 256 ? 256 : bytes;
        // headroom for slowly growing batches
        want += want / 8;
        void *p = nullptr;
        if (cudaMalloc(&p, want) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        bufs_[name] = {p, want};
        bytes_total_ += want;
        return p;
    }
    template <class T> T *get(const std::string &name, size_t count)
    {
        return static_cast<T *>(get(name, count * sizeof(T)));
    }
    void release()
    {
        for (auto &kv : bufs_)
            cudaFree(kv.second.ptr);
        bufs_.clear();
        bytes_total_ = 0;
    }
    size_t bytes() const { return bytes_total_; }

  private:
    struct Buf {
        void *ptr;
        size_t bytes;
    };
    std::map<std::string, Buf> bufs_;
    size_t bytes_total_ = 0;
};

// Host-prepared description of one periodic structure for the builder.
struct NbStruct {
    double cell[9];   // rows are lattice vectors
    double inv[9];    // Eigen-order inverse of cell
    double B[3][3];   // image basis: B[r][k] = cell(axes[k], r)
    int axes[3];
    int dims;
    int ncell[3];     // cells per lattice direction
    int stencil[3];   // +- cells searched per direction
    int cell0;        // first global cell index
    double cutsq;
};

struct NbBuildInput {
    int nstruct = 0;
    int natoms = 0;
    int ncenter = -1;   // centres are atoms [0, ncenter); -1: all atoms
    int total_cells = 0;
    const int *atom_offsets = nullptr;  // device [nstruct+1]
    const NbStruct *structs = nullptr;  // device [nstruct]
    const double *positions = nullptr;  // device [natoms*3]
    const int *types = nullptr;         // device [natoms]; checked against 0..K-1 when set
    int K = 0;
};

struct NbResult {
    long nedges = 0;
    int bad_type = -1;   // first atom whose species is outside 0..K-1, or -1
    const double *wx = nullptr, *wy = nullptr, *wz = nullptr;
    const int *offsets = nullptr;
    const int *nbr = nullptr;
    const int *shift = nullptr;
    const double *rx = nullptr, *ry = nullptr, *rz = nullptr;
    const int *in_offsets = nullptr;
    const int *in_edges = nullptr;
    const int *struct_of = nullptr;   // [natoms]
    const int *center = nullptr;      // [nedges] centre of every edge
    const int *pair = nullptr;        // [nedges] species pair it*K+jt, -1 for type -1
};

cudaError_t build_neighbors(const NbBuildInput &in, DeviceArena &arena, NbResult &res,
                            cudaStream_t s);
cudaError_t build_in_edges(int ntotal, long nedges, const int *nbr, DeviceArena &arena,
                           NbResult &res, cudaStream_t s);
// unwrapped: scratch of 4 * natoms doubles (per-atom positions relative to the
// build's images)
cudaError_t refresh_edges(int natoms, const NbStruct *structs, const int *struct_of,
                          const NbResult &nb, const double *x_build, const double *x,
                          double *unwrapped, double *rx, double *ry, double *rz, cudaStream_t s);
// the first half of refresh_edges: only the unwrapped positions (the edge
// vectors are then recomputed by the active-edge pass, refresh.cuh)
cudaError_t unwrap_positions(int natoms, const NbResult &nb, const double *x_build,
                             const double *x, double *unwrapped, cudaStream_t s);
cudaError_t edge_vectors(int ncenter, const int *offsets, const int *nbr, const double *x,
                         double *rx, double *ry, double *rz, cudaStream_t s);
cudaError_t edge_pairs(long nedges, const int *center, const int *nbr, const int *types, int K,
                       int *pair, cudaStream_t s);
cudaError_t exclusive_scan(const int *in, int *out, int n, DeviceArena &arena, cudaStream_t s);

// Host helper: fills the NbStruct of a periodic cell (Eigen-order inverse,
// sorted image basis, cell grid, stencil).  Returns false for unsupported
// cells (singular, or not fully periodic).
bool prepare_struct(const double *cell, const int *pbc, double cutoff, NbStruct &out,
                    std::string *error);

} // namespace mtpb
