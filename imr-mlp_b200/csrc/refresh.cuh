// refresh.cuh -- edge vectors of a stored neighbour list recomputed from
// moved positions, in the builder's own arithmetic (neighbors.cu): shared by
// the edge-parallel refresh kernel and the active-edge kernel (efs.cu), which
// refreshes the vectors of a list with a skin while it compacts its active
// edges.
#pragma once

#include "neighbors.hpp"

namespace mtpb {

// Image translation T = B * shift of a periodic structure, in Eigen's
// Matrix3d * Vector3d order: rows 0 and 1 (t0 + t1) + t2, row 2 t0 + (t1 + t2).
__device__ __forceinline__ void image_translation(const NbStruct &st, int s0, int s1, int s2,
                                                  double t[3])
{
    const int sh[3] = {s0, s1, s2};
    double img[3] = {0.0, 0.0, 0.0};
#pragma unroll
    for (int k = 0; k < 3; ++k)
        if (k < st.dims)
            img[k] = (double)sh[st.axes[k]];
#pragma unroll
    for (int r = 0; r < 2; ++r)
        t[r] = __dadd_rn(__dadd_rn(__dmul_rn(st.B[r][0], img[0]), __dmul_rn(st.B[r][1], img[1])),
                         __dmul_rn(st.B[r][2], img[2]));
    t[2] = __dadd_rn(__dmul_rn(st.B[2][0], img[0]),
                     __dadd_rn(__dmul_rn(st.B[2][1], img[1]), __dmul_rn(st.B[2][2], img[2])));
}

// r = x_o + T(shift) - x_i for centre i and neighbour o, with the positions
// as [atom][4] rows (x, y, z, 0) and the shift packed as three biased bytes;
// the builder's operation order, including its i > o form
// -(x_i - T - x_o), so that a refreshed list equals a rebuilt one bit for bit.
__device__ __forceinline__ void refresh_vector(const NbStruct &st, int i, int o, int code,
                                               const double *p, double &x, double &y, double &z)
{
    const double2 *P = reinterpret_cast<const double2 *>(p);
    const double2 i01 = P[2 * (size_t)i], i2 = P[2 * (size_t)i + 1];
    const double2 o01 = P[2 * (size_t)o], o2 = P[2 * (size_t)o + 1];
    const double pi[3] = {i01.x, i01.y, i2.x}, po[3] = {o01.x, o01.y, o2.x};
    const int s0 = (code & 0xff) - 128, s1 = ((code >> 8) & 0xff) - 128,
              s2 = ((code >> 16) & 0xff) - 128;
    const bool zero = (s0 == 0 && s1 == 0 && s2 == 0);
    double t[3] = {0.0, 0.0, 0.0};
    if (!zero)
        image_translation(st, s0, s1, s2, t);
    if (i <= o) {
        x = __dsub_rn(zero ? po[0] : __dadd_rn(po[0], t[0]), pi[0]);
        y = __dsub_rn(zero ? po[1] : __dadd_rn(po[1], t[1]), pi[1]);
        z = __dsub_rn(zero ? po[2] : __dadd_rn(po[2], t[2]), pi[2]);
    } else {
        x = -__dsub_rn(zero ? pi[0] : __dadd_rn(pi[0], -t[0]), po[0]);
        y = -__dsub_rn(zero ? pi[1] : __dadd_rn(pi[1], -t[1]), po[1]);
        z = -__dsub_rn(zero ? pi[2] : __dadd_rn(pi[2], -t[2]), po[2]);
    }
}

} // namespace mtpb
