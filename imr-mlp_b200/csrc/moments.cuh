// moments.cuh -- constants and helpers shared by the moment kernels of the
// energy/force path (efs.cu) and of the training path (grad.cu): staging
// geometry, warps per basis shape, and the accumulator layout of a chain.
#pragma once

#include "shapes.cuh"

namespace mtpb {

constexpr int KS = 8;     // edge slots staged per chunk
constexpr int STR = 36;   // row stride of the staging arrays (doubles): conflict-free
                          // writes from (lane, slot) pairs and reads by lane

// Warps per block of the moment kernels.  Blocks run 4 warps and two or
// three blocks share an SM: the warps that share a scheduler then run the
// same unrolled chain code (8 or 12 different bodies per SM thrashed the
// instruction cache).
template <class S> struct ShapeCfg;
template <> struct ShapeCfg<ShapeS1> { static constexpr int NW = 2, NPART = 1, NPART_REV = 1, SUB = 1, SUB_REV = 1; };
template <> struct ShapeCfg<ShapeS2> { static constexpr int NW = 2, NPART = 1, NPART_REV = 1, SUB = 1, SUB_REV = 1; };
template <> struct ShapeCfg<ShapeL16> { static constexpr int NW = 4, NPART = 1, NPART_REV = 1, SUB = 1, SUB_REV = 1; };
// level 20: one launch each way (a reverse split over 8 warps in two launches
// measured slower: 15.3 ms against 14.2 ms on the 1M-atom box); the reverse
// chains are partitioned 16 ways and every warp runs four members in turn
// (reverse 14.4 -> 10.2 ms; 2 / 3 / 5 / 6 / 8 members: 12.0 / 10.2 / 11.4 /
// 12.5 / 12.1 ms; more than one member per warp in the forward kernel was
// slower)
template <> struct ShapeCfg<ShapeL20> { static constexpr int NW = 4, NPART = 1, NPART_REV = 1, SUB = 1, SUB_REV = 4; };
// level 24: the chains are partitioned over 12 warps (register budget) and
// run as three launches ("parts") of 4 warps, three blocks per SM, so that
// every scheduler still runs a single unrolled body; the reverse partition
// has 24 members, two per warp
template <> struct ShapeCfg<ShapeL24> { static constexpr int NW = 4, NPART = 3, NPART_REV = 3, SUB = 1, SUB_REV = 2; };
template <> struct ShapeCfg<ShapePS> { static constexpr int NW = 4, NPART = 1, NPART_REV = 1, SUB = 1, SUB_REV = 1; };

// launches ("parts"), partition members per warp and blocks per SM of the
// forward (REV false) and reverse kernels
template <class S, bool REV> struct KCfg {
    static constexpr int NW = ShapeCfg<S>::NW;
    static constexpr int NPART = REV ? ShapeCfg<S>::NPART_REV : ShapeCfg<S>::NPART;
    static constexpr int SUB = REV ? ShapeCfg<S>::SUB_REV : ShapeCfg<S>::SUB;   // members per warp
    static constexpr int BLOCKS = NW > 4 ? 1 : NPART > 1 ? 3 : 2;
};

__device__ __forceinline__ double &SV(double *st, int row, int k, int lane)
{
    return st[(row * KS + k) * STR + lane];
}

// Partition members of warp W0 when NW members are shared by NW / SUB warps:
// W0, W0 + NW / SUB, ... (strided, which balances the warps' register counts
// better than consecutive members).  Accumulator base of the warp's s-th
// member in its register array; s = SUB gives the array's size.
template <class S, int NW, int W0, int SUB> constexpr int sub_base(int s)
{
    int b = 0;
    for (int i = 0; i < s; ++i)
        b += Partition<S, NW>::table.nacc[i * (NW / SUB) + W0];
    return b;
}

// accumulator offset of monomial a within a chain (sum of channel counts of
// the lower powers)
template <class S> constexpr int chain_acc_off(int s, int a)
{
    int o = 0;
    for (int aa = 0; aa < a; ++aa)
        o += S::cnt(aa + s);
    return o;
}

} // namespace mtpb
