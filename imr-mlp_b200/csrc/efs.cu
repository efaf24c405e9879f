// efs.cu -- FP64 moment kernels (forward and reverse), the per-atom moment
// graph kernel, the deterministic force gather and the energy/virial
// reductions of the MTP energy/force/stress path.
//
// Reference semantics (paths relative to the reference project):
//   forward   potentials/potential_mtp.cpp:2813-2925  (CalcSiteDescriptorsImpl)
//   energy    potentials/potential_mtp.cpp:2959-2984  (CalcSiteEFS)
//   reverse   potentials/potential_mtp.cpp:3292-3305, 2938-2957
//   scatter   potentials/potential_mtp.cpp:1909-1932  (getEFS)
//   radial    basis/basis.cpp:148-164                 (RBasis_Chebyshev::calc_der)
//
// The kernels use a factorised form of the same mathematics.  With
// rhat = r/|r| and f_mu the radial functions, every basic moment is
//   b[mu,abc] = sum_j f_mu(r_j) xhat^a yhat^b zhat^c.
// The force on edge j needs d_j = dE/dr_j = sum a[mu,abc] grad(f_mu u_abc):
//   d_j = rhat (V - H/r) + G/r,  with P_abc = sum_mu a f_mu,
//   P'_abc = sum_mu a f'_mu, V = sum P' u, H = sum nu P u, G = sum P grad u,
// each polynomial evaluated along x-chains with Horner's rule.  This replaces
// the reference's per-edge Jacobian (nb x n_e x 3 doubles per site) by
// registers.
#include "radial.cuh"
#include "internal.hpp"
#include "moments.cuh"
#include "dag.cuh"
#include "refresh.cuh"

#include <algorithm>
#include <cstdio>

namespace mtpb {

// staging arrays: 0 xhat, 1 yhat, 2 zhat, 3 1/r, 4.. f_mu, 4+NMU.. f'_mu
template <class S, bool REV> constexpr int stage_rows()
{
    return REV ? 4 + 2 * S::NMU : 4 + S::NMU;
}

template <class S, bool REV> constexpr int smem_doubles(int K, int R)
{
    constexpr int NW = ShapeCfg<S>::NW;
    int n = stage_rows<S, REV>() * KS * STR;
    if (REV)
        n += NW * 3 * KS * 32;
    n += PAIR_PARAM_DOUBLES * K * K;   // pair parameters
    n += K * K * S::NMU * R;    // radial coefficients of the used channels
    return n;
}

// Edge slot `slot` of centre `atom` in the staged arrays (the compacted
// active edges under ACT, else the list itself); false past the centre's
// (active) edges.  ACT is a compile-time choice so that each moment kernel
// carries one path only (the reverse kernel runs at the limit of the
// instruction cache).
template <bool ACT>
__device__ __forceinline__ bool slot_edge(const EdgeArgs &p, int atom, int slot, int &e)
{
    const int b = __ldg(p.offsets + atom);
    e = b + slot;
    if constexpr (ACT)
        return slot < __ldg(p.nact + atom);
    else
        return e < __ldg(p.offsets + atom + 1);
}

// List index of staged edge slot e (where its derivatives are stored)
template <bool ACT> __device__ __forceinline__ int list_edge(const EdgeArgs &p, int e)
{
    if constexpr (ACT)
        return __ldg(p.active + e);
    else
        return e;
}

struct StageView {
    double *st;       // [rows][KS][STR]
    double *part;     // [NW][3][KS][32] (reverse only)
    const PairParams *pairs;
    const double *radial;  // [K*K][NMU][R]
};

// Computes the per-edge quantities of one chunk of edge slots for the 32
// atoms of this block.  Every thread of the block takes part.
// RG: the model has radial families other than RBChebyshev (radial.cuh);
// the RBChebyshev-only kernels carry none of their code.
template <class S, int NW, bool REV, bool RG, bool ACT>
__device__ __forceinline__ void stage_chunk(const EdgeArgs &p, const StageView &v, int atom0,
                                            int chunk)
{
    constexpr int NMU = S::NMU;
    for (int item = threadIdx.x; item < 32 * KS; item += blockDim.x) {
        const int lane = item / KS;
        const int k = item - lane * KS;
        const int atom = atom0 + lane;
        double xh = 0.0, yh = 0.0, zh = 0.0, rinv = 0.0;
        double f[NMU], fp[NMU];
#pragma unroll
        for (int m = 0; m < NMU; ++m) {
            f[m] = 0.0;
            fp[m] = 0.0;
        }
        bool have = false;
        double x = 0.0, y = 0.0, z = 0.0;
        int pair = -1;
        int e = 0;
        if (atom < p.natoms) {
            if (slot_edge<ACT>(p, atom, chunk * KS + k, e)) {
                have = true;
                x = __ldg(p.rx + e);
                y = __ldg(p.ry + e);
                z = __ldg(p.rz + e);
                // the reverse staging keeps the type lookups: with the pair
                // array it measured slower (14.2 -> 14.75 ms, 1M atoms)
                if (!REV && p.pair) {
                    pair = __ldg(p.pair + e);
                } else {
                    const int it = __ldg(p.types + atom);
                    const int jt = __ldg(p.types + __ldg(p.nbr + e));
                    pair = (it >= 0 && jt >= 0) ? it * p.K + jt : -1;
                }
            }
        }
        {
            if (have) {
                // neighbour distance exactly as the reference list stores it:
                // sqrt((x*x + y*y) + z*z) without contraction
                const double r2 = __dadd_rn(__dadd_rn(__dmul_rn(x, x), __dmul_rn(y, y)),
                                            __dmul_rn(z, z));
                const double r = sqrt(r2);
                // atoms of type -1 are skipped (runtime/mtp/mlip.cpp:944, 952)
                const PairParams &pp = v.pairs[pair >= 0 ? pair : 0];
                // potential_mtp.cpp:2842 skips r > cutoff; mlip.cpp:966 r > 0
                if (pair >= 0 && r > 0.0 && r <= pp.rmax) {
                    rinv = 1.0 / r;
                    xh = x * rinv;
                    yh = y * rinv;
                    zh = z * rinv;
                    // radial basis of the pair's family (radial.cuh) folded
                    // into the channel sums f_mu = sum_xi c[pair,mu,xi] Q_xi(r)
                    const double *c = v.radial + pair * NMU * p.R;
                    auto emit = [&](int xi, double q, double d) {
#pragma unroll
                        for (int m = 0; m < NMU; ++m) {
                            f[m] = fma(c[m * p.R + xi], q, f[m]);
                            fp[m] = fma(c[m * p.R + xi], d, fp[m]);
                        }
                    };
                    if constexpr (RG)
                        radial_basis(pp, p.scaling, p.R, r, emit);
                    else
                        radial_chebyshev(pp, p.scaling, p.R, r, emit);
                }
            }
        }
        SV(v.st, 0, k, lane) = xh;
        SV(v.st, 1, k, lane) = yh;
        SV(v.st, 2, k, lane) = zh;
#pragma unroll
        for (int m = 0; m < NMU; ++m)
            SV(v.st, 4 + m, k, lane) = f[m];
        if constexpr (REV) {
            SV(v.st, 3, k, lane) = rinv;
#pragma unroll
            for (int m = 0; m < NMU; ++m)
                SV(v.st, 4 + NMU + m, k, lane) = fp[m];
        }
    }
}

// ----------------------------------------------------------------------------
// Forward: basic moments of 32 atoms (lane = atom).  NW is the size of the
// chain partition; the warp runs its SUB members (sub_base) one after the
// other over each chunk's edges (one pass per member keeps the
// unrolled per-edge code small).
// ----------------------------------------------------------------------------
template <class S, int NW, int W0, int SUB, bool RG, bool ACT>
__device__ __forceinline__ void fwd_warp(const EdgeArgs &p, const StageView &v, int atom0,
                                         int maxdeg, double *basic)
{
    using P = Partition<S, NW>;
    constexpr int NACC = sub_base<S, NW, W0, SUB>(SUB);
    constexpr int NMU = S::NMU;
    const int lane = threadIdx.x & 31;
    double acc[NACC > 0 ? NACC : 1];
#pragma unroll
    for (int i = 0; i < NACC; ++i)
        acc[i] = 0.0;
    const int nchunks = (maxdeg + KS - 1) / KS;
    for (int ch = 0; ch < nchunks; ++ch) {
        stage_chunk<S, NW / SUB, false, RG, ACT>(p, v, atom0, ch);
        __syncthreads();
        const int kend = min(KS, maxdeg - ch * KS);
        static_for<SUB>([&](auto is) {
            constexpr int W = decltype(is)::value * (NW / SUB) + W0;
            constexpr int BASE = sub_base<S, NW, W0, SUB>(decltype(is)::value);
            constexpr int NCHW = P::table.count[W];
            constexpr int MAXB = P::table.maxb[W];
            constexpr int MAXC = P::table.maxc[W];
            for (int k = 0; k < kend; ++k) {
                const double xh = SV(v.st, 0, k, lane);
                const double yh = SV(v.st, 1, k, lane);
                const double zh = SV(v.st, 2, k, lane);
                double f[NMU];
#pragma unroll
                for (int m = 0; m < NMU; ++m)
                    f[m] = SV(v.st, 4 + m, k, lane);
                double yp[MAXB + 1], zp[MAXC + 1];
                yp[0] = 1.0;
                zp[0] = 1.0;
#pragma unroll
                for (int i = 1; i <= MAXB; ++i)
                    yp[i] = yp[i - 1] * yh;
#pragma unroll
                for (int i = 1; i <= MAXC; ++i)
                    zp[i] = zp[i - 1] * zh;
                static_for<NCHW>([&](auto ii) {
                    constexpr int ci = P::table.list[W * S::NCH + decltype(ii)::value];
                    constexpr int a0 = BASE + P::table.acc0[W * S::NCH + decltype(ii)::value];
                    constexpr int b = S::chains.b[ci];
                    constexpr int c = S::chains.c[ci];
                    constexpr int L = S::chains.len[ci];
                    double u;
                    if constexpr (b == 0 && c == 0)
                        u = 1.0;
                    else if constexpr (b == 0)
                        u = zp[c];
                    else if constexpr (c == 0)
                        u = yp[b];
                    else
                        u = yp[b] * zp[c];
                    static_for<L>([&](auto ia) {
                        constexpr int a = decltype(ia)::value;
                        constexpr int nu = a + b + c;
                        constexpr int off = a0 + chain_acc_off<S>(b + c, a);
                        static_for<S::cnt(nu)>([&](auto iq) {
                            constexpr int q = decltype(iq)::value;
                            acc[off + q] = fma(f[S::chan(nu, q)], u, acc[off + q]);
                        });
                        if constexpr (a + 1 < L)
                            u *= xh;
                    });
                });
            }
        });
        __syncthreads();
    }
    const int atom = atom0 + lane;
    if (atom < p.natoms) {
        static_for<SUB>([&](auto is) {
            constexpr int W = decltype(is)::value * (NW / SUB) + W0;
            constexpr int BASE = sub_base<S, NW, W0, SUB>(decltype(is)::value);
            static_for<P::table.count[W]>([&](auto ii) {
                constexpr int ci = P::table.list[W * S::NCH + decltype(ii)::value];
                constexpr int a0 = BASE + P::table.acc0[W * S::NCH + decltype(ii)::value];
                constexpr int n = S::chains.nacc[ci];
                constexpr int slot0 = S::chains.slot0[ci];
#pragma unroll
                for (int i = 0; i < n; ++i)
                    basic[(size_t)(slot0 + i) * p.npad + atom] = acc[a0 + i];
            });
        });
    }
}

// One staged edge's share of the chains of partition member W (adjoints at
// adj[BASE..]): the partial dE/dr_j of the file header's formula.
template <class S, int NW, int W, int BASE, int NA>
__device__ __forceinline__ void rev_edge(const StageView &v, int k, int lane,
                                         const double (&adj)[NA], double &ox, double &oy,
                                         double &oz)
{
    using P = Partition<S, NW>;
    constexpr int NCHW = P::table.count[W];
    constexpr int MAXB = P::table.maxb[W];
    constexpr int MAXC = P::table.maxc[W];
    constexpr int NMU = S::NMU;
    const double xh = SV(v.st, 0, k, lane);
    const double yh = SV(v.st, 1, k, lane);
    const double zh = SV(v.st, 2, k, lane);
    const double rinv = SV(v.st, 3, k, lane);
    double f[NMU], fp[NMU];
#pragma unroll
    for (int m = 0; m < NMU; ++m) {
        f[m] = SV(v.st, 4 + m, k, lane);
        fp[m] = SV(v.st, 4 + NMU + m, k, lane);
    }
    double yp[MAXB + 1], zp[MAXC + 1];
    yp[0] = 1.0;
    zp[0] = 1.0;
#pragma unroll
    for (int i = 1; i <= MAXB; ++i)
        yp[i] = yp[i - 1] * yh;
#pragma unroll
    for (int i = 1; i <= MAXC; ++i)
        zp[i] = zp[i - 1] * zh;
    double V = 0.0, H = 0.0, Gx = 0.0, Gy = 0.0, Gz = 0.0;
    static_for<NCHW>([&](auto ii) {
        constexpr int ci = P::table.list[W * S::NCH + decltype(ii)::value];
        constexpr int a0 = BASE + P::table.acc0[W * S::NCH + decltype(ii)::value];
        constexpr int b = S::chains.b[ci];
        constexpr int c = S::chains.c[ci];
        constexpr int L = S::chains.len[ci];
        double h0 = 0.0, h1 = 0.0, g0 = 0.0;
        static_for<L>([&](auto ia) {
            constexpr int a = L - 1 - decltype(ia)::value;
            constexpr int nu = a + b + c;
            constexpr int off = a0 + chain_acc_off<S>(b + c, a);
            double Pv = adj[off] * f[S::chan(nu, 0)];
            double Pd = adj[off] * fp[S::chan(nu, 0)];
            static_for<S::cnt(nu) - 1>([&](auto iq) {
                constexpr int q = decltype(iq)::value + 1;
                Pv = fma(adj[off + q], f[S::chan(nu, q)], Pv);
                Pd = fma(adj[off + q], fp[S::chan(nu, q)], Pd);
            });
            if constexpr (a == L - 1) {
                h0 = Pv;
                g0 = Pd;
            } else {
                h1 = fma(h1, xh, h0);
                h0 = fma(h0, xh, Pv);
                g0 = fma(g0, xh, Pd);
            }
        });
        double q;
        if constexpr (b == 0 && c == 0)
            q = 1.0;
        else if constexpr (b == 0)
            q = zp[c];
        else if constexpr (c == 0)
            q = yp[b];
        else
            q = yp[b] * zp[c];
        V = fma(q, g0, V);
        Gx = fma(q, h1, Gx);
        if constexpr (b > 0) {
            double qy = (c == 0) ? yp[b - 1] : yp[b - 1] * zp[c];
            Gy = fma(double(b) * qy, h0, Gy);
        }
        if constexpr (c > 0) {
            double qz = (b == 0) ? zp[c - 1] : yp[b] * zp[c - 1];
            Gz = fma(double(c) * qz, h0, Gz);
        }
        H = fma(q, fma(xh, h1, double(b + c) * h0), H);
    });
    const double t = V - H * rinv;
    ox = fma(xh, t, Gx * rinv);
    oy = fma(yh, t, Gy * rinv);
    oz = fma(zh, t, Gz * rinv);
}

// ----------------------------------------------------------------------------
// Reverse: per-edge dE_i/dr_ij of 32 atoms.  Each warp adds its chains'
// share; the shares are summed in fixed warp order (deterministic).  NW is
// the size of the chain partition; the warp runs its SUB members (sub_base)
// one after the other over each chunk's edges (one pass
// per member, so that the unrolled code run per edge stays small: a long
// per-edge body stalls on instruction fetch), adding their shares in member
// order.  NWB is the warps of this block; the first part stores the sums,
// later parts add to them.
// ----------------------------------------------------------------------------
template <class S, int NW, int W0, int SUB, int NWB, bool FIRST, bool RG, bool ACT>
__device__ __forceinline__ void rev_warp(const EdgeArgs &p, const StageView &v, int atom0,
                                         int maxdeg, const double *adjoint, double *dx,
                                         double *dy, double *dz)
{
    using P = Partition<S, NW>;
    constexpr int NACC = sub_base<S, NW, W0, SUB>(SUB);
    const int lane = threadIdx.x & 31;
    const int atom = atom0 + lane;
    double adj[NACC > 0 ? NACC : 1];
    if (atom < p.natoms) {
        static_for<SUB>([&](auto is) {
            constexpr int W = decltype(is)::value * (NW / SUB) + W0;
            constexpr int BASE = sub_base<S, NW, W0, SUB>(decltype(is)::value);
            static_for<P::table.count[W]>([&](auto ii) {
                constexpr int ci = P::table.list[W * S::NCH + decltype(ii)::value];
                constexpr int a0 = BASE + P::table.acc0[W * S::NCH + decltype(ii)::value];
                constexpr int n = S::chains.nacc[ci];
                constexpr int slot0 = S::chains.slot0[ci];
#pragma unroll
                for (int i = 0; i < n; ++i)
                    adj[a0 + i] = __ldg(adjoint + (size_t)(slot0 + i) * p.npad + atom);
            });
        });
    } else {
#pragma unroll
        for (int i = 0; i < NACC; ++i)
            adj[i] = 0.0;
    }
    const int nchunks = (maxdeg + KS - 1) / KS;
    double *part = v.part + (size_t)(W0 % NWB) * 3 * KS * 32;
    for (int ch = 0; ch < nchunks; ++ch) {
        stage_chunk<S, NW / SUB, true, RG, ACT>(p, v, atom0, ch);
        __syncthreads();
        const int kend = min(KS, maxdeg - ch * KS);
        static_for<SUB>([&](auto is) {
            constexpr int s = decltype(is)::value;
            constexpr int W = s * (NW / SUB) + W0;
            constexpr int BASE = sub_base<S, NW, W0, SUB>(s);
            for (int k = 0; k < kend; ++k) {
                double ox, oy, oz;
                rev_edge<S, NW, W, BASE>(v, k, lane, adj, ox, oy, oz);
                double *px = part + (0 * KS + k) * 32 + lane;
                double *py = part + (1 * KS + k) * 32 + lane;
                double *pz = part + (2 * KS + k) * 32 + lane;
                if constexpr (s == 0) {
                    *px = ox;
                    *py = oy;
                    *pz = oz;
                } else {
                    *px += ox;
                    *py += oy;
                    *pz += oz;
                }
            }
        });
        __syncthreads();
        // sum the warps' shares in warp order and store per edge (thread ->
        // (slot, lane) so that the shared reads are lane-contiguous)
        for (int item = threadIdx.x; item < 32 * KS; item += NWB * 32) {
            const int k = item >> 5;
            const int ln = item & 31;
            const int at = atom0 + ln;
            if (k >= kend || at >= p.natoms)
                continue;
            int e;
            if (!slot_edge<ACT>(p, at, ch * KS + k, e))
                continue;
            e = list_edge<ACT>(p, e);
            double sx = 0.0, sy = 0.0, sz = 0.0;
#pragma unroll
            for (int w = 0; w < NWB; ++w) {
                const double *pw = v.part + (size_t)w * 3 * KS * 32;
                sx += pw[(0 * KS + k) * 32 + ln];
                sy += pw[(1 * KS + k) * 32 + ln];
                sz += pw[(2 * KS + k) * 32 + ln];
            }
            if constexpr (FIRST) {
                dx[e] = sx;
                dy[e] = sy;
                dz[e] = sz;
            } else {
                dx[e] += sx;
                dy[e] += sy;
                dz[e] += sz;
            }
        }
        __syncthreads();
    }
}

// PART: which block of NW warps of the NW * NPART chain partition this launch
// runs
template <class S, bool REV, int PART, bool RG, bool ACT>
__global__ void __launch_bounds__(ShapeCfg<S>::NW * 32, KCfg<S, REV>::BLOCKS)
    k_moments(EdgeArgs p, double *basic, const double *adjoint, double *dx, double *dy,
              double *dz)
{
    constexpr int NW = ShapeCfg<S>::NW;
    constexpr int NMU = S::NMU;
    extern __shared__ double smem[];
    StageView v;
    v.st = smem;
    double *cur = smem + stage_rows<S, REV>() * KS * STR;
    v.part = cur;
    if (REV)
        cur += NW * 3 * KS * 32;
    PairParams *pairs = reinterpret_cast<PairParams *>(cur);
    cur += PAIR_PARAM_DOUBLES * p.K * p.K;
    double *radial = cur;
    const int KK = p.K * p.K;
    for (int i = threadIdx.x; i < KK; i += blockDim.x)
        pairs[i] = p.pairs[i];
    for (int i = threadIdx.x; i < KK * NMU * p.R; i += blockDim.x) {
        const int pair = i / (NMU * p.R);
        const int rem = i - pair * NMU * p.R;
        radial[i] = p.radial[(size_t)pair * p.mu_total * p.R + rem];
    }
    v.pairs = pairs;
    v.radial = radial;
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    constexpr int NWT = NW * KCfg<S, REV>::NPART;
    constexpr int SUB = KCfg<S, REV>::SUB;
    auto run_group = [&](int group) {
        const int atom0 = group * 32;
        const int maxdeg = __ldg(p.group_maxdeg + group);
        static_for<NW>([&](auto iw) {
            constexpr int WL = decltype(iw)::value;
            constexpr int W = PART * NW + WL;
            if (warp == WL) {
                if constexpr (REV)
                    rev_warp<S, NWT * SUB, W, SUB, NW, PART == 0, RG, ACT>(p, v, atom0, maxdeg,
                                                                      adjoint, dx, dy, dz);
                else
                    fwd_warp<S, NWT * SUB, W, SUB, RG, ACT>(p, v, atom0, maxdeg, basic);
            }
        });
    };
    // a forward kernel launched in one part runs persistent blocks, each
    // taking groups of 32 centres in turn (the chunk loops end on a barrier,
    // so the staging is free between groups); the reverse kernel and the
    // multi-part forward kernels run one block per group (the reverse kernel's
    // code as it was: it runs at the limit of the instruction cache)
    constexpr bool PERSIST = !REV && KCfg<S, REV>::NPART == 1;
    if constexpr (!PERSIST) {
        run_group(blockIdx.x);
    } else {
        const int ngroups = (p.natoms + 31) / 32;
        for (int group = blockIdx.x; group < ngroups; group += gridDim.x)
            run_group(group);
    }
}

template <class S, bool REV> static cudaError_t launch_shape(const EdgeArgs &a, double *basic,
                                                             const double *adjoint, double *dx,
                                                             double *dy, double *dz,
                                                             cudaStream_t s)
{
    constexpr int NW = ShapeCfg<S>::NW;
    const int groups = (a.natoms + 31) / 32;
    if (groups == 0)
        return cudaSuccess;
    const size_t smem = sizeof(double) * smem_doubles<S, REV>(a.K, a.R);
    cudaError_t err = cudaSuccess;
    static_for<KCfg<S, REV>::NPART>([&](auto ip) {
        constexpr int P = decltype(ip)::value;
        if (err != cudaSuccess)
            return;
        auto kern = a.rb_generic ? (a.active ? k_moments<S, REV, P, true, true>
                                             : k_moments<S, REV, P, true, false>)
                                 : (a.active ? k_moments<S, REV, P, false, true>
                                             : k_moments<S, REV, P, false, false>);
        err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        // persistent blocks for a one-part forward kernel (level 20: 4.15 ->
        // 4.03 ms at 1M atoms); the reverse kernel balances better with one
        // block per group (11.0 ms against 12.1 ms persistent), and so do the
        // multi-part level-24 forward kernels (9.3 ms against 9.8 ms)
        constexpr bool persist = !REV && KCfg<S, REV>::NPART == 1;
        int per = 1, dev = 0, sms = 1;
        if (err == cudaSuccess && persist)
            err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, NW * 32, smem);
        if (err == cudaSuccess && persist)
            err = cudaGetDevice(&dev);
        if (err == cudaSuccess && persist)
            err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (err == cudaSuccess) {
            const int blocks = persist ? std::min(groups, sms * std::max(per, 1)) : groups;
            kern<<<blocks, NW * 32, smem, s>>>(a, basic, adjoint, dx, dy, dz);
            err = cudaGetLastError();
        }
    });
    return err;
}

template <bool REV> static cudaError_t dispatch(int shape, const EdgeArgs &a, double *basic,
                                                const double *adjoint, double *dx, double *dy,
                                                double *dz, cudaStream_t s)
{
    switch (shape) {
    case SHAPE_S1: return launch_shape<ShapeS1, REV>(a, basic, adjoint, dx, dy, dz, s);
    case SHAPE_S2: return launch_shape<ShapeS2, REV>(a, basic, adjoint, dx, dy, dz, s);
    case SHAPE_L16: return launch_shape<ShapeL16, REV>(a, basic, adjoint, dx, dy, dz, s);
    case SHAPE_L20: return launch_shape<ShapeL20, REV>(a, basic, adjoint, dx, dy, dz, s);
    case SHAPE_L24: return launch_shape<ShapeL24, REV>(a, basic, adjoint, dx, dy, dz, s);
    case SHAPE_PS: return launch_shape<ShapePS, REV>(a, basic, adjoint, dx, dy, dz, s);
    default: return cudaErrorInvalidValue;
    }
}

// launches issued by one launch_moments_fwd / launch_moments_rev call
int moment_kernel_parts(int shape, bool rev)
{
    switch (shape) {
    case SHAPE_S1: return rev ? KCfg<ShapeS1, true>::NPART : KCfg<ShapeS1, false>::NPART;
    case SHAPE_S2: return rev ? KCfg<ShapeS2, true>::NPART : KCfg<ShapeS2, false>::NPART;
    case SHAPE_L16: return rev ? KCfg<ShapeL16, true>::NPART : KCfg<ShapeL16, false>::NPART;
    case SHAPE_L20: return rev ? KCfg<ShapeL20, true>::NPART : KCfg<ShapeL20, false>::NPART;
    case SHAPE_L24: return rev ? KCfg<ShapeL24, true>::NPART : KCfg<ShapeL24, false>::NPART;
    case SHAPE_PS: return rev ? KCfg<ShapePS, true>::NPART : KCfg<ShapePS, false>::NPART;
    default: return 1;
    }
}

cudaError_t launch_moments_fwd(int shape, const EdgeArgs &a, double *basic, cudaStream_t s)
{
    return dispatch<false>(shape, a, basic, nullptr, nullptr, nullptr, nullptr, s);
}

cudaError_t launch_moments_rev(int shape, const EdgeArgs &a, const double *adjoint, double *dx,
                               double *dy, double *dz, cudaStream_t s)
{
    return dispatch<true>(shape, a, nullptr, adjoint, dx, dy, dz, s);
}

// ---- host-side shape queries ----------------------------------------------
template <class S> static ShapeDesc make_desc()
{
    ShapeDesc d{};
    d.nmu = S::NMU;
    for (int i = 0; i < S::NMU; ++i)
        d.numax[i] = S::numax[i];
    d.nslot = S::NSLOT;
    return d;
}

const ShapeDesc &shape_desc(int id)
{
    static const ShapeDesc descs[SHAPE_COUNT] = {make_desc<ShapeS1>(), make_desc<ShapeS2>(),
                                                 make_desc<ShapeL16>(), make_desc<ShapeL20>(),
                                                 make_desc<ShapeL24>(), make_desc<ShapePS>()};
    return descs[id];
}

int shape_slot(int id, int mu, int a, int b, int c)
{
    switch (id) {
    case SHAPE_S1: return ShapeS1::slot_of(mu, a, b, c);
    case SHAPE_S2: return ShapeS2::slot_of(mu, a, b, c);
    case SHAPE_L16: return ShapeL16::slot_of(mu, a, b, c);
    case SHAPE_L20: return ShapeL20::slot_of(mu, a, b, c);
    case SHAPE_L24: return ShapeL24::slot_of(mu, a, b, c);
    case SHAPE_PS: return ShapePS::slot_of(mu, a, b, c);
    default: return -1;
    }
}

// ----------------------------------------------------------------------------
// Active-edge lists: one warp per centre tests its edges against the pair
// cutoff with the staging arithmetic (r = sqrt((x*x + y*y) + z*z), the pair's
// rmax, atoms of type -1 and r = 0 excluded) and compacts the active edges in
// list order with a ballot: their list ids, vectors, neighbours and species
// pairs, so that the moment kernels stage the same edges in the same order as
// without the list, read them contiguously, and skip only slots that would
// add exact zeros.  Inactive edges get zero derivatives.  With `rf`, the
// vectors of all listed edges are first recomputed from the moved positions
// and stored (the edge-parallel refresh pass folded into this one).  Six
// blocks per SM (40 registers, no spills): the dependent position gathers want
// the warps (1M atoms: 1.94 -> 1.83 ms against the unbounded 56 registers).
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 6)
    k_active_edges(EdgeArgs p, ActiveEdges out, EdgeRefresh rf,
                               double *__restrict__ dx, double *__restrict__ dy,
                               double *__restrict__ dz)
{
    const int lane = threadIdx.x & 31;
    const int atom = (int)(((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (atom >= p.natoms)
        return;
    const int b = __ldg(p.offsets + atom), end = __ldg(p.offsets + atom + 1);
    const int it = __ldg(p.types + atom);
    int count = 0;
    for (int base = b; base < end; base += 32) {
        const int e = base + lane;
        bool act = false;
        int pair = -1, j = 0;
        double x = 0.0, y = 0.0, z = 0.0;
        if (e < end) {
            j = __ldg(p.nbr + e);
            if (p.pair) {
                pair = __ldg(p.pair + e);
            } else {
                const int jt = __ldg(p.types + j);
                pair = (it >= 0 && jt >= 0) ? it * p.K + jt : -1;
            }
            if (rf.unwrapped) {
                refresh_vector(rf.structs[__ldg(rf.struct_of + atom)], atom, j,
                               __ldg(rf.shift + e), rf.unwrapped, x, y, z);
                rf.rx[e] = x;
                rf.ry[e] = y;
                rf.rz[e] = z;
            } else if (pair >= 0) {
                x = __ldg(p.rx + e);
                y = __ldg(p.ry + e);
                z = __ldg(p.rz + e);
            }
            if (pair >= 0) {
                const double r2 = __dadd_rn(__dadd_rn(__dmul_rn(x, x), __dmul_rn(y, y)),
                                            __dmul_rn(z, z));
                // the staging's test is sqrt(r2) <= rmax (sqrt correctly
                // rounded, monotonic); r2 outside rmax^2 (1 -+ 4 eps) decides
                // it without the square root, the thin band in between takes
                // the staging's own expression
                const double rmax = p.pairs[pair].rmax, q = rmax * rmax;
                if (r2 <= q * (1.0 - 8.9e-16))
                    act = r2 > 0.0;
                else if (r2 < q * (1.0 + 8.9e-16))
                    act = sqrt(r2) <= rmax;
            }
            if (!act && dx) {
                dx[e] = 0.0;
                dy[e] = 0.0;
                dz[e] = 0.0;
            }
        }
        const unsigned m = __ballot_sync(0xffffffffu, act);
        if (act) {
            const int slot = b + count + __popc(m & ((1u << lane) - 1u));
            out.active[slot] = e;
            out.cx[slot] = x;
            out.cy[slot] = y;
            out.cz[slot] = z;
            out.cnbr[slot] = j;
            out.cpair[slot] = pair;
        }
        count += __popc(m);
    }
    if (lane == 0)
        out.nact[atom] = count;
}

__global__ void k_group_max_count(int natoms, const int *__restrict__ count, int *out)
{
    const int atom = blockIdx.x * blockDim.x + threadIdx.x;
    int deg = atom < natoms ? count[atom] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        deg = max(deg, __shfl_xor_sync(0xffffffffu, deg, o));
    if ((threadIdx.x & 31) == 0 && atom - (int)(threadIdx.x & 31) < natoms)
        out[atom >> 5] = deg;
}

cudaError_t launch_active_edges(const EdgeArgs &a, const ActiveEdges &out,
                                const EdgeRefresh *refresh, double *dx, double *dy, double *dz,
                                cudaStream_t s)
{
    if (a.natoms == 0)
        return cudaSuccess;
    EdgeRefresh rf{};
    if (refresh)
        rf = *refresh;
    const long threads = 32L * a.natoms;
    k_active_edges<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(a, out, rf, dx, dy, dz);
    k_group_max_count<<<(a.natoms + 255) / 256, 256, 0, s>>>(a.natoms, out.nact,
                                                             out.group_maxdeg);
    return cudaGetLastError();
}

// ----------------------------------------------------------------------------
// Per-32-atom-group maximum neighbour count (chunk count of the edge kernels)
// ----------------------------------------------------------------------------
__global__ void k_group_maxdeg(int natoms, const int *offsets, int *out)
{
    const int atom = blockIdx.x * blockDim.x + threadIdx.x;
    int deg = 0;
    if (atom < natoms)
        deg = offsets[atom + 1] - offsets[atom];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        deg = max(deg, __shfl_xor_sync(0xffffffffu, deg, o));
    if ((threadIdx.x & 31) == 0 && atom - (int)(threadIdx.x & 31) < natoms)
        out[atom >> 5] = deg;
}

cudaError_t launch_group_maxdeg(int natoms, const int *offsets, int *group_maxdeg,
                                cudaStream_t s)
{
    if (natoms == 0)
        return cudaSuccess;
    const int threads = 256;
    const int blocks = (natoms + threads - 1) / threads;
    k_group_maxdeg<<<blocks, threads, 0, s>>>(natoms, offsets, group_maxdeg);
    return cudaGetLastError();
}

// ----------------------------------------------------------------------------
// Moment graph: forward product rules, site energy, reverse adjoints.
// One block = 16 atoms; each half-warp runs one record stream of the plan.
// Shared memory holds one row of 16 doubles per graph value (basic moments,
// product moments that feed later rules, their adjoints, 1 and 0).  Record
// rows (16 B per stream) are streamed into a double-buffered shared ring by
// TMA bulk copies completing on an mbarrier.
//
// Record semantics (one record = one product rule, use, or marker):
//   acc = (c * row[s1]) * row[s2] + (START ? 0 : acc)
//   END:    GLOBAL ? adjoint[out][atom] = acc : row[out] = acc
//   ENERGY: E += c * acc          (its own product is 0 * 0)
// ----------------------------------------------------------------------------
// Runs n consecutive records of one stream.  All records belong to one
// phase, so a row written here is never read here and record loads may move
// ahead of stores.
template <int ATOMS, int STREAMS, bool FWD, bool GR>
__device__ __forceinline__ void dag_segment(unsigned rec_addr, const Rows<GR> &rowsA, int n,
                                            double *acc, double *E, double *adjoint, int npad,
                                            int natoms, int atom_a)
{
    using G = DagGeom<ATOMS, STREAMS>;
    constexpr unsigned REC_STRIDE = G::SPW * sizeof(DagDevRec);
    auto rare = [&](unsigned outf, double c) {
        if constexpr (FWD) {
            if (outf & DEV_ENERGY) {
                E[0] = fma(c, acc[0], E[0]);
                E[1] = fma(c, acc[1], E[1]);
            }
        }
        if (outf & DEV_END) {
            const unsigned out = outf & DEV_OUT_MASK;
            if (!FWD && (outf & DEV_GLOBAL)) {
                if (atom_a < natoms)
                    __stcs(adjoint + (size_t)out * npad + atom_a, acc[0]);   // streamed out
                if (atom_a + 1 < natoms)
                    __stcs(adjoint + (size_t)out * npad + atom_a + 1, acc[1]);
            } else {
                rowsA.st(out, acc[0], acc[1]);
            }
            acc[0] = 0.0;
            acc[1] = 0.0;
        }
    };
    // groups of four records: the records and operand values of the next group
    // are loaded before the current group is accumulated, so that shared-memory
    // latency overlaps the FP64 work (rows written in this phase are never read
    // in it, so the loads may pass the stores of earlier groups)
    constexpr unsigned RS = ATOMS == 16 ? 7 : 6;   // log2 of the row size in bytes
    struct Grp {
        double c[4];
        unsigned of[4];
        double2 x[4], y[4];
    };
    auto load = [&](Grp &g, int k) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint4 w = lds128(rec_addr + (k + u) * REC_STRIDE);
            g.of[u] = w.y;
            g.c[u] = __hiloint2double((int)w.w, (int)w.z);
            g.x[u] = rowsA.ld((w.x & 0xffffu) << RS);
            g.y[u] = rowsA.ld((w.x >> 16) << RS);
        }
    };
    auto accumulate = [&](const Grp &g) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            acc[0] = fma(g.c[u] * g.x[u].x, g.y[u].x, acc[0]);
            acc[1] = fma(g.c[u] * g.x[u].y, g.y[u].y, acc[1]);
            if (g.of[u])
                rare(g.of[u], g.c[u]);
        }
    };
    int k = 0;
    if (n == G::CH) {   // full ring slot: two-stage schedule over CH/4 groups
        Grp g[2];
        load(g[0], 0);
#pragma unroll
        for (int i = 0; i < G::CH / 4; ++i) {
            if (i + 1 < G::CH / 4)
                load(g[(i + 1) & 1], 4 * (i + 1));
            accumulate(g[i & 1]);
        }
        return;
    }
    for (; k + 4 <= n; k += 4) {
        Grp a;
        load(a, k);
        accumulate(a);
    }
    for (; k < n; ++k) {
        const uint4 w = lds128(rec_addr + k * REC_STRIDE);
        const double2 x = rowsA.ld((w.x & 0xffffu) << RS), y = rowsA.ld((w.x >> 16) << RS);
        const double c = __hiloint2double((int)w.w, (int)w.z);
        acc[0] = fma(c * x.x, y.x, acc[0]);
        acc[1] = fma(c * x.y, y.y, acc[1]);
        if (w.y)
            rare(w.y, c);
    }
}

// GR: rows in the global scratch slice of this block (graphs larger than
// shared memory); the blocks then loop over the atom groups.
template <int ATOMS, bool GR, int STREAMS>
__global__ void __launch_bounds__(DagGeom<ATOMS, STREAMS>::THREADS)
    k_dag(const DagDevRec *__restrict__ recs, const int *__restrict__ phase_row0, int n_fwd,
          int n_rev, int one_row, int zero_row, int nrows, int nslot, int natoms, int npad,
          const int *__restrict__ types, const double *__restrict__ species_coeffs,
          const double *__restrict__ basic, double *__restrict__ adjoint,
          double *__restrict__ site_energy, double *__restrict__ gscratch,
          int *__restrict__ err_flag)
{
    using G = DagGeom<ATOMS, STREAMS>;
    extern __shared__ __align__(128) unsigned char dsm[];
    __shared__ unsigned long long bar[G::WARPS][2];
    __shared__ double epart[STREAMS][ATOMS];
    __shared__ int ph0[DAG_MAX_PHASES + 1];
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int nph = n_fwd + n_rev;
    unsigned char *ring = dsm + (size_t)warp * 2 * G::SLOT_BYTES;   // this warp's two slots
    double *rows = GR ? gscratch + (size_t)blockIdx.x * nrows * ATOMS
                      : reinterpret_cast<double *>(dsm + G::ring_bytes());   // [nrows][ATOMS]
    for (int i = tid; i <= nph; i += blockDim.x)
        ph0[i] = phase_row0[i];
    if (lane == 0) {
        mbar_init(&bar[warp][0], 1);
        mbar_init(&bar[warp][1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    const unsigned rows_u32 = smem_u32(dsm + G::ring_bytes());
    const int g = lane / G::LPS, q = lane - g * G::LPS;
    const int a0 = 2 * q;   // this lane's atoms: a0, a0 + 1
    Rows<GR> rowsA;
    if constexpr (GR)
        rowsA.base = reinterpret_cast<char *>(rows + a0);
    else
        rowsA.base = rows_u32 + a0 * 8;
    const unsigned ring_u32 = smem_u32(ring) + g * sizeof(DagDevRec);
    auto phase_src = [&](int ph) {
        const int rows_p = ph0[ph + 1] - ph0[ph];
        return recs + (size_t)ph0[ph] * STREAMS + (size_t)warp * rows_p * G::SPW;
    };
    auto nchunks = [&](int ph) { return (ph0[ph + 1] - ph0[ph] + G::CH - 1) / G::CH; };
    // lane 0 issues the warp's chunks in consumption order (phase by phase,
    // skipping empty phases); issue j goes to slot j & 1 and is made only
    // after chunk j - 2 has been consumed.  Records do not depend on the
    // phase barriers, so the next phase's chunks are fetched early.
    int iph = 0, ic = 0, nissued = 0, kw = 0;
    auto issue_next = [&]() {
        while (iph < nph && ic >= nchunks(iph)) {
            ++iph;
            ic = 0;
        }
        if (iph < nph) {
            const int rows_p = ph0[iph + 1] - ph0[iph];
            const int r = min(G::CH, rows_p - ic * G::CH);
            const int slot = nissued & 1;
            bulk_load(ring + slot * G::SLOT_BYTES, phase_src(iph) + (size_t)ic * G::CH * G::SPW,
                      (unsigned)(r * G::SPW * sizeof(DagDevRec)), &bar[warp][slot]);
            ++ic;
            ++nissued;
        }
    };
    const int ngroups = (natoms + ATOMS - 1) / ATOMS;
    for (int grp = blockIdx.x; grp < ngroups; grp += gridDim.x) {
        const int atom0 = grp * ATOMS;
        __syncthreads();   // the previous group's rows are no longer read
        // basic moments (two atoms per copy); in a partial last group the
        // lanes past natoms read row padding (inside the npad stride) and
        // their results are never written out
        for (int i = tid; i < nslot * (ATOMS / 2); i += blockDim.x) {
            const int sl = i / (ATOMS / 2), a = 2 * (i - sl * (ATOMS / 2));
            const double *src = basic + (size_t)sl * npad + atom0 + a;
            if constexpr (GR)
                *reinterpret_cast<double2 *>(rows + (size_t)sl * ATOMS + a) =
                    __ldcs(reinterpret_cast<const double2 *>(src));   // read once
            else
                cp_async16(rows_u32 + (unsigned)(sl * ATOMS + a) * 8, src);
        }
        if constexpr (!GR)
            asm volatile("cp.async.wait_all;" ::: "memory");
        if (tid < ATOMS) {
            rows[(size_t)one_row * ATOMS + tid] = 1.0;
            rows[(size_t)zero_row * ATOMS + tid] = 0.0;
        }
        __syncthreads();
        if (lane == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            iph = 0;
            ic = 0;
            issue_next();
            issue_next();
        }
        double E[2] = {0.0, 0.0}, acc[2] = {0.0, 0.0};
        for (int ph = 0; ph < nph; ++ph) {
            const int rows_p = ph0[ph + 1] - ph0[ph];
            const int nch = nchunks(ph);
            const bool fwd = ph < n_fwd;
            for (int c = 0; c < nch; ++c, ++kw) {
                const int slot = kw & 1;
                long it = 0;
                while (!mbar_try_wait(&bar[warp][slot], (unsigned)((kw >> 1) & 1))) {
                    if (++it > DAG_WAIT_LIMIT) {
                        *err_flag = 1;
                        break;
                    }
                }
                const int n = min(G::CH, rows_p - c * G::CH);
                const unsigned rec_addr = ring_u32 + slot * G::SLOT_BYTES;
                if (fwd)
                    dag_segment<ATOMS, STREAMS, true, GR>(rec_addr, rowsA, n, acc, E, adjoint, npad,
                                                 natoms, atom0 + a0);
                else
                    dag_segment<ATOMS, STREAMS, false, GR>(rec_addr, rowsA, n, acc, E, adjoint, npad,
                                                  natoms, atom0 + a0);
                __syncwarp();
                if (lane == 0) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue_next();
                }
            }
            __syncthreads();
            if (ph + 1 == n_fwd) {
                const int stream = warp * G::SPW + g;
                epart[stream][a0] = E[0];
                epart[stream][a0 + 1] = E[1];
                __syncthreads();
                if (tid < ATOMS && atom0 + tid < natoms) {
                    const int t = types[atom0 + tid];
                    double se = 0.0;
                    if (t >= 0) {
                        se = species_coeffs[t];
                        for (int s2 = 0; s2 < STREAMS; ++s2)
                            se += epart[s2][tid];
                    }
                    site_energy[atom0 + tid] = se;
                }
            }
        }
    }
}

// Device records of a plan: warp-major per phase ([phase][warp][row][SPW
// streams]) for the selected block geometry; store targets become byte
// offsets, operand rows stay indices.
std::vector<DagDevRec> dag_device_records(const DagPlan &plan)
{
    const int spw = plan.atoms == 16 ? DagGeom<16, 32>::SPW : DagGeom<8, 32>::SPW;
    const unsigned row_bytes = (unsigned)plan.atoms * 8;
    std::vector<DagDevRec> out(plan.recs.size());
    size_t row0 = 0, o = 0;
    const int S = plan.streams;
    const int warps = S / spw;
    for (int rows_p : plan.phase_rows) {
        for (int w = 0; w < warps; ++w)
            for (int r = 0; r < rows_p; ++r)
                for (int s = 0; s < spw; ++s) {
                    const DagRec &in = plan.recs[(row0 + r) * S + w * spw + s];
                    DagDevRec d{};
                    d.rows = in.s12;   // row indices; the kernel scales them
                    d.c = in.c;
                    const unsigned flags = in.outf >> 16, out_ = in.outf & 0xffffu;
                    unsigned f = 0;
                    if (flags & DAG_END)
                        f |= DEV_END;
                    if (flags & DAG_GLOBAL)
                        f |= DEV_GLOBAL;
                    if (flags & DAG_ENERGY)
                        f |= DEV_ENERGY;
                    d.outf = f ? (f | ((flags & DAG_GLOBAL) ? out_ : out_ * row_bytes)) : 0u;
                    out[o++] = d;
                }
        row0 += rows_p;
    }
    return out;
}

size_t dag_ring_bytes(int atoms)
{
    // the same for both stream counts (dag_chunk_rows)
    return atoms == 16 ? DagGeom<16, 32>::ring_bytes() : DagGeom<8, 32>::ring_bytes();
}

template <int ATOMS, bool GR, int STREAMS>
static cudaError_t launch_dag_geom(const DagPlan &plan, const DagDevRec *recs,
                                   const int *phase_row0, int nslot, int natoms, int npad,
                                   const int *types, const double *species_coeffs,
                                   const double *basic, double *adjoint, double *site_energy,
                                   double *gscratch, int *err_flag, cudaStream_t s)
{
    using G = DagGeom<ATOMS, STREAMS>;
    const int ngroups = (natoms + ATOMS - 1) / ATOMS;
    const size_t smem = G::ring_bytes() + (GR ? 0 : sizeof(double) * (size_t)plan.nrows * ATOMS);
    auto kern = k_dag<ATOMS, GR, STREAMS>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
    if (err == cudaSuccess && GR)   // leave the rest of the SM's memory to L1
        err = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 25);
    // persistent blocks (as many as fit the SMs; with global rows one per SM,
    // the scratch slices), each looping over atom groups
    int per = 1;
    if (err == cudaSuccess && !GR)
        err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, G::THREADS, smem);
    if (err != cudaSuccess)
        return err;
    const int blocks = std::min(ngroups, plan.grid * std::max(per, 1));
    kern<<<blocks, G::THREADS, smem, s>>>(recs, phase_row0, plan.n_fwd, plan.n_rev, plan.one_row,
                                          plan.zero_row, plan.nrows, nslot, natoms, npad, types,
                                          species_coeffs, basic, adjoint, site_energy, gscratch,
                                          err_flag);
    return cudaGetLastError();
}

cudaError_t launch_dag(const DagPlan &plan, const DagDevRec *recs, const int *phase_row0, int nslot,
                       int natoms, int npad, const int *types, const double *species_coeffs,
                       const double *basic, double *adjoint, double *site_energy,
                       double *gscratch, int *err_flag, cudaStream_t s)
{
    if (natoms == 0)
        return cudaSuccess;
    if (plan.n_fwd + plan.n_rev > DAG_MAX_PHASES)
        return cudaErrorInvalidValue;
    const bool large = plan.streams == DAG_STREAMS_LARGE;
    if (plan.streams != DAG_STREAMS && !large)
        return cudaErrorInvalidValue;
#define MTPB_DAG_LAUNCH(A, GR, S, SCR)                                                             \
    launch_dag_geom<A, GR, S>(plan, recs, phase_row0, nslot, natoms, npad, types, species_coeffs, \
                              basic, adjoint, site_energy, SCR, err_flag, s)
    if (plan.global_rows) {
        if (plan.atoms != 16 || !gscratch || plan.grid < 1)
            return cudaErrorInvalidValue;
        return large ? MTPB_DAG_LAUNCH(16, true, 64, gscratch)
                     : MTPB_DAG_LAUNCH(16, true, 32, gscratch);
    }
    if (plan.atoms == 16)
        return large ? MTPB_DAG_LAUNCH(16, false, 64, nullptr)
                     : MTPB_DAG_LAUNCH(16, false, 32, nullptr);
    return large ? MTPB_DAG_LAUNCH(8, false, 64, nullptr) : MTPB_DAG_LAUNCH(8, false, 32, nullptr);
#undef MTPB_DAG_LAUNCH
}

// ----------------------------------------------------------------------------
// Forces and per-atom virial by gather (deterministic, no atomics):
//   F_k = sum_{e in out(k)} d_e - sum_{e in in(k)} d_e      (getEFS scatter)
//   W_k = - sum_{e in out(k)} d_e (x) r_e                   (stress_ -= d r)
// One warp per atom: lanes stride over the atom's out- and in-edges
// (coalesced edge arrays), then a fixed shuffle tree sums the lanes.
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    k_force_gather(int natoms, int ntotal, const int *__restrict__ offsets,
                   const int *__restrict__ in_offsets, const int *__restrict__ in_edges,
                   const double *__restrict__ dx, const double *__restrict__ dy,
                   const double *__restrict__ dz, const double *__restrict__ rx,
                   const double *__restrict__ ry, const double *__restrict__ rz,
                   double *__restrict__ forces, double *__restrict__ atom_virial,
                   int accumulate)
{
    const int k = (int)(((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (k >= ntotal)
        return;   // whole warps leave together
    double v[12] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};   // F (3), W (9)
    if (k < natoms) {
        const int e1 = offsets[k + 1];
        for (int e = offsets[k] + lane; e < e1; e += 32) {
            const double a = dx[e], b = dy[e], c = dz[e];
            const double x = rx[e], y = ry[e], z = rz[e];
            v[0] += a;
            v[1] += b;
            v[2] += c;
            v[3] -= a * x; v[4] -= a * y; v[5] -= a * z;
            v[6] -= b * x; v[7] -= b * y; v[8] -= b * z;
            v[9] -= c * x; v[10] -= c * y; v[11] -= c * z;
        }
    }
    const int q1 = in_offsets[k + 1];
    for (int q = in_offsets[k] + lane; q < q1; q += 32) {
        const int e = in_edges[q];
        v[0] -= dx[e];
        v[1] -= dy[e];
        v[2] -= dz[e];
    }
    const bool vir = atom_virial && k < natoms;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
    if (vir) {
#pragma unroll
        for (int i = 3; i < 12; ++i)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
                v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
    }
    if (lane == 0) {
        if (accumulate) {
            forces[3 * (size_t)k] += v[0];
            forces[3 * (size_t)k + 1] += v[1];
            forces[3 * (size_t)k + 2] += v[2];
        } else {
            forces[3 * (size_t)k] = v[0];
            forces[3 * (size_t)k + 1] = v[1];
            forces[3 * (size_t)k + 2] = v[2];
        }
    }
    if (vir && lane == 0) {
#pragma unroll
        for (int i = 0; i < 9; ++i)
            atom_virial[(size_t)i * natoms + k] = v[3 + i];
    }
}

cudaError_t launch_force_gather(int natoms, int ntotal, const int *offsets, const int *in_offsets,
                                const int *in_edges, const double *dx, const double *dy,
                                const double *dz, const double *rx, const double *ry,
                                const double *rz, double *forces, double *atom_virial,
                                int accumulate, cudaStream_t s)
{
    if (ntotal == 0)
        return cudaSuccess;
    const int threads = 256;   // 8 atoms per block
    const long blocks = ((long)ntotal * 32 + threads - 1) / threads;
    k_force_gather<<<(unsigned)blocks, threads, 0, s>>>(natoms, ntotal, offsets, in_offsets,
                                                        in_edges, dx, dy, dz, rx, ry, rz, forces,
                                                        atom_virial, accumulate);
    return cudaGetLastError();
}

// ----------------------------------------------------------------------------
// Deterministic reductions: segments (contiguous atoms of one structure, at
// most 1024 atoms) -> partials[seg][10] = {E, W00..W22}; then per structure.
// ----------------------------------------------------------------------------
__global__ void k_segment_reduce(const int *__restrict__ seg_begin,
                                 const int *__restrict__ seg_end,
                                 const double *__restrict__ site_energy,
                                 const double *__restrict__ atom_virial, int natoms,
                                 double *__restrict__ partials)
{
    __shared__ double sh[10][256];
    const int seg = blockIdx.x;
    const int b = seg_begin[seg], e = seg_end[seg];
    double v[10] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = b + threadIdx.x; i < e; i += blockDim.x) {
        v[0] += site_energy[i];
        if (atom_virial)
#pragma unroll
            for (int q = 0; q < 9; ++q)
                v[1 + q] += atom_virial[(size_t)q * natoms + i];
    }
#pragma unroll
    for (int q = 0; q < 10; ++q)
        sh[q][threadIdx.x] = v[q];
    __syncthreads();
    for (int st = blockDim.x / 2; st > 0; st >>= 1) {
        if (threadIdx.x < st)
#pragma unroll
            for (int q = 0; q < 10; ++q)
                sh[q][threadIdx.x] += sh[q][threadIdx.x + st];
        __syncthreads();
    }
    if (threadIdx.x < 10)
        partials[(size_t)seg * 10 + threadIdx.x] = sh[threadIdx.x][0];
}

cudaError_t launch_segment_reduce(int nseg, const int *seg_begin, const int *seg_end,
                                  const double *site_energy, const double *atom_virial,
                                  int natoms, double *partials, cudaStream_t s)
{
    if (nseg == 0)
        return cudaSuccess;
    k_segment_reduce<<<nseg, 256, 0, s>>>(seg_begin, seg_end, site_energy, atom_virial, natoms,
                                          partials);
    return cudaGetLastError();
}

__global__ void k_struct_reduce(int nstruct, const int *__restrict__ struct_seg0,
                                const double *__restrict__ partials, double *__restrict__ energy,
                                double *__restrict__ virial)
{
    // one block per structure; fixed-order tree over its segments
    __shared__ double sh[10][128];
    const int s = blockIdx.x;
    double v[10] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
    for (int g = struct_seg0[s] + threadIdx.x; g < struct_seg0[s + 1]; g += blockDim.x)
#pragma unroll
        for (int q = 0; q < 10; ++q)
            v[q] += partials[(size_t)g * 10 + q];
#pragma unroll
    for (int q = 0; q < 10; ++q)
        sh[q][threadIdx.x] = v[q];
    __syncthreads();
    for (int st = blockDim.x / 2; st > 0; st >>= 1) {
        if (threadIdx.x < st)
#pragma unroll
            for (int q = 0; q < 10; ++q)
                sh[q][threadIdx.x] += sh[q][threadIdx.x + st];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        if (energy)
            energy[s] = sh[0][0];
        if (virial)
#pragma unroll
            for (int q = 0; q < 9; ++q)
                virial[(size_t)s * 9 + q] = sh[1 + q][0];
    }
}

cudaError_t launch_struct_reduce(int nstruct, const int *struct_seg0, const double *partials,
                                 double *energy, double *virial, cudaStream_t s)
{
    if (nstruct == 0)
        return cudaSuccess;
    k_struct_reduce<<<nstruct, 128, 0, s>>>(nstruct, struct_seg0, partials, energy, virial);
    return cudaGetLastError();
}

} // namespace mtpb
