// grad.cu -- FP64 kernels of the coefficient gradient of the training loss:
// tangent basic moments, the dual moment graph and the per-edge radial
// gradient records.
//
// Reference semantics (paths relative to the reference project):
//   PotMTP::accumulate_site_parameter_gradient
//                 potentials/potential_mtp.cpp:3348-3550
//   PotMTP::AccumulateEFSCombinationGard  potential_mtp.cpp:6896-6922
//
// For one site with loss weights dLdE (energy) and w_j (per edge; from the
// force and stress terms, w_j = dLdF_i - dLdF_j - dLdS r_j) the reference
// differentiates Phi = dLdE * E_i + sum_j w_j . dE_i/dr_j with respect to the
// coefficients.  With D_w = sum_j w_j . d/dr_j this is Phi = dLdE E + D_w E,
// so the kernels carry dual numbers (value, D_w value):
//   - tangent basics   Db[mu,abc] = sum_j D_w (f_mu u_abc),  u = xhat^a yhat^b zhat^c,
//     D_w xhat = (w_x - xhat s)/r, D_w f_mu = f'_mu s, s = w . rhat
//     (the reference's dlds of the basic moments, :3431-3446);
//   - dual graph: forward m, D_w m (dlds, :3477-3483); reverse a = dE/dm (sed)
//     and abar = dPhi/dm (dldm, :3484-3497), one product rule in dual
//     arithmetic; the moment-coefficient gradient dLdE m + D_w m (:3540-3546);
//   - radial gradient by channel:  dPhi/dc[pair,mu,xi] =
//     sum_j Q_xi(r_j) (A_mu + P_mu) + Q'_xi(r_j) s S_mu,
//     S_mu = sum a_k u_k, P_mu = sum a_k D_w u_k, A_mu = sum abar_k u_k over the
//     basics k of channel mu -- the contraction of the reference's
//     moment_jacobian_coeffs / _coord workspaces (:3424-3452, 3520-3535)
//     without materialising them.
#include "radial.cuh"
#include "internal.hpp"
#include "moments.cuh"
#include "dag.cuh"

#include <algorithm>

namespace mtpb {

// warps of the gradient edge kernels and edge slots per staged chunk: the
// level-20 shape runs 8 warps; the level-24 shape partitions its chains over
// 12 warps (so that a thread may hold the value and weighted adjoints of its
// chains in registers) run as three launches of 4 warps, three blocks per SM
// (one unrolled body per scheduler)
template <class S> struct GradCfg {
    static constexpr int NW = S::NSLOT > 400 ? 4 : S::NSLOT > 200 ? 8 : ShapeCfg<S>::NW;
    static constexpr int NPART = S::NSLOT > 400 ? 3 : 1;
    static constexpr int KSG = S::NMU >= 6 ? 4 : 8;
    static constexpr int BLOCKS = NPART > 1 ? 3 : 1;   // blocks per SM
};

template <int KSG> __device__ __forceinline__ double &SG(double *st, int row, int k, int lane)
{
    return st[(row * KSG + k) * STR + lane];
}

// staging rows: 0-2 rhat, 3-5 D_w rhat, 6 s = w.rhat; TAN adds f_mu, D_w f_mu
template <class S, bool TAN> constexpr int grad_stage_rows()
{
    return TAN ? 7 + 2 * S::NMU : 7;
}

template <class S, bool TAN> constexpr size_t grad_smem_doubles(int K, int R)
{
    constexpr int KSG = GradCfg<S>::KSG;
    constexpr int NW = GradCfg<S>::NW;
    size_t n = (size_t)grad_stage_rows<S, TAN>() * KSG * STR;
    if (!TAN)
        n += (size_t)NW * 2 * S::NMU * KSG * 32;   // per-warp partial sums
    n += PAIR_PARAM_DOUBLES * K * K + (size_t)K * K * S::NMU * R;
    return n;
}

struct GradView {
    double *st;
    double *part;
    const PairParams *pairs;
    const double *radial;   // [K*K][NMU][R]
};

// Per-edge dual geometry (and for TAN the radial functions with their
// directional derivatives) of one chunk of edge slots of 32 atoms.  Edges the
// reference skips (r > cutoff, r = 0, type -1) stage zeros.
template <class S, int NW, bool TAN, bool RG>
__device__ __forceinline__ void grad_stage(const EdgeArgs &p, const double *__restrict__ wx,
                                           const double *__restrict__ wy,
                                           const double *__restrict__ wz, const GradView &v,
                                           int atom0, int chunk)
{
    constexpr int NMU = S::NMU;
    constexpr int KSG = GradCfg<S>::KSG;
    for (int item = threadIdx.x; item < 32 * KSG; item += blockDim.x) {
        const int lane = item / KSG;
        const int k = item - lane * KSG;
        const int atom = atom0 + lane;
        double h[3] = {0.0, 0.0, 0.0}, hd[3] = {0.0, 0.0, 0.0}, sw = 0.0;
        double f[NMU], fd[NMU];
#pragma unroll
        for (int m = 0; m < NMU; ++m) {
            f[m] = 0.0;
            fd[m] = 0.0;
        }
        if (atom < p.natoms) {
            const int e = __ldg(p.offsets + atom) + chunk * KSG + k;
            if (e < __ldg(p.offsets + atom + 1)) {
                const double x = __ldg(p.rx + e), y = __ldg(p.ry + e), z = __ldg(p.rz + e);
                const double r2 = __dadd_rn(__dadd_rn(__dmul_rn(x, x), __dmul_rn(y, y)),
                                            __dmul_rn(z, z));
                const double r = sqrt(r2);
                const int it = __ldg(p.types + atom);
                const int jt = __ldg(p.types + __ldg(p.nbr + e));
                const int pair = (it >= 0 && jt >= 0) ? it * p.K + jt : 0;
                const PairParams &pp = v.pairs[pair];
                if (it >= 0 && jt >= 0 && r > 0.0 && r <= pp.rmax) {
                    const double rinv = 1.0 / r;
                    const double w[3] = {__ldg(wx + e), __ldg(wy + e), __ldg(wz + e)};
                    h[0] = x * rinv;
                    h[1] = y * rinv;
                    h[2] = z * rinv;
                    sw = fma(w[2], h[2], fma(w[1], h[1], w[0] * h[0]));
#pragma unroll
                    for (int a = 0; a < 3; ++a)
                        hd[a] = (w[a] - h[a] * sw) * rinv;
                    if constexpr (TAN) {
                        const double *c = v.radial + pair * NMU * p.R;
                        double fp[NMU];
#pragma unroll
                        for (int m = 0; m < NMU; ++m) {
                            f[m] = 0.0;
                            fp[m] = 0.0;
                        }
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
#pragma unroll
                        for (int m = 0; m < NMU; ++m)
                            fd[m] = fp[m] * sw;
                    }
                }
            }
        }
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            SG<KSG>(v.st, a, k, lane) = h[a];
            SG<KSG>(v.st, 3 + a, k, lane) = hd[a];
        }
        SG<KSG>(v.st, 6, k, lane) = sw;
        if constexpr (TAN) {
#pragma unroll
            for (int m = 0; m < NMU; ++m) {
                SG<KSG>(v.st, 7 + m, k, lane) = f[m];
                SG<KSG>(v.st, 7 + NMU + m, k, lane) = fd[m];
            }
        }
    }
}

// powers of yhat and zhat
template <int N> __device__ __forceinline__ void powers(double h, double *p)
{
    p[0] = 1.0;
#pragma unroll
    for (int i = 1; i <= N; ++i)
        p[i] = p[i - 1] * h;
}

// chain base u = yhat^b zhat^c and D_w u = b yhat^(b-1) zhat^c D_w yhat
// + c yhat^b zhat^(c-1) D_w zhat
template <int B, int C>
__device__ __forceinline__ void chain_base(const double *yp, const double *zp, double yd,
                                           double zd, double &u, double &ud)
{
    if constexpr (B == 0 && C == 0) {
        u = 1.0;
        ud = 0.0;
    } else if constexpr (B == 0) {
        u = zp[C];
        ud = double(C) * zp[C - 1] * zd;
    } else if constexpr (C == 0) {
        u = yp[B];
        ud = double(B) * yp[B - 1] * yd;
    } else {
        u = yp[B] * zp[C];
        ud = fma(double(B) * yp[B - 1] * yd, zp[C], double(C) * yp[B] * zp[C - 1] * zd);
    }
}

// ----------------------------------------------------------------------------
// Tangent basic moments of 32 atoms: Db = sum_j (D_w f) u + f D_w u.  Warp W
// owns the chains of Partition, as in the forward kernel.
// ----------------------------------------------------------------------------
template <class S, int NW, int W, bool RG>
__device__ __forceinline__ void tan_warp(const EdgeArgs &p, const double *wx, const double *wy,
                                         const double *wz, const GradView &v, int atom0,
                                         int maxdeg, double *tangent)
{
    using P = Partition<S, NW>;
    constexpr int NACC = P::table.nacc[W];
    constexpr int NCHW = P::table.count[W];
    constexpr int MAXB = P::table.maxb[W];
    constexpr int MAXC = P::table.maxc[W];
    constexpr int NMU = S::NMU;
    constexpr int KSG = GradCfg<S>::KSG;
    const int lane = threadIdx.x & 31;
    double acc[NACC > 0 ? NACC : 1];
#pragma unroll
    for (int i = 0; i < NACC; ++i)
        acc[i] = 0.0;
    const int nchunks = (maxdeg + KSG - 1) / KSG;
    for (int ch = 0; ch < nchunks; ++ch) {
        grad_stage<S, NW, true, RG>(p, wx, wy, wz, v, atom0, ch);
        __syncthreads();
        const int kend = min(KSG, maxdeg - ch * KSG);
        for (int k = 0; k < kend; ++k) {
            const double xh = SG<KSG>(v.st, 0, k, lane);
            const double xd = SG<KSG>(v.st, 3, k, lane);
            double f[NMU], fd[NMU];
#pragma unroll
            for (int m = 0; m < NMU; ++m) {
                f[m] = SG<KSG>(v.st, 7 + m, k, lane);
                fd[m] = SG<KSG>(v.st, 7 + NMU + m, k, lane);
            }
            const double yd = SG<KSG>(v.st, 4, k, lane), zd = SG<KSG>(v.st, 5, k, lane);
            double yp[MAXB + 1], zp[MAXC + 1];
            powers<MAXB>(SG<KSG>(v.st, 1, k, lane), yp);
            powers<MAXC>(SG<KSG>(v.st, 2, k, lane), zp);
            static_for<NCHW>([&](auto ii) {
                constexpr int ci = P::table.list[W * S::NCH + decltype(ii)::value];
                constexpr int a0 = P::table.acc0[W * S::NCH + decltype(ii)::value];
                constexpr int b = S::chains.b[ci];
                constexpr int c = S::chains.c[ci];
                constexpr int L = S::chains.len[ci];
                double u, ud;
                chain_base<b, c>(yp, zp, yd, zd, u, ud);
                static_for<L>([&](auto ia) {
                    constexpr int a = decltype(ia)::value;
                    constexpr int nu = a + b + c;
                    constexpr int off = a0 + chain_acc_off<S>(b + c, a);
                    static_for<S::cnt(nu)>([&](auto iq) {
                        constexpr int q = decltype(iq)::value;
                        constexpr int m = S::chan(nu, q);
                        acc[off + q] = fma(fd[m], u, fma(f[m], ud, acc[off + q]));
                    });
                    if constexpr (a + 1 < L) {
                        ud = fma(ud, xh, u * xd);
                        u *= xh;
                    }
                });
            });
        }
        __syncthreads();
    }
    const int atom = atom0 + lane;
    if (atom < p.natoms) {
        static_for<NCHW>([&](auto ii) {
            constexpr int ci = P::table.list[W * S::NCH + decltype(ii)::value];
            constexpr int a0 = P::table.acc0[W * S::NCH + decltype(ii)::value];
            constexpr int n = S::chains.nacc[ci];
            constexpr int slot0 = S::chains.slot0[ci];
#pragma unroll
            for (int i = 0; i < n; ++i)
                tangent[(size_t)(slot0 + i) * p.npad + atom] = acc[a0 + i];
        });
    }
}

// ----------------------------------------------------------------------------
// Per-edge channel sums of 32 atoms for the radial gradient.  Each warp adds
// its chains' share of U_mu = A_mu + P_mu and S_mu; the shares are summed in
// warp order and stored as uv[e] = {U_0..U_{NMU-1}, s S_0 .. s S_{NMU-1}}.
// PASS 0 does all terms; where the two adjoint sets do not fit the registers
// PASS 1 stores the terms of a (U = P) and PASS 2 adds A_mu to U.  NW is the
// size of the chain partition, W the warp's index in it, NWB the warps of the
// block; only the first part of the first pass stores, the others add.
// ----------------------------------------------------------------------------
template <class S, int NW, int W, int PASS, int NWB, bool FIRST>
__device__ __forceinline__ void edge_grad_warp(const EdgeArgs &p, const double *wx,
                                               const double *wy, const double *wz,
                                               const GradView &v, int atom0, int maxdeg,
                                               const double *adjoint, const double *adjoint2,
                                               double *uv)
{
    using P = Partition<S, NW>;
    constexpr int NACC = P::table.nacc[W];
    constexpr int NCHW = P::table.count[W];
    constexpr int MAXB = P::table.maxb[W];
    constexpr int MAXC = P::table.maxc[W];
    constexpr int NMU = S::NMU;
    constexpr int KSG = GradCfg<S>::KSG;
    constexpr bool HA = PASS != 2, HB = PASS != 1;
    const int lane = threadIdx.x & 31;
    const int atom = atom0 + lane;
    double adj[(HA && NACC > 0) ? NACC : 1], adj2[(HB && NACC > 0) ? NACC : 1];
    if (atom < p.natoms) {
        static_for<NCHW>([&](auto ii) {
            constexpr int ci = P::table.list[W * S::NCH + decltype(ii)::value];
            constexpr int a0 = P::table.acc0[W * S::NCH + decltype(ii)::value];
            constexpr int n = S::chains.nacc[ci];
            constexpr int slot0 = S::chains.slot0[ci];
#pragma unroll
            for (int i = 0; i < n; ++i) {
                if constexpr (HA)
                    adj[a0 + i] = __ldg(adjoint + (size_t)(slot0 + i) * p.npad + atom);
                if constexpr (HB)
                    adj2[a0 + i] = __ldg(adjoint2 + (size_t)(slot0 + i) * p.npad + atom);
            }
        });
    } else {
#pragma unroll
        for (int i = 0; i < NACC; ++i) {
            if constexpr (HA)
                adj[i] = 0.0;
            if constexpr (HB)
                adj2[i] = 0.0;
        }
    }
    const int nchunks = (maxdeg + KSG - 1) / KSG;
    double *part = v.part + (size_t)(W % NWB) * 2 * NMU * KSG * 32;
    for (int ch = 0; ch < nchunks; ++ch) {
        grad_stage<S, NW, false, false>(p, wx, wy, wz, v, atom0, ch);
        __syncthreads();
        const int kend = min(KSG, maxdeg - ch * KSG);
        for (int k = 0; k < kend; ++k) {
            const double xh = SG<KSG>(v.st, 0, k, lane);
            const double xd = SG<KSG>(v.st, 3, k, lane);
            const double yd = SG<KSG>(v.st, 4, k, lane), zd = SG<KSG>(v.st, 5, k, lane);
            double yp[MAXB + 1], zp[MAXC + 1];
            powers<MAXB>(SG<KSG>(v.st, 1, k, lane), yp);
            powers<MAXC>(SG<KSG>(v.st, 2, k, lane), zp);
            double Sm[NMU], Um[NMU];
#pragma unroll
            for (int m = 0; m < NMU; ++m) {
                Sm[m] = 0.0;
                Um[m] = 0.0;
            }
            static_for<NCHW>([&](auto ii) {
                constexpr int ci = P::table.list[W * S::NCH + decltype(ii)::value];
                constexpr int a0 = P::table.acc0[W * S::NCH + decltype(ii)::value];
                constexpr int b = S::chains.b[ci];
                constexpr int c = S::chains.c[ci];
                constexpr int L = S::chains.len[ci];
                double u, ud;
                chain_base<b, c>(yp, zp, yd, zd, u, ud);
                static_for<L>([&](auto ia) {
                    constexpr int a = decltype(ia)::value;
                    constexpr int nu = a + b + c;
                    constexpr int off = a0 + chain_acc_off<S>(b + c, a);
                    static_for<S::cnt(nu)>([&](auto iq) {
                        constexpr int q = decltype(iq)::value;
                        constexpr int m = S::chan(nu, q);
                        if constexpr (HA) {
                            Sm[m] = fma(adj[off + q], u, Sm[m]);
                            Um[m] = fma(adj[off + q], ud, Um[m]);
                        }
                        if constexpr (HB)
                            Um[m] = fma(adj2[off + q], u, Um[m]);
                    });
                    if constexpr (a + 1 < L) {
                        if constexpr (HA)
                            ud = fma(ud, xh, u * xd);
                        u *= xh;
                    }
                });
            });
#pragma unroll
            for (int m = 0; m < NMU; ++m) {
                part[(m * KSG + k) * 32 + lane] = Um[m];
                if constexpr (HA)
                    part[((NMU + m) * KSG + k) * 32 + lane] = Sm[m];
            }
        }
        __syncthreads();
        for (int item = threadIdx.x; item < 32 * KSG; item += NWB * 32) {
            const int k = item >> 5;
            const int ln = item & 31;
            const int at = atom0 + ln;
            if (k >= kend || at >= p.natoms)
                continue;
            const int e = __ldg(p.offsets + at) + ch * KSG + k;
            if (e >= __ldg(p.offsets + at + 1))
                continue;
            const double sw = SG<KSG>(v.st, 6, k, ln);
            double *o = uv + (size_t)e * 2 * NMU;
#pragma unroll
            for (int m = 0; m < (HA ? 2 * NMU : NMU); ++m) {
                double t = 0.0;
#pragma unroll
                for (int w = 0; w < NWB; ++w)
                    t += v.part[(size_t)w * 2 * NMU * KSG * 32 + (m * KSG + k) * 32 + ln];
                const double val = m < NMU ? t : t * sw;
                if constexpr (PASS != 2 && FIRST)
                    o[m] = val;
                else
                    o[m] += val;
            }
        }
        __syncthreads();
    }
}

// MODE 0: tangent basics; 1-3: edge records with PASS = MODE - 1; PART: which
// block of NW warps of the chain partition this launch runs
template <class S, int MODE, int PART, bool RG>
__global__ void __launch_bounds__(GradCfg<S>::NW * 32, GradCfg<S>::BLOCKS)
    k_grad_moments(EdgeArgs p, const double *__restrict__ wx, const double *__restrict__ wy,
                   const double *__restrict__ wz, const double *__restrict__ adjoint,
                   const double *__restrict__ adjoint2, double *__restrict__ out)
{
    constexpr int NW = GradCfg<S>::NW;
    constexpr int NMU = S::NMU;
    constexpr int KSG = GradCfg<S>::KSG;
    constexpr bool TAN = MODE == 0;
    extern __shared__ double smem[];
    GradView v;
    v.st = smem;
    double *cur = smem + grad_stage_rows<S, TAN>() * KSG * STR;
    v.part = cur;
    if (!TAN)
        cur += NW * 2 * NMU * KSG * 32;
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
    const int group = blockIdx.x;
    const int atom0 = group * 32;
    const int maxdeg = __ldg(p.group_maxdeg + group);
    const int warp = threadIdx.x >> 5;
    constexpr int NWT = NW * GradCfg<S>::NPART;
    static_for<NW>([&](auto iw) {
        constexpr int WL = decltype(iw)::value;
        constexpr int W = PART * NW + WL;
        if (warp == WL) {
            if constexpr (TAN)
                tan_warp<S, NWT, W, RG>(p, wx, wy, wz, v, atom0, maxdeg, out);
            else
                edge_grad_warp<S, NWT, W, MODE - 1, NW, PART == 0>(p, wx, wy, wz, v, atom0,
                                                                   maxdeg, adjoint, adjoint2,
                                                                   out);
        }
    });
}

template <class S, int MODE>
static cudaError_t launch_grad_shape(const EdgeArgs &a, const double *wx, const double *wy,
                                     const double *wz, const double *adjoint,
                                     const double *adjoint2, double *out, cudaStream_t s)
{
    constexpr int NW = GradCfg<S>::NW;
    const int groups = (a.natoms + 31) / 32;
    if (groups == 0)
        return cudaSuccess;
    const size_t smem = sizeof(double) * grad_smem_doubles<S, MODE == 0>(a.K, a.R);
    cudaError_t err = cudaSuccess;
    static_for<GradCfg<S>::NPART>([&](auto ip) {
        constexpr int P = decltype(ip)::value;
        if (err != cudaSuccess)
            return;
        // the edge records take no radial values: one instantiation
        auto kern = (MODE == 0 && a.rb_generic) ? k_grad_moments<S, MODE, P, MODE == 0>
                                                : k_grad_moments<S, MODE, P, false>;
        err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (err == cudaSuccess) {
            kern<<<groups, NW * 32, smem, s>>>(a, wx, wy, wz, adjoint, adjoint2, out);
            err = cudaGetLastError();
        }
    });
    return err;
}

template <int MODE>
static cudaError_t grad_dispatch(int shape, const EdgeArgs &a, const double *wx, const double *wy,
                                 const double *wz, const double *adjoint, const double *adjoint2,
                                 double *out, cudaStream_t s)
{
    switch (shape) {
    case SHAPE_S1:
        return launch_grad_shape<ShapeS1, MODE>(a, wx, wy, wz, adjoint, adjoint2, out, s);
    case SHAPE_S2:
        return launch_grad_shape<ShapeS2, MODE>(a, wx, wy, wz, adjoint, adjoint2, out, s);
    case SHAPE_L16:
        return launch_grad_shape<ShapeL16, MODE>(a, wx, wy, wz, adjoint, adjoint2, out, s);
    case SHAPE_L20:
        return launch_grad_shape<ShapeL20, MODE>(a, wx, wy, wz, adjoint, adjoint2, out, s);
    case SHAPE_L24:
        if constexpr (MODE == 0) {
            return launch_grad_shape<ShapeL24, 0>(a, wx, wy, wz, adjoint, adjoint2, out, s);
        } else {
            // two passes: the value and weighted adjoints do not fit together
            cudaError_t e = launch_grad_shape<ShapeL24, 2>(a, wx, wy, wz, adjoint, adjoint2, out, s);
            if (e != cudaSuccess)
                return e;
            return launch_grad_shape<ShapeL24, 3>(a, wx, wy, wz, adjoint, adjoint2, out, s);
        }
    case SHAPE_PS:
        return launch_grad_shape<ShapePS, MODE>(a, wx, wy, wz, adjoint, adjoint2, out, s);
    default: return cudaErrorInvalidValue;
    }
}

// launches issued by one launch_moments_tangent / launch_edge_grad call
int grad_kernel_launches(int shape, bool edge)
{
    const int parts = shape == SHAPE_L24 ? GradCfg<ShapeL24>::NPART : 1;
    return edge && shape == SHAPE_L24 ? 2 * parts : parts;
}

cudaError_t launch_moments_tangent(int shape, const EdgeArgs &a, const double *wx,
                                   const double *wy, const double *wz, double *tangent,
                                   cudaStream_t s)
{
    return grad_dispatch<0>(shape, a, wx, wy, wz, nullptr, nullptr, tangent, s);
}

cudaError_t launch_edge_grad(int shape, const EdgeArgs &a, const double *wx, const double *wy,
                             const double *wz, const double *adjoint, const double *adjoint2,
                             double *uv, cudaStream_t s)
{
    return grad_dispatch<1>(shape, a, wx, wy, wz, adjoint, adjoint2, uv, s);
}

// ----------------------------------------------------------------------------
// Dual moment graph.  One block runs 8 atoms at a time (one atom per lane,
// a record stream per 8 lanes, 4 streams per warp, 8 warps) and loops over
// atom groups, keeping the block's moment-coefficient gradient in shared
// memory.  Every shared row holds (value, tangent) pairs per atom:
//   moment rows   (m, D_w m)          adjoint rows   (a, abar)
//   one_row       (1, 0)              one_adj_row    (1, dLdE of the atom)
// and every record is the dual product  acc += c * x * y  with
//   acc.v += c x.v y.v,   acc.t += c (x.t y.v + x.v y.t).
// Forward records give m and D_w m; reverse records (x an adjoint row, y a
// moment row) give a and abar = dLdE a + sum c (abar_id m_o + a_id D_w m_o),
// whose seeds dLdE * coefficient come from one_adj_row.  ENERGY records add
// dLdE m + D_w m of their scalar moment to the block's gradient (the record's
// coefficient names it); reverse END|GLOBAL records store abar of a basic moment.
// ----------------------------------------------------------------------------
template <int STREAMS> struct DagGradGeomT {
    static constexpr int ATOMS = 8;
    static constexpr int LPS = 8;                 // lanes per stream (one atom each)
    static constexpr int SPW = 32 / LPS;          // streams per warp
    static constexpr int WARPS = STREAMS / SPW;
    static constexpr int THREADS = WARPS * 32;
    static constexpr int CH = dag_chunk_rows(STREAMS);
    static constexpr unsigned SLOT_BYTES = CH * SPW * sizeof(DagDevRec);
    static constexpr unsigned ROW_BYTES = ATOMS * 16;
    static constexpr size_t ring_bytes() { return (size_t)WARPS * 2 * SLOT_BYTES; }
};
// ring and row sizes are the same for both stream counts
using DagGradGeom = DagGradGeomT<DAG_STREAMS>;
static_assert(DagGradGeomT<DAG_STREAMS_LARGE>::ring_bytes() == DagGradGeom::ring_bytes(), "");

template <bool FWD, bool GR, int STREAMS>
__device__ __forceinline__ void dag_grad_segment(unsigned rec_addr, const Rows<GR> &rowA, int n,
                                                 double &acc, double &accd, double dlde,
                                                 bool valid, unsigned gmask, int q, double *gsm,
                                                 double *adjoint2, int npad, int atom)
{
    using G = DagGradGeomT<STREAMS>;
    constexpr unsigned REC_STRIDE = G::SPW * sizeof(DagDevRec);
    constexpr unsigned RS = 7;   // log2 of the row size in bytes (8 atoms x 16 B)
    // ENERGY records multiply the zero row by itself; their coefficient holds
    // the index of the scalar moment in the energy list
    auto rare = [&](unsigned outf, double c) {
        if constexpr (FWD) {
            if (outf & DEV_ENERGY) {
                double val = valid ? fma(dlde, acc, accd) : 0.0;
                val += __shfl_xor_sync(gmask, val, 4);
                val += __shfl_xor_sync(gmask, val, 2);
                val += __shfl_xor_sync(gmask, val, 1);
                if (q == 0)
                    gsm[(int)c] += val;
            }
        }
        if (outf & DEV_END) {
            const unsigned out = outf & DEV_OUT_MASK;
            if (!FWD && (outf & DEV_GLOBAL)) {
                if (valid)
                    __stcs(adjoint2 + (size_t)out * npad + atom, accd);   // streamed out
            } else {
                rowA.st(out, acc, accd);
            }
            acc = 0.0;
            accd = 0.0;
        }
    };
    // two-stage schedule as in the value graph (efs.cu dag_segment): the next
    // group's records and operands are loaded before the current group is
    // accumulated
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
            g.x[u] = rowA.ld((w.x & 0xffffu) << RS);
            g.y[u] = rowA.ld((w.x >> 16) << RS);
        }
    };
    auto accumulate = [&](const Grp &g) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const double cx = g.c[u] * g.x[u].x;
            acc = fma(cx, g.y[u].x, acc);
            accd = fma(cx, g.y[u].y, fma(g.c[u] * g.x[u].y, g.y[u].x, accd));
            if (g.of[u])
                rare(g.of[u], g.c[u]);
        }
    };
    int k = 0;
    if (n == G::CH) {
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
        const double2 x = rowA.ld((w.x & 0xffffu) << RS), y = rowA.ld((w.x >> 16) << RS);
        const double c = __hiloint2double((int)w.w, (int)w.z);
        const double cx = c * x.x;
        acc = fma(cx, y.x, acc);
        accd = fma(cx, y.y, fma(c * x.y, y.x, accd));
        if (w.y)
            rare(w.y, c);
    }
}

// GR: rows in the global scratch slice of this block (graphs larger than
// shared memory)
template <bool GR, int STREAMS>
__global__ void __launch_bounds__(DagGradGeomT<STREAMS>::THREADS)
    k_dag_grad(const DagDevRec *__restrict__ recs, const int *__restrict__ phase_row0, int n_fwd,
               int n_rev, int one_row, int zero_row, int one_adj_row, int nrows, int nslot,
               int natoms, int npad, const double *__restrict__ basic,
               const double *__restrict__ tangent, const double *__restrict__ dlde_atom,
               int n_energy, double *__restrict__ adjoint2, double *__restrict__ energy_partials,
               double *__restrict__ gscratch, int *__restrict__ err_flag)
{
    using G = DagGradGeomT<STREAMS>;
    extern __shared__ __align__(128) unsigned char dsm[];
    __shared__ unsigned long long bar[G::WARPS][2];
    __shared__ int ph0[DAG_MAX_PHASES + 1];
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int nph = n_fwd + n_rev;
    unsigned char *ring = dsm + (size_t)warp * 2 * G::SLOT_BYTES;
    double *srows = reinterpret_cast<double *>(dsm + G::ring_bytes());
    double *rows = GR ? gscratch + (size_t)blockIdx.x * nrows * G::ATOMS * 2
                      : srows;                                       // [nrows][ATOMS][2]
    double *gsm = GR ? srows : srows + (size_t)nrows * G::ATOMS * 2;  // [n_energy]
    for (int i = tid; i <= nph; i += blockDim.x)
        ph0[i] = phase_row0[i];
    for (int i = tid; i < n_energy; i += blockDim.x)
        gsm[i] = 0.0;
    if (lane == 0) {
        mbar_init(&bar[warp][0], 1);
        mbar_init(&bar[warp][1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    const int g = lane / G::LPS, q = lane - g * G::LPS;
    const unsigned gmask = 0xffu << (g * G::LPS);
    Rows<GR> rowA;
    if constexpr (GR)
        rowA.base = reinterpret_cast<char *>(rows + 2 * q);
    else
        rowA.base = smem_u32(srows) + q * 16;
    const unsigned ring_u32 = smem_u32(ring) + g * sizeof(DagDevRec);
    auto phase_src = [&](int ph) {
        const int rows_p = ph0[ph + 1] - ph0[ph];
        return recs + (size_t)ph0[ph] * STREAMS + (size_t)warp * rows_p * G::SPW;
    };
    auto nchunks = [&](int ph) { return (ph0[ph + 1] - ph0[ph] + G::CH - 1) / G::CH; };
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
    const int ngroups = (natoms + G::ATOMS - 1) / G::ATOMS;
    for (int grp = blockIdx.x; grp < ngroups; grp += gridDim.x) {
        const int atom0 = grp * G::ATOMS;
        __syncthreads();   // the previous group's rows are no longer read
        for (int i = tid; i < nslot * G::ATOMS; i += blockDim.x) {
            const int sl = i / G::ATOMS, a = i - sl * G::ATOMS;
            const int atom = atom0 + a;
            double v = 0.0, t = 0.0;
            if (atom < natoms) {
                v = __ldcs(basic + (size_t)sl * npad + atom);   // read once: keep the
                t = __ldcs(tangent + (size_t)sl * npad + atom);   // L2 for the row slices
            }
            rows[(size_t)(sl * G::ATOMS + a) * 2] = v;
            rows[(size_t)(sl * G::ATOMS + a) * 2 + 1] = t;
        }
        if (tid < G::ATOMS) {
            const int atom = atom0 + tid;
            const double d = atom < natoms ? dlde_atom[atom] : 0.0;
            rows[(size_t)(one_row * G::ATOMS + tid) * 2] = 1.0;
            rows[(size_t)(one_row * G::ATOMS + tid) * 2 + 1] = 0.0;
            rows[(size_t)(zero_row * G::ATOMS + tid) * 2] = 0.0;
            rows[(size_t)(zero_row * G::ATOMS + tid) * 2 + 1] = 0.0;
            rows[(size_t)(one_adj_row * G::ATOMS + tid) * 2] = 1.0;
            rows[(size_t)(one_adj_row * G::ATOMS + tid) * 2 + 1] = d;
        }
        __syncthreads();
        const int atom = atom0 + q;
        const bool valid = atom < natoms;
        const double dlde = valid ? dlde_atom[atom] : 0.0;
        if (lane == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            iph = 0;
            ic = 0;
            issue_next();
            issue_next();
        }
        double acc = 0.0, accd = 0.0;
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
                    dag_grad_segment<true, GR, STREAMS>(rec_addr, rowA, n, acc, accd, dlde, valid, gmask, q,
                                           gsm, adjoint2, npad, atom);
                else
                    dag_grad_segment<false, GR, STREAMS>(rec_addr, rowA, n, acc, accd, dlde, valid, gmask, q,
                                            gsm, adjoint2, npad, atom);
                __syncwarp();
                if (lane == 0) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue_next();
                }
            }
            __syncthreads();
            acc = 0.0;
            accd = 0.0;
        }
    }
    __syncthreads();
    for (int i = tid; i < n_energy; i += blockDim.x)
        energy_partials[(size_t)blockIdx.x * n_energy + i] = gsm[i];
}

// Device records of the dual graph: warp-major per phase for 4 streams per
// warp, 128-byte rows, reverse-phase operands of the constant one taken from
// one_adj_row (row index plan.nrows), and the energy index as the coefficient
// of ENERGY records.
std::vector<DagDevRec> dag_grad_records(const DagPlan &plan)
{
    using G = DagGradGeom;
    const int one_adj = plan.nrows;
    std::vector<DagDevRec> out(plan.recs.size());
    size_t row0 = 0, o = 0;
    for (size_t ph = 0; ph < plan.phase_rows.size(); ++ph) {
        const int rows_p = plan.phase_rows[ph];
        const bool rev = (int)ph >= plan.n_fwd;
        for (int w = 0; w < plan.streams / G::SPW; ++w)
            for (int r = 0; r < rows_p; ++r)
                for (int s = 0; s < G::SPW; ++s) {
                    const size_t idx = (row0 + r) * plan.streams + w * G::SPW + s;
                    const DagRec &in = plan.recs[idx];
                    DagDevRec d{};
                    int s1 = (int)(in.s12 & 0xffffu), s2 = (int)(in.s12 >> 16);
                    if (rev && s1 == plan.one_row)
                        s1 = one_adj;
                    d.rows = (unsigned)s1 | ((unsigned)s2 << 16);
                    d.c = in.c;
                    const unsigned flags = in.outf >> 16, out_ = in.outf & 0xffffu;
                    unsigned f = 0;
                    if (flags & DAG_END)
                        f |= DEV_END;
                    if (flags & DAG_GLOBAL)
                        f |= DEV_GLOBAL;
                    if (flags & DAG_ENERGY)
                        f |= DEV_ENERGY;
                    d.outf = f ? (f | ((flags & DAG_GLOBAL) ? out_ : out_ * G::ROW_BYTES)) : 0u;
                    const int e = plan.rec_energy.empty() ? -1 : plan.rec_energy[idx];
                    if (flags & DAG_ENERGY)   // product 0 * 0: the coefficient is free
                        d.c = e < 0 ? 0.0 : (double)e;
                    out[o++] = d;
                }
        row0 += rows_p;
    }
    return out;
}

size_t dag_grad_smem_bytes(const DagPlan &plan, bool global_rows)
{
    using G = DagGradGeom;
    return G::ring_bytes() + (global_rows ? 0 : (size_t)(plan.nrows + 1) * G::ROW_BYTES) +
           sizeof(double) * plan.energy_moments.size();
}

size_t dag_grad_scratch_doubles(const DagPlan &plan)
{
    using G = DagGradGeom;
    return plan.grad_global_rows
               ? (size_t)plan.grad_grid * (plan.nrows + 1) * G::ATOMS * 2
               : 0;
}

int dag_grad_grid(const DagPlan &plan, int natoms)
{
    using G = DagGradGeom;
    const int ngroups = (natoms + G::ATOMS - 1) / G::ATOMS;
    if (plan.grad_global_rows)
        return std::max(1, std::min(ngroups, plan.grad_grid));
    int dev = 0, sms = 148, per = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t smem = dag_grad_smem_bytes(plan, false);
    const bool large = plan.streams == DAG_STREAMS_LARGE;
    auto kern = large ? k_dag_grad<false, DAG_STREAMS_LARGE> : k_dag_grad<false, DAG_STREAMS>;
    const int threads = large ? DagGradGeomT<DAG_STREAMS_LARGE>::THREADS : G::THREADS;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
        cudaSuccess)
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, threads, smem);
    per = per < 1 ? 1 : per;
    return std::max(1, std::min(ngroups, sms * per));
}

cudaError_t launch_dag_grad(const DagPlan &plan, const DagDevRec *recs, const int *phase_row0,
                            int grid, int nslot, int natoms, int npad, const double *basic,
                            const double *tangent, const double *dlde_atom, double *adjoint2,
                            double *energy_partials, double *gscratch, int *err_flag,
                            cudaStream_t s)
{
    using G = DagGradGeom;
    if (natoms == 0)
        return cudaSuccess;
    if (plan.n_fwd + plan.n_rev > DAG_MAX_PHASES)
        return cudaErrorInvalidValue;
    const bool gr = plan.grad_global_rows;
    if (gr && (!gscratch || grid > plan.grad_grid))
        return cudaErrorInvalidValue;
    const size_t smem = dag_grad_smem_bytes(plan, gr);
    const bool large = plan.streams == DAG_STREAMS_LARGE;
    if (plan.streams != DAG_STREAMS && !large)
        return cudaErrorInvalidValue;
    auto kern = gr ? (large ? k_dag_grad<true, DAG_STREAMS_LARGE> : k_dag_grad<true, DAG_STREAMS>)
                   : (large ? k_dag_grad<false, DAG_STREAMS_LARGE>
                            : k_dag_grad<false, DAG_STREAMS>);
    const int threads = large ? DagGradGeomT<DAG_STREAMS_LARGE>::THREADS : G::THREADS;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
    if (err == cudaSuccess && gr)   // leave the rest of the SM's memory to L1
        err = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 25);
    if (err != cudaSuccess)
        return err;
    kern<<<grid, threads, smem, s>>>(recs, phase_row0, plan.n_fwd, plan.n_rev, plan.one_row,
                                        plan.zero_row, plan.nrows, plan.nrows + 1, nslot, natoms,
                                        npad, basic, tangent, dlde_atom,
                                        (int)plan.energy_moments.size(), adjoint2,
                                        energy_partials, gscratch, err_flag);
    return cudaGetLastError();
}

} // namespace mtpb
