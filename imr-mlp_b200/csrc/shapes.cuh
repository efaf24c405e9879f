// shapes.cuh -- compile-time layout of the basic moments for the moment
// kernels.
//
// A Shapeev-style MTP basis (potentials/potential_mtp.cpp:578-606 reads it
// from alpha_index_basic) is a union of complete moment tensors
// M_{mu,nu} = sum_j f_mu(r_j) rhat_j^{(x) nu}: for radial channel mu every
// monomial x^a y^b z^c with a+b+c = nu <= numax(mu) is present.  Shape<numax
// ...> fixes numax per channel at compile time so that each warp's share of
// the work unrolls into straight-line FP64 code with register-resident
// accumulators.
//
// Monomials are organised in "chains": for a fixed (b, c) the chain runs over
// a = 0 .. NU-b-c and every monomial is the previous one times xhat.  A chain
// owns, for each a, the accumulators of the channels mu with
// numax(mu) >= a+b+c.  Kernel slot numbering is chain-major, then a, then mu.
#pragma once

#include <cstdint>
#include <utility>

namespace mtpb {

template <int N> struct IArr {
    int v[N > 0 ? N : 1];
    constexpr int operator[](int i) const { return v[i]; }
    constexpr int &operator[](int i) { return v[i]; }
};

template <int... NUMAX> struct Shape {
    static constexpr int NMU = sizeof...(NUMAX);
    static constexpr IArr<NMU> numax{{NUMAX...}};
    static constexpr int max_nu()
    {
        int m = 0;
        for (int i = 0; i < NMU; ++i)
            m = numax[i] > m ? numax[i] : m;
        return m;
    }
    static constexpr int NU = max_nu();
    // number of channels carrying degree nu
    static constexpr int cnt(int nu)
    {
        int c = 0;
        for (int i = 0; i < NMU; ++i)
            c += (numax[i] >= nu) ? 1 : 0;
        return c;
    }
    // channel list of degree nu is not necessarily a prefix of 0..NMU-1;
    // k-th channel carrying degree nu:
    static constexpr int chan(int nu, int k)
    {
        for (int i = 0; i < NMU; ++i)
            if (numax[i] >= nu) {
                if (k == 0)
                    return i;
                --k;
            }
        return -1;
    }
    static constexpr int NCH = (NU + 1) * (NU + 2) / 2;
    struct Chains {
        IArr<NCH> b, c, len, nacc, slot0;
        int nslot;
    };
    static constexpr Chains make_chains()
    {
        Chains t{};
        int k = 0, slot = 0;
        for (int s = 0; s <= NU; ++s)
            for (int b = s; b >= 0; --b) {
                int c = s - b;
                t.b[k] = b;
                t.c[k] = c;
                t.len[k] = NU - s + 1;
                int na = 0;
                for (int a = 0; a <= NU - s; ++a)
                    na += cnt(a + s);
                t.nacc[k] = na;
                t.slot0[k] = slot;
                slot += na;
                ++k;
            }
        t.nslot = slot;
        return t;
    }
    static constexpr Chains chains = make_chains();
    static constexpr int NSLOT = chains.nslot;
    // slot of channel mu, monomial (a, b, c); -1 when absent
    static constexpr int slot_of(int mu, int a, int b, int c)
    {
        int s = b + c;
        if (s > NU || a > NU - s || mu >= NMU || numax[mu] < a + s)
            return -1;
        for (int k = 0; k < NCH; ++k)
            if (chains.b[k] == b && chains.c[k] == c) {
                int slot = chains.slot0[k];
                for (int aa = 0; aa < a; ++aa)
                    slot += cnt(aa + s);
                for (int q = 0; q < cnt(a + s); ++q)
                    if (chan(a + s, q) == mu)
                        return slot + q;
            }
        return -1;
    }
};

// Per-chain cost model (FP64 instructions per edge) used to balance warps:
// forward = one FMA per accumulator + one multiply per monomial; reverse = two
// FMAs per accumulator + three per monomial + the chain epilogue.
template <class S> constexpr int chain_cost(int k)
{
    return 3 * S::chains.nacc[k] + 4 * S::chains.len[k] + 8;
}

// Greedy longest-processing-time assignment of chains to NW warps.
template <class S, int NW> struct Partition {
    struct Table {
        IArr<NW> count;       // chains per warp
        IArr<NW> nacc;        // accumulators per warp
        IArr<NW> maxb, maxc;  // highest y / z power a warp needs
        IArr<NW * S::NCH> list;   // chain ids, warp-major
        IArr<NW * S::NCH> acc0;   // accumulator base of each listed chain
        IArr<S::NCH> warp_of;
    };
    static constexpr Table make()
    {
        Table t{};
        int order[S::NCH] = {};
        for (int k = 0; k < S::NCH; ++k)
            order[k] = k;
        // sort by cost, descending (selection sort: constexpr friendly)
        for (int i = 0; i < S::NCH; ++i) {
            int best = i;
            for (int j = i + 1; j < S::NCH; ++j)
                if (chain_cost<S>(order[j]) > chain_cost<S>(order[best]))
                    best = j;
            int tmp = order[i];
            order[i] = order[best];
            order[best] = tmp;
        }
        int load[NW] = {};
        for (int w = 0; w < NW; ++w) {
            t.count[w] = 0;
            t.nacc[w] = 0;
            t.maxb[w] = 0;
            t.maxc[w] = 0;
        }
        for (int i = 0; i < S::NCH; ++i) {
            int k = order[i];
            int w = 0;
            for (int q = 1; q < NW; ++q)
                if (load[q] < load[w])
                    w = q;
            load[w] += chain_cost<S>(k);
            t.warp_of[k] = w;
        }
        // list chains per warp in chain order (keeps powers monotone)
        for (int w = 0; w < NW; ++w)
            for (int k = 0; k < S::NCH; ++k)
                if (t.warp_of[k] == w) {
                    int idx = w * S::NCH + t.count[w];
                    t.list[idx] = k;
                    t.acc0[idx] = t.nacc[w];
                    t.nacc[w] += S::chains.nacc[k];
                    if (S::chains.b[k] > t.maxb[w])
                        t.maxb[w] = S::chains.b[k];
                    if (S::chains.c[k] > t.maxc[w])
                        t.maxc[w] = S::chains.c[k];
                    t.count[w]++;
                }
        return t;
    }
    static constexpr Table table = make();
};

// ---- compile-time loop helper -------------------------------------------
template <class F, int... Is>
__host__ __device__ __forceinline__ void static_for_impl(F &&f, std::integer_sequence<int, Is...>)
{
    (f(std::integral_constant<int, Is>{}), ...);
}
template <int N, class F> __host__ __device__ __forceinline__ void static_for(F &&f)
{
    if constexpr (N > 0)
        static_for_impl(f, std::make_integer_sequence<int, N>{});
}

// ---- instantiated shapes -------------------------------------------------
// Level 2/6-style small bases, the shipped Shapeev level 16 and 20 templates
// (numax 6,4,2,0 and 8,6,4,2,0), the level-24 family (10,8,6,4,2,0) and the
// deep ps1 family (4,3,3,2,2,1).
using ShapeS1 = Shape<1>;
using ShapeS2 = Shape<2, 0>;
using ShapeL16 = Shape<6, 4, 2, 0>;
using ShapeL20 = Shape<8, 6, 4, 2, 0>;
using ShapeL24 = Shape<10, 8, 6, 4, 2, 0>;
using ShapePS = Shape<4, 3, 3, 2, 2, 1>;

} // namespace mtpb
