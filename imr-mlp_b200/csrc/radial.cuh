// radial.cuh -- radial basis functions Q_xi(r) and dQ_xi/dr of every supported
// family, evaluated per edge in xi order.
//
// Reference formulas (paths relative to the reference project):
//   RBChebyshev              basis/basis.cpp:148-164
//   RBChebyCos               basis/basis.cpp:265-280
//   RBChebyshevPoly4         basis/basis.cpp:644-673
//   RBChebyshevPoly5         basis/basis.cpp:776-806
//   RBChebyshevConfigurable  basis/basis.cpp:937-1013 with the cutoffs of
//                            basis/cutoff.cpp and the shifts of basis/xtrans.cpp
// The configurable cutoffs and shifts that the reference writes as value /
// derivative jets are evaluated the same way here (Jet below, first order).
#pragma once

#include "internal.hpp"

namespace mtpb {

struct Jet {
    double v, d;   // value and derivative with respect to r
};
__device__ __forceinline__ Jet jadd(Jet a, Jet b) { return {a.v + b.v, a.d + b.d}; }
__device__ __forceinline__ Jet jsub(Jet a, Jet b) { return {a.v - b.v, a.d - b.d}; }
__device__ __forceinline__ Jet jmul(Jet a, Jet b) { return {a.v * b.v, a.d * b.v + a.v * b.d}; }
__device__ __forceinline__ Jet jscale(double s, Jet a) { return {s * a.v, s * a.d}; }
__device__ __forceinline__ Jet jcos(Jet a)
{
    const double s = sin(a.v), c = cos(a.v);
    return {c, -s * a.d};
}
__device__ __forceinline__ Jet jsin(Jet a)
{
    const double s = sin(a.v), c = cos(a.v);
    return {s, c * a.d};
}
__device__ __forceinline__ Jet jexp(Jet a)
{
    const double e = exp(a.v);
    return {e, e * a.d};
}
__device__ __forceinline__ Jet jtanh(Jet a)
{
    const double t = tanh(a.v);
    return {t, (1.0 - t * t) * a.d};
}
__device__ __forceinline__ Jet jpow2(Jet a) { return jmul(a, a); }
__device__ __forceinline__ Jet jpow3(Jet a) { return jmul(jmul(a, a), a); }
__device__ __forceinline__ Jet jpow4(Jet a) { return jpow2(jpow2(a)); }
__device__ __forceinline__ Jet jpow5(Jet a) { return jmul(jpow4(a), a); }
__device__ __forceinline__ Jet jpow6(Jet a) { return jmul(jpow3(a), jpow3(a)); }
__device__ __forceinline__ Jet jpow7(Jet a) { return jmul(jpow6(a), a); }

constexpr double RB_PI = 3.141592653589793238462643383279502884;

// Envelope fc(r), dfc/dr of the configurable family (cutoff.cpp: the dedicated
// quadratic, cosine and poly5 classes, the others as jets of FormulaCutoff).
static __device__ __noinline__ void radial_cutoff(const PairParams &pp, double r, double &fc,
                                           double &dfc)
{
    switch (pp.cutoff) {
    case CUT_QUADRATIC: {
        const double delta = r - pp.rmax;
        fc = delta * delta;
        dfc = 2.0 * delta;
        return;
    }
    case CUT_COSINE: {
        const double phase = (r - pp.rmin) * pp.cfreq;
        fc = 0.5 * (1.0 + cos(phase));
        dfc = -0.5 * pp.cfreq * sin(phase);
        return;
    }
    case CUT_POLY5: {
        const double x = (r - pp.rmin) * pp.inv_range;
        const double omx = 1.0 - x;
        const double square = omx * omx;
        const double cube = square * omx;
        fc = square * square * (1.0 + (4.0 + pp.b) * x);
        dfc = -cube * (20.0 * x + pp.b * (5.0 * x - 1.0)) * pp.inv_range;
        return;
    }
    default:
        break;
    }
    const Jet radius{r, 1.0}, one{1.0, 0.0};
    const Jet t = jmul(jsub(radius, Jet{pp.rmin, 0.0}), Jet{pp.inv_range, 0.0});
    const Jet q = jsub(one, t);
    Jet out{0.0, 0.0};
    switch (pp.cutoff) {
    case CUT_NORMALIZED_QUADRATIC: out = jpow2(q); break;
    case CUT_COSINE_LEFT: out = jscale(0.5, jadd(one, jcos(jscale(RB_PI / pp.rmax, radius)))); break;
    case CUT_COSINE_UNSCALED: out = jadd(one, jcos(jscale(RB_PI, t))); break;
    case CUT_COSINE_SQUARED: out = jpow2(jadd(one, jcos(jscale(RB_PI, t)))); break;
    case CUT_SINE_SQUARED: out = jpow2(jsin(jscale(RB_PI, t))); break;
    case CUT_POLY3: out = jmul(jpow2(q), jadd(one, jscale(pp.b + 2.0, t))); break;
    case CUT_POLY4: out = jmul(jpow3(q), jadd(one, jscale(pp.b + 3.0, t))); break;
    case CUT_SMOOTHSTEP5:
        out = jadd(jsub(jscale(6.0, jpow5(q)), jscale(15.0, jpow4(q))), jscale(10.0, jpow3(q)));
        break;
    case CUT_SMOOTHSTEP7:
        if (r <= pp.r1) {
            const Jet p = jscale(1.0 / (pp.r1 - pp.rmin), jsub(radius, Jet{pp.rmin, 0.0}));
            out = jsub(jadd(jsub(jscale(35.0, jpow4(p)), jscale(84.0, jpow5(p))),
                            jscale(70.0, jpow6(p))),
                       jscale(20.0, jpow7(p)));
        } else if (r >= pp.r2) {
            const Jet p = jscale(1.0 / (pp.rmax - pp.r2), jsub(radius, Jet{pp.r2, 0.0}));
            out = jadd(jsub(jadd(jsub(one, jscale(35.0, jpow4(p))), jscale(84.0, jpow5(p))),
                            jscale(70.0, jpow6(p))),
                       jscale(20.0, jpow7(p)));
        } else {
            out = one;
        }
        break;
    default: break;
    }
    fc = out.v;
    dfc = out.d;
}

// Coordinate x(r), dx/dr of the configurable family (xtrans.cpp: the
// dedicated linear and exponential classes, the others as jets of
// FormulaShift).  pp.den = expm1(lambda), pp.sden = tanh(scale_lambda).
static __device__ __noinline__ void radial_shift(const PairParams &pp, double r, double &x, double &dx)
{
    switch (pp.shift) {
    case SHIFT_LINEAR:
        x = -1.0 + pp.slope * (r - pp.rmin);
        dx = pp.slope;
        return;
    case SHIFT_EXPONENTIAL:
        if (pp.lambda == 0.0) {
            x = -1.0 + 2.0 * (r - pp.rmin) * pp.inv_range;
            dx = 2.0 * pp.inv_range;
        } else {
            const double exponent = pp.lambda * (pp.rmax - r) * pp.inv_range;
            const double e = exp(exponent);
            x = 1.0 - 2.0 * expm1(exponent) / pp.den;
            dx = 2.0 * pp.lambda * pp.inv_range * e / pp.den;
        }
        return;
    default:
        break;
    }
    const Jet radius{r, 1.0}, one{1.0, 0.0};
    const Jet t = jmul(jsub(radius, Jet{pp.rmin, 0.0}), Jet{pp.inv_range, 0.0});
    Jet out{0.0, 0.0};
    switch (pp.shift) {
    case SHIFT_I2: {
        const Jet k = jmul(jsub(radius, Jet{pp.rmax, 0.0}), Jet{pp.inv_range, 0.0});
        out = jsub(jscale(2.0, jmul(k, k)), one);
        break;
    }
    case SHIFT_EXPONENTIAL_LEFT:
        if (pp.lambda == 0.0) {
            out = jsub(jscale(1.0 / pp.rmax, jscale(2.0, radius)), one);
        } else {
            const Jet exponent = jscale(pp.lambda, jsub(one, jscale(1.0 / pp.rmax, radius)));
            out = jsub(one, jscale(2.0 / pp.den, jsub(jexp(exponent), one)));
        }
        break;
    case SHIFT_EXPONENTIAL_TANH: {
        Jet shifted;
        if (pp.lambda == 0.0)
            shifted = jsub(jscale(2.0, t), one);
        else
            shifted = jsub(one, jscale(2.0 / pp.den,
                                       jsub(jexp(jscale(pp.lambda, jsub(one, t))), one)));
        out = pp.scale_lambda == 0.0
                  ? shifted
                  : jscale(1.0 / pp.sden, jtanh(jscale(pp.scale_lambda, shifted)));
        break;
    }
    default: break;
    }
    x = out.v;
    dx = out.d;
}

// RBChebyshev alone (basis.cpp:148-164): the kernels of models without other
// families use this.
template <class Emit>
__device__ __forceinline__ void radial_chebyshev(const PairParams &pp, double s, int R, double r,
                                                 Emit &&emit)
{
    const double ksi = (2.0 * r - pp.pu) / pp.su;
    const double ru = r - pp.rmax;
    double q0 = s * (ru * ru), d0 = s * (2.0 * ru);
    emit(0, q0, d0);
    if (R > 1) {
        double q1 = s * (ksi * ru * ru);
        double d1 = s * (pp.mult * ru * ru + 2.0 * ksi * ru);
        emit(1, q1, d1);
        for (int xi = 2; xi < R; ++xi) {
            const double q2 = 2.0 * ksi * q1 - q0;
            const double d2 = 2.0 * (pp.mult * q1 + ksi * d1) - d0;
            emit(xi, q2, d2);
            q0 = q1;
            q1 = q2;
            d0 = d1;
            d1 = d2;
        }
    }
}

// Coordinate and envelope of the families other than RBChebyshev, out of
// line so that their transcendental functions stay out of the moment kernels'
// instruction stream.  mode 0: the family vanishes at r (below min_dist for
// Poly4, Poly5 and the configurable family); 1: Chebyshev series in x times
// the envelope, carried through the recurrence (basis.cpp calc_der of
// RBChebyCos, Poly4, Poly5); 2: configurable, polynomials first, then scaled
// by the envelope (basis.cpp:937-1013).
struct RadialStart {
    int mode;
    double x, dx, fc, dfc;
};
static __device__ __noinline__ RadialStart radial_start(const PairParams &pp, double r)
{
    RadialStart st{0, 0.0, 0.0, 0.0, 0.0};
    if (pp.type != RB_CHEBY_COS && r < pp.rmin)
        return st;
    if (pp.type == RB_CONFIGURABLE) {
        radial_shift(pp, r, st.x, st.dx);
        radial_cutoff(pp, r, st.fc, st.dfc);
        st.mode = 2;
        return st;
    }
    st.mode = 1;
    st.x = (2.0 * r - pp.pu) / pp.su;
    st.dx = pp.mult;
    if (pp.type == RB_CHEBY_COS) {
        st.fc = 0.5 * (1.0 + cos(r * pp.irpi));
        st.dfc = -0.5 * pp.irpi * sin(r * pp.irpi);
        return st;
    }
    // Poly4 / Poly5 envelopes in t = (r - min) / (max - min)
    const double t = (r - pp.rmin) / pp.su;
    const double dtdr = 1.0 / pp.su;
    const double vx = 1.0 - t;
    const double vxx = vx * vx;
    const double vxxx = vxx * vx;
    if (pp.type == RB_CHEBY_POLY5) {
        st.fc = vxx * vxx * (1 + (4 + pp.b) * t);
        st.dfc = -vxxx * (20 * t + pp.b * (5 * t - 1)) * dtdr;
    } else {
        st.fc = vxxx * (1 + (3 + pp.b) * t);
        st.dfc = vxx * (pp.b * (1. - 4.0 * t) - 12.0 * t) * dtdr;
    }
    return st;
}

// Q_xi(r) and dQ_xi/dr for xi = 0..R-1 of the pair's family, in order, passed
// to emit(xi, q, dq); s is the model's scaling.  Returns false (and emits
// nothing: every Q is zero) where the family vanishes.  Callers have already
// skipped r > max_dist.
template <class Emit>
__device__ __forceinline__ bool radial_basis(const PairParams &pp, double s, int R, double r,
                                             Emit &&emit)
{
    double x, dx, q0, d0, q1, d1;
    if (pp.type == RB_POLYB || pp.type == RB_POLYB_COS) {
        // powers s (max - r)^(xi + first) and their r-derivatives, times the
        // CosineLeft envelope for RBPolyBCos (runtime/mtp/radial_basis.h:
        // 223-290); the orthogonalisation matrix and normalisations are folded
        // into the coefficients at upload
        const int first = pp.type == RB_POLYB ? 3 : 2;
        double fc = 1.0, dfc = 0.0;
        if (pp.type == RB_POLYB_COS)
            radial_cutoff(pp, r, fc, dfc);
        const double delta = pp.rmax - r;
        double prev = s * delta;   // s delta^(first - 1)
        if (first == 3)
            prev *= delta;
        for (int xi = 0; xi < R; ++xi) {
            const double q = prev * delta;
            const double dq = -(double)(xi + first) * prev;
            emit(xi, q * fc, dq * fc + q * dfc);
            prev = q;
        }
        return true;
    }
    if (pp.type == RB_CHEBYSHEV) {
        x = (2.0 * r - pp.pu) / pp.su;
        dx = pp.mult;
        const double ru = r - pp.rmax;
        q0 = s * (ru * ru);
        d0 = s * (2.0 * ru);
        q1 = s * (x * ru * ru);
        d1 = s * (dx * ru * ru + 2.0 * x * ru);
    } else {
        const RadialStart st = radial_start(pp, r);
        if (st.mode == 0)
            return false;
        x = st.x;
        dx = st.dx;
        if (st.mode == 2) {
            // T_i(x) and their r-derivatives, then Q_i = s raw_i fc with
            // raw_i = T_i, or 1 - T_(i+1) for the one-minus-Chebyshev type
            double t0 = 1.0, g0 = 0.0, t1 = x, g1 = dx;
            for (int i = 0; i < R; ++i) {
                const double raw = pp.flipped ? 1.0 - t1 : t0;
                const double rawd = pp.flipped ? -g1 : g0;
                emit(i, s * raw * st.fc, s * (rawd * st.fc + raw * st.dfc));
                const double t2 = 2.0 * x * t1 - t0;
                const double g2 = 2.0 * (dx * t1 + x * g1) - g0;
                t0 = t1;
                t1 = t2;
                g0 = g1;
                g1 = g2;
            }
            return true;
        }
        q0 = s * st.fc;
        d0 = s * st.dfc;
        q1 = s * (x * st.fc);
        d1 = s * (dx * st.fc + x * st.dfc);
    }
    emit(0, q0, d0);
    if (R > 1) {
        emit(1, q1, d1);
        for (int xi = 2; xi < R; ++xi) {
            const double q2 = 2.0 * x * q1 - q0;
            const double d2 = 2.0 * (dx * q1 + x * d1) - d0;
            emit(xi, q2, d2);
            q0 = q1;
            q1 = q2;
            d0 = d1;
            d1 = d2;
        }
    }
    return true;
}

} // namespace mtpb
