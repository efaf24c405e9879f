/*
 * mtp_oracle.c -- CPU restatement of the reference MTP hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see mtp_oracle.h).  Compiled with
 * -ffp-contract=off so that every expression rounds exactly as written; the
 * comments name the reference lines each block follows.
 */
#include "mtp_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* Cell algebra in Eigen's evaluation order (fixed-size 3x3, no FMA).         */
/* ------------------------------------------------------------------------ */

/* Eigen compute_inverse<3x3>: cofactors of column 0, det = (c0*m00 + c1*m10)
 * + c2*m20, inverse(i,j) = cofactor(j,i) * (1/det).  Used by
 * base/neighborhoods_base.h:118 (atom.cell_.inverse()). */
static double cofactor3(const double *m, int i, int j)
{
    int i1 = (i + 1) % 3, i2 = (i + 2) % 3, j1 = (j + 1) % 3, j2 = (j + 2) % 3;
    return m[i1 * 3 + j1] * m[i2 * 3 + j2] - m[i1 * 3 + j2] * m[i2 * 3 + j1];
}

static void inverse3(const double *m, double *inv)
{
    double c0 = cofactor3(m, 0, 0), c1 = cofactor3(m, 1, 0), c2 = cofactor3(m, 2, 0);
    double det = (c0 * m[0] + c1 * m[3]) + c2 * m[6];
    double invdet = 1.0 / det;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j)
            inv[i * 3 + j] = cofactor3(m, j, i) * invdet;
}

/* Row vector times matrix: component d = (p0*M(0,d) + p1*M(1,d)) + p2*M(2,d). */
static void rowvec_mat(const double *p, const double *mat, double *out)
{
    double r[3];
    for (int d = 0; d < 3; ++d)
        r[d] = (p[0] * mat[0 * 3 + d] + p[1] * mat[1 * 3 + d]) + p[2] * mat[2 * 3 + d];
    out[0] = r[0];
    out[1] = r[1];
    out[2] = r[2];
}

void oracle_wrap_positions(const double *cell, const int *pbc, int n, const double *pos,
                           double *wrapped)
{
    /* base/neighborhoods_base.h:113-126: only fully periodic cells wrap. */
    int full = pbc[0] && pbc[1] && pbc[2];
    if (!full) {
        memcpy(wrapped, pos, sizeof(double) * 3 * (size_t)n);
        return;
    }
    double inv[9];
    inverse3(cell, inv);
    for (int i = 0; i < n; ++i) {
        double f[3];
        rowvec_mat(pos + 3 * i, inv, f);
        for (int d = 0; d < 3; ++d)
            f[d] -= floor(f[d]);
        rowvec_mat(f, cell, wrapped + 3 * i);
    }
}

/* Translation of a periodic image, base/neighborhoods_base.h:36-78: the basis
 * holds the periodic cell rows as columns, sorted by squared length (ties in
 * axis order); translation = basis * image with Eigen's fixed 3x3
 * matrix-vector order: rows 0 and 1 accumulate (t0 + t1) + t2, row 2 uses
 * t0 + (t1 + t2). */
typedef struct image_basis {
    int dims;
    int axes[3];     /* periodic cell rows, sorted */
    double B[3][3];  /* B[r][k] = cell(axes[k], r) */
} image_basis;

static double row_sqnorm(const double *cell, int a)
{
    const double *r = cell + 3 * a;
    return r[0] * r[0] + (r[1] * r[1] + r[2] * r[2]);
}

static void make_image_basis(const double *cell, const int *pbc, image_basis *ib)
{
    int axes[3] = {0, 1, 2};
    /* insertion sort (stable), as libstdc++ std::sort on three elements */
    for (int i = 1; i < 3; ++i) {
        int v = axes[i];
        int j = i;
        while (j > 0 && row_sqnorm(cell, v) < row_sqnorm(cell, axes[j - 1])) {
            axes[j] = axes[j - 1];
            --j;
        }
        axes[j] = v;
    }
    ib->dims = 0;
    memset(ib->B, 0, sizeof(ib->B));
    for (int k = 0; k < 3; ++k) {
        int a = axes[k];
        if (pbc[a]) {
            ib->axes[ib->dims] = a;
            for (int r = 0; r < 3; ++r)
                ib->B[r][ib->dims] = cell[3 * a + r];
            ib->dims++;
        }
    }
}

/* shift[a] is the integer image along cell row a; image[k] = shift[axes[k]]. */
static void image_translation(const image_basis *ib, const int *shift, double *t)
{
    double img[3] = {0.0, 0.0, 0.0};
    for (int k = 0; k < ib->dims; ++k)
        img[k] = (double)shift[ib->axes[k]];
    for (int r = 0; r < 2; ++r)
        t[r] = (ib->B[r][0] * img[0] + ib->B[r][1] * img[1]) + ib->B[r][2] * img[2];
    t[2] = ib->B[2][0] * img[0] + (ib->B[2][1] * img[1] + ib->B[2][2] * img[2]);
}

/* ------------------------------------------------------------------------ */
/* Neighbour lists                                                           */
/* ------------------------------------------------------------------------ */

typedef struct edge_rec {
    int center, nbr;
    double r[3];
} edge_rec;

static int edge_cmp(const void *pa, const void *pb)
{
    const edge_rec *a = (const edge_rec *)pa, *b = (const edge_rec *)pb;
    if (a->center != b->center)
        return a->center < b->center ? -1 : 1;
    if (a->nbr != b->nbr)
        return a->nbr < b->nbr ? -1 : 1;
    for (int d = 0; d < 3; ++d)
        if (a->r[d] != b->r[d])
            return a->r[d] < b->r[d] ? -1 : 1;
    return 0;
}

long oracle_neighbors(const double *cell, const int *pbc, int n, const double *pos,
                      double cutoff, int *offsets, int *nbr, double *rij)
{
    if (n < 0 || cutoff <= 0)
        return -1;
    if (n == 0) {
        if (offsets)
            offsets[0] = 0;
        return 0;
    }
    double *w = (double *)malloc(sizeof(double) * 3 * (size_t)n);
    if (!w)
        return -1;
    oracle_wrap_positions(cell, pbc, n, pos, w);

    image_basis ib;
    make_image_basis(cell, pbc, &ib);

    /* image range per cell row: every image that can hold a point within the
     * cutoff of an original (the reference's QR bound keeps a superset of
     * these; points farther away never pass the distance test). */
    int smax[3] = {0, 0, 0};
    {
        double lo[3], hi[3];
        for (int d = 0; d < 3; ++d)
            lo[d] = hi[d] = w[d];
        for (int i = 1; i < n; ++i)
            for (int d = 0; d < 3; ++d) {
                if (w[3 * i + d] < lo[d])
                    lo[d] = w[3 * i + d];
                if (w[3 * i + d] > hi[d])
                    hi[d] = w[3 * i + d];
            }
        double ext = 0;
        for (int d = 0; d < 3; ++d)
            ext += (hi[d] - lo[d] + cutoff) * (hi[d] - lo[d] + cutoff);
        ext = sqrt(ext);
        /* perpendicular width of each lattice plane family: V / |a x b| */
        const double *a0 = cell, *a1 = cell + 3, *a2 = cell + 6;
        double cr[3][3];
        const double *rows[3] = {a0, a1, a2};
        for (int a = 0; a < 3; ++a) {
            const double *u = rows[(a + 1) % 3], *v = rows[(a + 2) % 3];
            cr[a][0] = u[1] * v[2] - u[2] * v[1];
            cr[a][1] = u[2] * v[0] - u[0] * v[2];
            cr[a][2] = u[0] * v[1] - u[1] * v[0];
        }
        double vol = fabs(a0[0] * cr[0][0] + a0[1] * cr[0][1] + a0[2] * cr[0][2]);
        for (int a = 0; a < 3; ++a) {
            if (!pbc[a])
                continue;
            double nrm = sqrt(cr[a][0] * cr[a][0] + cr[a][1] * cr[a][1] + cr[a][2] * cr[a][2]);
            double width = vol / nrm;
            smax[a] = (int)ceil(ext / width) + 1;
        }
    }

    const double cutsq = cutoff * cutoff;
    size_t cap = 1024, cnt = 0;
    edge_rec *edges = (edge_rec *)malloc(sizeof(edge_rec) * cap);
    if (!edges) {
        free(w);
        return -1;
    }
#define PUSH_EDGE(C, N, X, Y, Z)                                                                   \
    do {                                                                                           \
        if (cnt == cap) {                                                                          \
            cap *= 2;                                                                              \
            edge_rec *ne = (edge_rec *)realloc(edges, sizeof(edge_rec) * cap);                     \
            if (!ne) {                                                                             \
                free(edges);                                                                       \
                free(w);                                                                           \
                return -1;                                                                         \
            }                                                                                      \
            edges = ne;                                                                            \
        }                                                                                          \
        edges[cnt].center = (C);                                                                   \
        edges[cnt].nbr = (N);                                                                      \
        edges[cnt].r[0] = (X);                                                                     \
        edges[cnt].r[1] = (Y);                                                                     \
        edges[cnt].r[2] = (Z);                                                                     \
        ++cnt;                                                                                     \
    } while (0)

    int s[3];
    for (s[0] = -smax[0]; s[0] <= smax[0]; ++s[0])
        for (s[1] = -smax[1]; s[1] <= smax[1]; ++s[1])
            for (s[2] = -smax[2]; s[2] <= smax[2]; ++s[2]) {
                int zero = (s[0] == 0 && s[1] == 0 && s[2] == 0);
                double t[3];
                image_translation(&ib, s, t);
                for (int o = 0; o < n; ++o) {
                    /* ghost point: pos[o] + translation (neighborhoods_base.h:82) */
                    double p[3];
                    if (zero) {
                        p[0] = w[3 * o];
                        p[1] = w[3 * o + 1];
                        p[2] = w[3 * o + 2];
                    } else {
                        p[0] = w[3 * o] + t[0];
                        p[1] = w[3 * o + 1] + t[1];
                        p[2] = w[3 * o + 2] + t[2];
                    }
                    /* neighborhood.cpp:113-134: center i <= orig(j), i != j */
                    for (int i = 0; i <= o; ++i) {
                        if (zero && i == o)
                            continue;
                        double r0 = p[0] - w[3 * i], r1 = p[1] - w[3 * i + 1],
                               r2 = p[2] - w[3 * i + 2];
                        double dsq = r0 * r0 + r1 * r1 + r2 * r2;
                        if (dsq < cutsq) {
                            PUSH_EDGE(i, o, r0, r1, r2);
                            if (i != o)
                                PUSH_EDGE(o, i, -r0, -r1, -r2);
                        }
                    }
                }
            }
#undef PUSH_EDGE
    qsort(edges, cnt, sizeof(edge_rec), edge_cmp);
    if (offsets) {
        size_t e = 0;
        for (int i = 0; i < n; ++i) {
            offsets[i] = (int)e;
            while (e < cnt && edges[e].center == i) {
                if (nbr)
                    nbr[e] = edges[e].nbr;
                if (rij) {
                    rij[3 * e] = edges[e].r[0];
                    rij[3 * e + 1] = edges[e].r[1];
                    rij[3 * e + 2] = edges[e].r[2];
                }
                ++e;
            }
        }
        offsets[n] = (int)e;
    }
    free(edges);
    free(w);
    return (long)cnt;
}

/* ------------------------------------------------------------------------ */
/* Model helpers                                                             */
/* ------------------------------------------------------------------------ */

typedef struct site_ws {
    int nb, M, T, S, K, mu, R, maxmu, maxnu; /* maxnu = max(a+b+c)+1 */
    double *mv, *sed, *rv, *rd, *vm, *dm, *dp, *cp; /* cp: [(maxnu+1)][3] */
    double *mj;                                     /* [nb][nmax][3] */
    int nmax;
    /* gradient workspace */
    double *mjc, *mjcc; /* [nb][K][mu*R] */
    double *dldm, *dlds;
    double *w; /* combination weights [nmax][3] */
} site_ws;

static int model_maxmu(const oracle_model *m)
{
    int mx = 0;
    for (int i = 0; i < m->alpha_index_basic_count; ++i)
        if (m->alpha_index_basic[4 * i] > mx)
            mx = m->alpha_index_basic[4 * i];
    return mx + 1;
}

static int model_maxnu(const oracle_model *m)
{
    int mx = 0;
    for (int i = 0; i < m->alpha_index_basic_count; ++i) {
        const int *b = m->alpha_index_basic + 4 * i;
        int nu = b[1] + b[2] + b[3];
        if (nu > mx)
            mx = nu;
    }
    return mx + 1;
}

static void ws_free(site_ws *ws)
{
    free(ws->mv);
    free(ws->sed);
    free(ws->rv);
    free(ws->rd);
    free(ws->vm);
    free(ws->dm);
    free(ws->dp);
    free(ws->cp);
    free(ws->mj);
    free(ws->mjc);
    free(ws->mjcc);
    free(ws->dldm);
    free(ws->dlds);
    free(ws->w);
    memset(ws, 0, sizeof(*ws));
}

static int ws_init(site_ws *ws, const oracle_model *m, int nmax, int grad)
{
    memset(ws, 0, sizeof(*ws));
    ws->nb = m->alpha_index_basic_count;
    ws->M = m->alpha_moments_count;
    ws->T = m->alpha_index_times_count;
    ws->S = m->alpha_scalar_moments;
    ws->K = m->species_count;
    ws->mu = m->radial_func_count;
    ws->R = m->rb_size;
    ws->maxmu = model_maxmu(m);
    ws->maxnu = model_maxnu(m);
    ws->nmax = nmax < 1 ? 1 : nmax;
    ws->mv = (double *)calloc((size_t)ws->M, sizeof(double));
    ws->sed = (double *)calloc((size_t)ws->M, sizeof(double));
    ws->rv = (double *)calloc((size_t)ws->R, sizeof(double));
    ws->rd = (double *)calloc((size_t)ws->R, sizeof(double));
    ws->vm = (double *)calloc((size_t)ws->mu + 1, sizeof(double));
    ws->dm = (double *)calloc((size_t)ws->mu + 1, sizeof(double));
    ws->dp = (double *)calloc((size_t)ws->maxnu + 1, sizeof(double));
    ws->cp = (double *)calloc(3 * ((size_t)ws->maxnu + 2), sizeof(double));
    ws->mj = (double *)calloc((size_t)ws->nb * ws->nmax * 3, sizeof(double));
    if (!ws->mv || !ws->sed || !ws->rv || !ws->rd || !ws->vm || !ws->dm || !ws->dp || !ws->cp ||
        !ws->mj) {
        ws_free(ws);
        return -1;
    }
    if (grad) {
        size_t g = (size_t)ws->nb * ws->K * ws->mu * ws->R;
        ws->mjc = (double *)calloc(g, sizeof(double));
        ws->mjcc = (double *)calloc(g, sizeof(double));
        ws->dldm = (double *)calloc((size_t)ws->M, sizeof(double));
        ws->dlds = (double *)calloc((size_t)ws->M, sizeof(double));
        ws->w = (double *)calloc((size_t)ws->nmax * 3, sizeof(double));
        if (!ws->mjc || !ws->mjcc || !ws->dldm || !ws->dlds || !ws->w) {
            ws_free(ws);
            return -1;
        }
    }
    /* coords_powers rows 0 and 1 are constant: cp(0,:) = 0, cp(1,:) = 1 */
    for (int a = 0; a < 3; ++a) {
        ws->cp[0 * 3 + a] = 0.0;
        ws->cp[1 * 3 + a] = 1.0;
    }
    return 0;
}

static double pair_min(const oracle_model *m, int pair)
{
    return m->radial_basis_split ? m->min_dist[pair] : m->min_dist[0];
}
static double pair_max(const oracle_model *m, int pair)
{
    return m->radial_basis_split ? m->max_dist[pair] : m->max_dist[0];
}

/* RBasis_Chebyshev::calc_der, basis/basis.cpp:119-164 (mult, su, pu from
 * setup(); the value recurrence and the derivative recurrence). */
static void cheb_calc_der(double rmin, double rmax, double scaling, int R, double r, double *val,
                          double *der)
{
    double mult = 2.0 / (rmax - rmin);
    double su = rmax - rmin;
    double pu = rmax + rmin;
    double ksi = (2 * r - pu) / su;
    double ru = r - rmax;
    val[0] = scaling * (1 * ru * ru);
    der[0] = scaling * (0 * ru * ru + 2 * ru);
    if (R == 1)
        return;
    val[1] = scaling * (ksi * ru * ru);
    der[1] = scaling * (mult * ru * ru + 2 * ksi * ru);
    for (int i = 2; i < R; i++) {
        val[i] = 2 * ksi * val[i - 1] - val[i - 2];
        der[i] = 2 * (mult * val[i - 1] + ksi * der[i - 1]) - der[i - 2];
    }
}

/* ---- other radial families ---------------------------------------------
 * Value / derivative jets of basis/cutoff.cpp FormulaCutoff and
 * basis/xtrans.cpp FormulaShift (their Jet2 arithmetic, first order). */
typedef struct {
    double v, d;
} jet;
static jet j_add(jet a, jet b) { jet r = {a.v + b.v, a.d + b.d}; return r; }
static jet j_sub(jet a, jet b) { jet r = {a.v - b.v, a.d - b.d}; return r; }
static jet j_mul(jet a, jet b) { jet r = {a.v * b.v, a.d * b.v + a.v * b.d}; return r; }
static jet j_sc(double s, jet a) { jet r = {s * a.v, s * a.d}; return r; }
static jet j_div(jet a, double s) { return j_sc(1.0 / s, a); }
static jet j_cos(jet a) { jet r = {cos(a.v), -sin(a.v) * a.d}; return r; }
static jet j_sin(jet a) { jet r = {sin(a.v), cos(a.v) * a.d}; return r; }
static jet j_exp(jet a) { double e = exp(a.v); jet r = {e, e * a.d}; return r; }
static jet j_tanh(jet a)
{
    double t = tanh(a.v);
    jet r = {t, (1.0 - t * t) * a.d};
    return r;
}
static jet j_pow2(jet a) { return j_mul(a, a); }
static jet j_pow3(jet a) { return j_mul(j_mul(a, a), a); }
static jet j_pow4(jet a) { return j_pow2(j_pow2(a)); }
static jet j_pow5(jet a) { return j_mul(j_pow4(a), a); }
static jet j_pow6(jet a) { return j_mul(j_pow3(a), j_pow3(a)); }
static jet j_pow7(jet a) { return j_mul(j_pow6(a), a); }
static const double ORACLE_PI = 3.141592653589793238462643383279502884;

/* AnyCutoff::compute_der of basis/cutoff.cpp (QuadraticCutoff, CosineCutoff,
 * Poly5Cutoff, FormulaCutoff::evaluate). */
static void cutoff_der(const oracle_radial_family *f, double lo, double hi, double r, double *val,
                       double *der)
{
    const double inv_range = 1.0 / (hi - lo);
    if (f->cutoff_type == 0) { /* quadratic */
        double delta = r - hi;
        *val = delta * delta;
        *der = 2.0 * delta;
        return;
    }
    if (f->cutoff_type == 1) { /* cosine */
        double freq = ORACLE_PI / (hi - lo);
        double phase = (r - lo) * freq;
        *val = 0.5 * (1.0 + cos(phase));
        *der = -0.5 * freq * sin(phase);
        return;
    }
    if (f->cutoff_type == 2) { /* poly5 */
        double x = (r - lo) * inv_range;
        double omx = 1.0 - x;
        double square = omx * omx;
        double cube = square * omx;
        *val = square * square * (1.0 + (4.0 + f->b) * x);
        *der = -cube * (20.0 * x + f->b * (5.0 * x - 1.0)) * inv_range;
        return;
    }
    jet radius = {r, 1.0}, one = {1.0, 0.0}, lo_j = {lo, 0.0}, ir = {inv_range, 0.0};
    jet t = j_mul(j_sub(radius, lo_j), ir);
    jet q = j_sub(one, t);
    jet out = {0.0, 0.0};
    switch (f->cutoff_type) {
    case 3: out = j_pow2(q); break;
    case 4: out = j_sc(0.5, j_add(one, j_cos(j_sc(ORACLE_PI / hi, radius)))); break;
    case 5: out = j_add(one, j_cos(j_sc(ORACLE_PI, t))); break;
    case 6: out = j_pow2(j_add(one, j_cos(j_sc(ORACLE_PI, t)))); break;
    case 7: out = j_pow2(j_sin(j_sc(ORACLE_PI, t))); break;
    case 8: out = j_mul(j_pow2(q), j_add(one, j_sc(f->b + 2.0, t))); break;
    case 9: out = j_mul(j_pow3(q), j_add(one, j_sc(f->b + 3.0, t))); break;
    case 10:
        out = j_add(j_sub(j_sc(6.0, j_pow5(q)), j_sc(15.0, j_pow4(q))), j_sc(10.0, j_pow3(q)));
        break;
    case 11:
        if (r <= f->r1) {
            jet p = j_div(j_sub(radius, lo_j), f->r1 - lo);
            out = j_sub(j_add(j_sub(j_sc(35.0, j_pow4(p)), j_sc(84.0, j_pow5(p))),
                              j_sc(70.0, j_pow6(p))),
                        j_sc(20.0, j_pow7(p)));
        } else if (r >= f->r2) {
            jet r2 = {f->r2, 0.0};
            jet p = j_div(j_sub(radius, r2), hi - f->r2);
            out = j_add(j_sub(j_add(j_sub(one, j_sc(35.0, j_pow4(p))), j_sc(84.0, j_pow5(p))),
                              j_sc(70.0, j_pow6(p))),
                        j_sc(20.0, j_pow7(p)));
        } else {
            out = one;
        }
        break;
    default: break;
    }
    *val = out.v;
    *der = out.d;
}

/* AnyTrans::compute_der of basis/xtrans.cpp (LinearShift, ExponentialShift,
 * FormulaShift::evaluate). */
static void shift_der(const oracle_radial_family *f, double lo, double hi, double r, double *val,
                      double *der)
{
    const double inv_range = 1.0 / (hi - lo);
    const double lambda = f->lambda;
    if (f->shift_type == 0) { /* linear */
        double slope = 2.0 / (hi - lo);
        *val = -1.0 + slope * (r - lo);
        *der = slope;
        return;
    }
    if (f->shift_type == 1) { /* exponential */
        if (lambda == 0.0) {
            *val = -1.0 + 2.0 * (r - lo) * inv_range;
            *der = 2.0 * inv_range;
            return;
        }
        double denominator = expm1(lambda);
        double exponent = lambda * (hi - r) * inv_range;
        double exponential = exp(exponent);
        *val = 1.0 - 2.0 * expm1(exponent) / denominator;
        *der = 2.0 * lambda * inv_range * exponential / denominator;
        return;
    }
    jet radius = {r, 1.0}, one = {1.0, 0.0}, lo_j = {lo, 0.0}, ir = {inv_range, 0.0};
    jet t = j_mul(j_sub(radius, lo_j), ir);
    jet out = {0.0, 0.0};
    if (f->shift_type == 3) { /* i2 */
        jet hi_j = {hi, 0.0};
        jet k = j_mul(j_sub(radius, hi_j), ir);
        out = j_sub(j_sc(2.0, j_mul(k, k)), one);
    } else if (f->shift_type == 2) { /* exponential_left */
        if (lambda == 0.0) {
            out = j_sub(j_div(j_sc(2.0, radius), hi), one);
        } else {
            double denominator = expm1(lambda);
            jet exponent = j_sc(lambda, j_sub(one, j_div(radius, hi)));
            out = j_sub(one, j_sc(2.0 / denominator, j_sub(j_exp(exponent), one)));
        }
    } else if (f->shift_type == 4) { /* exponential_tanh */
        jet shifted;
        if (lambda == 0.0) {
            shifted = j_sub(j_sc(2.0, t), one);
        } else {
            double denominator = expm1(lambda);
            shifted =
                j_sub(one, j_sc(2.0 / denominator, j_sub(j_exp(j_sc(lambda, j_sub(one, t))), one)));
        }
        if (f->scale_lambda == 0.0)
            out = shifted;
        else
            out = j_div(j_tanh(j_sc(f->scale_lambda, shifted)), tanh(f->scale_lambda));
    }
    *val = out.v;
    *der = out.d;
}

/* Radial basis values and derivatives of a pair's family. */
static void rb_calc_der(const oracle_model *m, int pair, int R, double r, double *val,
                        double *der)
{
    const double lo = pair_min(m, pair), hi = pair_max(m, pair), s = m->scaling;
    const oracle_radial_family *f = NULL;
    if (m->radial_family)
        f = &m->radial_family[m->radial_basis_split ? pair : 0];
    if (!f || f->type == 0) {
        cheb_calc_der(lo, hi, s, R, r, val, der);
        return;
    }
    const double mult = 2.0 / (hi - lo), su = hi - lo, pu = hi + lo;
    if (f->type == 5 || f->type == 6) {
        /* RBPolyB / RBPolyBCos: MLIPCore::Radial::evaluate_polynomial
         * (runtime/mtp/radial_basis.h:223-290) in its order: column 0 seeds
         * the sums, the other columns add in j order; the CosineLeft envelope
         * of RBPolyBCos is applied last.  excludes() zeroes r >= max_dist. */
        if (r >= hi) {
            for (int i = 0; i < R; ++i)
                val[i] = der[i] = 0.0;
            return;
        }
        const double *M = f->poly_matrix, *N = f->poly_norm;
        const double delta = hi - r;
        const int first = f->type == 5 ? 3 : 2;
        double fc = 1.0, dfc = 0.0;
        if (first == 2) {
            const double freq = ORACLE_PI / hi;
            fc = 0.5 * (1.0 + cos(r * freq));
            dfc = -0.5 * sin(r * freq) * freq;
        }
        double previous = s * delta;
        if (first == 3)
            previous *= delta;
        const double first_power = previous * delta;
        const double first_value = N[0] * first_power;
        const double first_derivative = -(N[0] * first) * previous;
        for (int i = 0; i < R; ++i) {
            val[i] = 0.0 + M[i] * first_value;
            der[i] = 0.0 + M[i] * first_derivative;
        }
        previous = first_power;
        for (int j = 1; j < R; ++j) {
            const double power = previous * delta;
            const double value = N[j] * power;
            const double derivative = -(N[j] * (j + first)) * previous;
            const double *column = M + (size_t)j * R;
            for (int i = 0; i < R; ++i) {
                val[i] += column[i] * value;
                der[i] += column[i] * derivative;
            }
            previous = power;
        }
        if (first == 2)
            for (int i = 0; i < R; ++i) {
                der[i] = der[i] * fc + val[i] * dfc;
                val[i] *= fc;
            }
        return;
    }
    if (f->type == 3) { /* RBasis_ChebyshevConfigurable::calculate, order 1 */
        if (r < lo || r > hi) {
            for (int i = 0; i < R; ++i)
                val[i] = der[i] = 0.0;
            return;
        }
        double x, dx, fc, dfc;
        shift_der(f, lo, hi, r, &x, &dx);
        cutoff_der(f, lo, hi, r, &fc, &dfc);
        const int flipped = f->one_minus_chebyshev != 0;
        const int n = R + (flipped ? 1 : 0);
        double *tv = (double *)calloc((size_t)n, sizeof(double));
        double *td = (double *)calloc((size_t)n, sizeof(double));
        tv[0] = 1.0;
        if (n > 1) {
            tv[1] = x;
            td[1] = dx;
        }
        for (int i = 2; i < n; ++i) {
            tv[i] = 2.0 * x * tv[i - 1] - tv[i - 2];
            td[i] = 2.0 * (dx * tv[i - 1] + x * td[i - 1]) - td[i - 2];
        }
        for (int i = 0; i < R; ++i) {
            const int k = i + (flipped ? 1 : 0);
            const double raw = flipped ? 1.0 - tv[k] : tv[k];
            const double raw_der = flipped ? -td[k] : td[k];
            val[i] = s * raw * fc;
            der[i] = s * (raw_der * fc + raw * dfc);
        }
        free(tv);
        free(td);
        return;
    }
    double ksi = (2 * r - pu) / su;
    double rc, drc;
    if (f->type == 1) { /* RBasis_ChebyCos::calc_der */
        double irpi = ORACLE_PI / hi;   /* M_PI of basis.cpp */
        rc = 0.5 * (1.0 + cos(r * irpi));
        drc = -0.5 * irpi * sin(r * irpi);
        val[0] = s * (1 * rc);
        der[0] = s * (0 * rc + drc);
    } else { /* RBasis_ChebyshevPoly4 / Poly5::calc_der */
        if (r < lo || r > hi) {
            for (int i = 0; i < R; ++i)
                val[i] = der[i] = 0.0;
            return;
        }
        double x = (r - lo) / su;
        double dxdr = 1.0 / su;
        double vx = 1.0 - x;
        double vxx = vx * vx;
        double vxxx = vxx * vx;
        if (f->type == 2) {
            double vxxxx = vxx * vxx;
            rc = vxxxx * (1 + (4 + f->b) * x);
            drc = -vxxx * (20 * x + f->b * (5 * x - 1)) * dxdr;
        } else {
            rc = vxxx * (1 + (3 + f->b) * x);
            drc = vxx * (f->b * (1. - 4.0 * x) - 12.0 * x) * dxdr;
        }
        val[0] = s * rc;
        der[0] = s * drc;
    }
    if (R == 1)
        return;
    val[1] = s * (ksi * rc);
    der[1] = s * (mult * rc + ksi * drc);
    for (int i = 2; i < R; i++) {
        val[i] = 2 * ksi * val[i - 1] - val[i - 2];
        der[i] = 2 * (mult * val[i - 1] + ksi * der[i - 1]) - der[i - 2];
    }
}

#define CP(ws, k, a) ((ws)->cp[(k)*3 + (a)])
#define MJ(ws, n, i, j, a) ((ws)->mj[((size_t)(i) * (n) + (j)) * 3 + (a)])

/* PotMTP::CalcSiteDescriptorsImpl (potential_mtp.cpp:2813-2925): basic
 * moments, basic Jacobian, forward product rules. */
static void site_descriptors(const oracle_model *m, site_ws *ws, int itype, int nn,
                             const int *jtypes, const double *rij, const double *dist)
{
    const int nb = ws->nb;
    memset(ws->mj, 0, sizeof(double) * (size_t)nb * nn * 3);
    memset(ws->mv, 0, sizeof(double) * ws->M);
    memset(ws->rv, 0, sizeof(double) * ws->R);
    memset(ws->rd, 0, sizeof(double) * ws->R);
    const int K = ws->K, MU = ws->mu, R = ws->R;
    for (int jj = 0; jj < nn; ++jj) {
        const double r = dist[jj];
        const int jt = jtypes[jj];
        const int pair = itype * K + jt;
        if (r > pair_max(m, pair))
            continue;
        const double rinv = 1.0 / r;
        rb_calc_der(m, pair, R, r, ws->rv, ws->rd);
        ws->dp[0] = 1;
        for (int k = 1; k < ws->maxnu; ++k) {
            ws->dp[k] = ws->dp[k - 1] * rinv;
            for (int a = 0; a < 3; a++)
                CP(ws, k + 1, a) = CP(ws, k, a) * rij[3 * jj + a];
        }
        for (int mu = 0; mu < ws->maxmu; ++mu) {
            ws->vm[mu] = 0;
            ws->dm[mu] = 0;
            int off = (itype * K + jt) * MU * R + mu * R;
            for (int xi = 0; xi < R; ++xi) {
                ws->vm[mu] += m->radial_coeffs[off + xi] * ws->rv[xi];
                ws->dm[mu] += m->radial_coeffs[off + xi] * ws->rd[xi];
            }
        }
        for (int i = 0; i < nb; ++i) {
            const int *bi = m->alpha_index_basic + 4 * i;
            int mu = bi[0];
            double val = ws->vm[mu];
            double der = ws->dm[mu];
            int k = bi[1] + bi[2] + bi[3];
            double powk = ws->dp[k];
            val *= powk;
            der = der * powk - k * val / r;
            double pow0 = CP(ws, bi[1] + 1, 0);
            double pow1 = CP(ws, bi[2] + 1, 1);
            double pow2 = CP(ws, bi[3] + 1, 2);
            double mult0 = pow0 * pow1 * pow2;
            ws->mv[i] += val * mult0;
            mult0 *= der / r;
            MJ(ws, nn, i, jj, 0) += mult0 * rij[3 * jj + 0];
            MJ(ws, nn, i, jj, 1) += mult0 * rij[3 * jj + 1];
            MJ(ws, nn, i, jj, 2) += mult0 * rij[3 * jj + 2];
            MJ(ws, nn, i, jj, 0) += bi[1] * val * CP(ws, bi[1], 0) * pow1 * pow2;
            MJ(ws, nn, i, jj, 1) += bi[2] * val * CP(ws, bi[2], 1) * pow0 * pow2;
            MJ(ws, nn, i, jj, 2) += bi[3] * val * CP(ws, bi[3], 2) * pow0 * pow1;
        }
    }
    for (int i = 0; i < ws->T; ++i) {
        const int *t = m->alpha_index_times + 4 * i;
        double val0 = ws->mv[t[0]];
        double val1 = ws->mv[t[1]];
        int val2 = t[2];
        ws->mv[t[3]] += val2 * val0 * val1;
    }
}

/* PotMTP::backpropagate_moments (potential_mtp.cpp:3292-3305) */
static void backpropagate(const oracle_model *m, site_ws *ws)
{
    for (int i = ws->T - 1; i >= 0; i--) {
        const int *t = m->alpha_index_times + 4 * i;
        double val0 = ws->mv[t[0]];
        double val1 = ws->mv[t[1]];
        int val2 = t[2];
        ws->sed[t[1]] += ws->sed[t[3]] * val2 * val0;
        ws->sed[t[0]] += ws->sed[t[3]] * val2 * val1;
    }
}

/* PotMTP::CalcSiteEFS (potential_mtp.cpp:2959-2984) + contract_site_forces
 * (:2938-2957).  dedr[nn][3] receives buff_site_energy_ders. */
static double site_efs(const oracle_model *m, site_ws *ws, int itype, int nn, const int *jtypes,
                       const double *rij, const double *dist, double *dedr)
{
    site_descriptors(m, ws, itype, nn, jtypes, rij, dist);
    double se = 0;
    se += m->species_coeffs[itype];
    for (int i = 0; i < ws->S; ++i)
        se += m->moment_coeffs[i] * ws->mv[m->alpha_moment_mapping[i]];
    memset(ws->sed, 0, sizeof(double) * ws->M);
    for (int i = 0; i < ws->S; ++i)
        ws->sed[m->alpha_moment_mapping[i]] += m->moment_coeffs[i];
    backpropagate(m, ws);
    memset(dedr, 0, sizeof(double) * 3 * (size_t)nn);
    const size_t stride = (size_t)nn * 3;
    for (int i = 0; i < ws->nb; ++i) {
        const double weight = ws->sed[i];
        const double *row = ws->mj + i * stride;
        for (size_t j = 0; j < stride; ++j)
            dedr[j] += weight * row[j];
    }
    return se;
}

static int max_degree(int n, const int *offsets)
{
    int mx = 0;
    for (int i = 0; i < n; ++i)
        if (offsets[i + 1] - offsets[i] > mx)
            mx = offsets[i + 1] - offsets[i];
    return mx;
}

static void gather_site(int i, const int *types, const int *offsets, const int *nbr,
                        const double *rij, int *jt, double *dist)
{
    for (int e = offsets[i]; e < offsets[i + 1]; ++e) {
        const double *r = rij + 3 * (size_t)e;
        jt[e - offsets[i]] = types[nbr[e]];
        dist[e - offsets[i]] = sqrt(r[0] * r[0] + r[1] * r[1] + r[2] * r[2]);
    }
}

/* PotMTP::getEFS(Atoms&, AnyNeighborhoods&), potential_mtp.cpp:1899-1933 */
static int efs_range(const oracle_model *m, int a0, int a1, const int *types, const int *offsets,
                     const int *nbr, const double *rij, double *energy, double *site_energy,
                     double *forces, double *stress, site_ws *ws, double *dedr, int *jt,
                     double *dist)
{
    *energy = 0;
    for (int a = 0; a < 9; ++a)
        stress[a] = 0;
    for (int i = a0; i < a1; ++i)
        forces[3 * i] = forces[3 * i + 1] = forces[3 * i + 2] = 0;
    for (int ii = a0; ii < a1; ii++) {
        int nn = offsets[ii + 1] - offsets[ii];
        gather_site(ii, types, offsets, nbr, rij, jt, dist);
        const double *r = rij + 3 * (size_t)offsets[ii];
        double se = site_efs(m, ws, types[ii], nn, jt, r, dist, dedr);
        *energy += se;
        if (site_energy)
            site_energy[ii] = se;
        for (int i = 0; i < nn; ++i) {
            int j = nbr[offsets[ii] + i];
            for (int a = 0; a < 3; ++a)
                forces[3 * ii + a] += dedr[3 * i + a];
            for (int a = 0; a < 3; ++a)
                forces[3 * j + a] -= dedr[3 * i + a];
            for (int a = 0; a < 3; a++)
                for (int b = 0; b < 3; b++)
                    stress[a * 3 + b] -= dedr[3 * i + a] * r[3 * i + b];
        }
    }
    return 0;
}

int oracle_efs(const oracle_model *m, int n, const int *types, const int *offsets,
               const int *nbr, const double *rij, double *energy, double *site_energy,
               double *forces, double *stress)
{
    int nmax = max_degree(n, offsets);
    site_ws ws;
    if (ws_init(&ws, m, nmax, 0))
        return -1;
    double *dedr = (double *)malloc(sizeof(double) * 3 * (size_t)(nmax + 1));
    int *jt = (int *)malloc(sizeof(int) * (size_t)(nmax + 1));
    double *dist = (double *)malloc(sizeof(double) * (size_t)(nmax + 1));
    int rc = -1;
    if (dedr && jt && dist)
        rc = efs_range(m, 0, n, types, offsets, nbr, rij, energy, site_energy, forces, stress, &ws,
                       dedr, jt, dist);
    free(dedr);
    free(jt);
    free(dist);
    ws_free(&ws);
    return rc;
}

int oracle_site_derivatives(const oracle_model *m, int n, const int *types,
                            const int *offsets, const int *nbr, const double *rij,
                            double *site_energy, double *dedr)
{
    int nmax = max_degree(n, offsets);
    site_ws ws;
    if (ws_init(&ws, m, nmax, 0))
        return -1;
    int *jt = (int *)malloc(sizeof(int) * (size_t)(nmax + 1));
    double *dist = (double *)malloc(sizeof(double) * (size_t)(nmax + 1));
    if (!jt || !dist) {
        free(jt);
        free(dist);
        ws_free(&ws);
        return -1;
    }
    for (int ii = 0; ii < n; ++ii) {
        int nn = offsets[ii + 1] - offsets[ii];
        gather_site(ii, types, offsets, nbr, rij, jt, dist);
        double se = site_efs(m, &ws, types[ii], nn, jt, rij + 3 * (size_t)offsets[ii], dist,
                             dedr + 3 * (size_t)offsets[ii]);
        if (site_energy)
            site_energy[ii] = se;
    }
    free(jt);
    free(dist);
    ws_free(&ws);
    return 0;
}

int oracle_site_moments(const oracle_model *m, int n, const int *types, const int *offsets,
                        const int *nbr, const double *rij, double *basic, double *adjoint)
{
    int nmax = max_degree(n, offsets);
    site_ws ws;
    if (ws_init(&ws, m, nmax, 0))
        return -1;
    int *jt = (int *)malloc(sizeof(int) * (size_t)(nmax + 1));
    double *dist = (double *)malloc(sizeof(double) * (size_t)(nmax + 1));
    double *dedr = (double *)malloc(sizeof(double) * 3 * (size_t)(nmax + 1));
    if (!jt || !dist || !dedr) {
        free(jt);
        free(dist);
        free(dedr);
        ws_free(&ws);
        return -1;
    }
    const int nb = ws.nb;
    for (int ii = 0; ii < n; ++ii) {
        int nn = offsets[ii + 1] - offsets[ii];
        gather_site(ii, types, offsets, nbr, rij, jt, dist);
        site_efs(m, &ws, types[ii], nn, jt, rij + 3 * (size_t)offsets[ii], dist, dedr);
        /* the forward rules only add to non-basic targets, so mv[0..nb) are
         * the basic moments themselves */
        if (basic)
            memcpy(basic + (size_t)ii * nb, ws.mv, sizeof(double) * nb);
        if (adjoint)
            memcpy(adjoint + (size_t)ii * nb, ws.sed, sizeof(double) * nb);
    }
    free(jt);
    free(dist);
    free(dedr);
    ws_free(&ws);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Parameter gradient                                                        */
/* ------------------------------------------------------------------------ */

#define MJC(ws, i, j, k) ((ws)->mjc[(((size_t)(i) * (ws)->K + (j)) * (ws)->mu * (ws)->R) + (k)])
#define MJCC(ws, i, j, k) ((ws)->mjcc[(((size_t)(i) * (ws)->K + (j)) * (ws)->mu * (ws)->R) + (k)])

/* PotMTP::accumulate_site_parameter_gradient, potential_mtp.cpp:3348-3550.
 * f_weight: [nn][3] or NULL (energy-only). */
static void site_parameter_gradient(const oracle_model *m, site_ws *ws, int itype, int nn,
                                    const int *jtypes, const double *rij, const double *dist,
                                    double se_weight, const double *f_weight,
                                    double *radial_gradient, double *moment_gradient)
{
    const int need = f_weight != NULL;
    const int nb = ws->nb, K = ws->K, MU = ws->mu, R = ws->R;
    const size_t g = (size_t)nb * K * MU * R;
    memset(ws->mjc, 0, sizeof(double) * g);
    memset(ws->rd, 0, sizeof(double) * R);
    if (need) {
        memset(ws->mjcc, 0, sizeof(double) * g);
        memset(ws->dm, 0, sizeof(double) * (MU + 1));
        memset(ws->dlds, 0, sizeof(double) * ws->M);
    }
    memset(ws->mv, 0, sizeof(double) * ws->M);
    memset(ws->rv, 0, sizeof(double) * R);
    memset(ws->vm, 0, sizeof(double) * (MU + 1));
    memset(ws->dldm, 0, sizeof(double) * ws->M);
    memset(ws->sed, 0, sizeof(double) * ws->M);
    for (int jj = 0; jj < nn; ++jj) {
        const double r = dist[jj];
        const int jt = jtypes[jj];
        const int pair = itype * K + jt;
        if (r > pair_max(m, pair))
            continue;
        const double rinv = 1.0 / r;
        rb_calc_der(m, pair, R, r, ws->rv, ws->rd);
        ws->dp[0] = 1;
        for (int k = 1; k < ws->maxnu; ++k) {
            ws->dp[k] = ws->dp[k - 1] * rinv;
            for (int a = 0; a < 3; a++)
                CP(ws, k + 1, a) = CP(ws, k, a) * rij[3 * jj + a];
        }
        for (int mu = 0; mu < ws->maxmu; ++mu) {
            ws->vm[mu] = 0;
            if (need)
                ws->dm[mu] = 0;
            int off = (itype * K + jt) * MU * R + mu * R;
            for (int xi = 0; xi < R; ++xi) {
                ws->vm[mu] += m->radial_coeffs[off + xi] * ws->rv[xi];
                if (need)
                    ws->dm[mu] += m->radial_coeffs[off + xi] * ws->rd[xi];
            }
        }
        for (int i = 0; i < nb; ++i) {
            const int *index = m->alpha_index_basic + 4 * i;
            const int mu = index[0], x = index[1], y = index[2], z = index[3];
            const int k = x + y + z;
            const double powk = ws->dp[k];
            const double val = ws->vm[mu] * powk;
            const double pow0 = CP(ws, x + 1, 0);
            const double pow1 = CP(ws, y + 1, 1);
            const double pow2 = CP(ws, z + 1, 2);
            const double mult0 = pow0 * pow1 * pow2;
            ws->mv[i] += val * mult0;
            for (int xi = 0; xi < R; xi++) {
                MJC(ws, i, jt, mu * R + xi) += ws->rv[xi] * powk * mult0;
                if (need) {
                    double tail = (ws->rd[xi] * powk * mult0 -
                                   ws->rv[xi] * k * powk * mult0 / dist[jj]);
                    double derx = (rij[3 * jj + 0] / dist[jj]) * tail;
                    double dery = (rij[3 * jj + 1] / dist[jj]) * tail;
                    double derz = (rij[3 * jj + 2] / dist[jj]) * tail;
                    derx += ws->rv[xi] * powk * x * CP(ws, x, 0) * pow1 * pow2;
                    dery += ws->rv[xi] * powk * y * CP(ws, y, 1) * pow0 * pow2;
                    derz += ws->rv[xi] * powk * z * CP(ws, z, 2) * pow0 * pow1;
                    MJCC(ws, i, jt, mu * R + xi) += f_weight[3 * jj + 0] * derx +
                                                    f_weight[3 * jj + 1] * dery +
                                                    f_weight[3 * jj + 2] * derz;
                }
            }
            if (need) {
                const double der = ws->dm[mu] * powk - k * val / r;
                const double radial = mult0 * (der / r);
                const double dx = radial * rij[3 * jj + 0] + x * val * CP(ws, x, 0) * pow1 * pow2;
                const double dy = radial * rij[3 * jj + 1] + y * val * CP(ws, y, 1) * pow0 * pow2;
                const double dz = radial * rij[3 * jj + 2] + z * val * CP(ws, z, 2) * pow0 * pow1;
                ws->dlds[i] += f_weight[3 * jj + 0] * dx;
                ws->dlds[i] += f_weight[3 * jj + 1] * dy;
                ws->dlds[i] += f_weight[3 * jj + 2] * dz;
            }
        }
    }
    const int T = ws->T;
    for (int i = 0; i < T; ++i) {
        const int *t = m->alpha_index_times + 4 * i;
        double val0 = ws->mv[t[0]];
        double val1 = ws->mv[t[1]];
        double val2 = t[2];
        ws->mv[t[3]] += val2 * val0 * val1;
    }
    for (int i = 0; i < ws->S; ++i)
        ws->sed[m->alpha_moment_mapping[i]] += m->moment_coeffs[i];
    backpropagate(m, ws);
    for (int i = 0; i < nb; ++i)
        ws->dldm[i] = se_weight * ws->sed[i];
    if (need) {
        for (int i = 0; i < T; ++i) {
            const int *t = m->alpha_index_times + 4 * i;
            double val2 = t[2];
            double val0 = ws->mv[t[0]];
            double val1 = ws->mv[t[1]];
            ws->dlds[t[3]] += ws->dlds[t[0]] * val2 * val1 + ws->dlds[t[1]] * val2 * val0;
        }
        for (int i = 0; i < T; ++i) {
            const int *t = m->alpha_index_times + 4 * i;
            double val2 = t[2];
            ws->dldm[t[1]] += ws->dlds[t[0]] * ws->sed[t[3]] * val2;
            ws->dldm[t[0]] += ws->dlds[t[1]] * ws->sed[t[3]] * val2;
        }
        for (int i = T - 1; i >= 0; --i) {
            const int *t = m->alpha_index_times + 4 * i;
            double val0 = ws->mv[t[0]];
            double val1 = ws->mv[t[1]];
            double val2 = t[2];
            ws->dldm[t[0]] += ws->dldm[t[3]] * val2 * val1;
            ws->dldm[t[1]] += ws->dldm[t[3]] * val2 * val0;
        }
    }
    for (int i = 0; i < nb; ++i) {
        const int channel = m->alpha_index_basic[4 * i] * R;
        for (int j = 0; j < K; ++j) {
            const int pair = itype * K + j;
            for (int k = channel; k < channel + R; ++k) {
                const int idx = pair * R * MU + k;
                radial_gradient[idx] += ws->dldm[i] * MJC(ws, i, j, k);
                if (need)
                    radial_gradient[idx] += ws->sed[i] * MJCC(ws, i, j, k);
            }
        }
    }
    if (moment_gradient) {
        for (int i = 0; i < ws->S; ++i) {
            moment_gradient[i] += se_weight * ws->mv[m->alpha_moment_mapping[i]];
            if (need)
                moment_gradient[i] += ws->dlds[m->alpha_moment_mapping[i]];
        }
    }
}

static double sqnorm3(double a, double b, double c)
{
    return a * a + b * b + c * c;
}

/* one structure: Trainer_MTP::AddLossGard (train_mtp.cpp:3839-3996) followed
 * by PotMTP::AccumulateEFSCombinationGard (potential_mtp.cpp:6896-6922). */
static int structure_loss_grad(const oracle_model *m, const oracle_loss_weights *w, int a0,
                               int a1, const int *types, const int *offsets, const int *nbr,
                               const double *rij, double target_e, const double *target_f,
                               const double *target_s, int has_e, int has_f, int has_s,
                               double *loss, double *metrics, double *grad, site_ws *ws,
                               double *dedr, int *jt, double *dist, double *forces)
{
    const int n = a1 - a0;
    if (n == 0)
        return 0;
    const int energy_only = !(w->weight_force > 0 && has_f) && !(w->weight_stress > 0 && has_s);
    double energy = 0, stress[9];
    /* forces buffer is indexed by global atom index */
    efs_range(m, a0, a1, types, offsets, nbr, rij, &energy, NULL, forces, stress, ws, dedr, jt,
              dist);
    (void)energy_only; /* getE and getEFS agree on energy; forces unused then */

    double *dLdF = (double *)calloc(3 * (size_t)n, sizeof(double));
    if (!dLdF)
        return -1;
    double dLdS[9] = {0};
    double dLdE = 0;
    const double cc = 1.0;
    if (w->weight_force > 0 && has_f) {
        double wf = w->weight_force / pow((double)n, w->weight_force_power) * cc;
        for (int i = 0; i < n; ++i) {
            const double *fp = forces + 3 * (size_t)(a0 + i);
            const double *ft = target_f + 3 * (size_t)(a0 + i);
            double ff = sqnorm3(fp[0] - ft[0], fp[1] - ft[1], fp[2] - ft[2]);
            metrics[5] += ff;
            double ll = wf * ff;
            *loss += ll;
            metrics[2] += ll;
            for (int a = 0; a < 3; ++a)
                dLdF[3 * i + a] = 2.0 * wf * (fp[a] - ft[a]);
        }
    }
    if (w->weight_stress > 0 && has_s) {
        double ws_ = w->weight_stress / pow((double)n, w->weight_stress_power) * cc;
        double ff = 0;
        /* Eigen squaredNorm of a 3x3 difference */
        for (int a = 0; a < 9; ++a)
            ff += (stress[a] - target_s[a]) * (stress[a] - target_s[a]);
        metrics[6] += ff;
        double ll = ws_ * ff;
        *loss += ll;
        metrics[3] += ll;
        for (int a = 0; a < 9; ++a)
            dLdS[a] = 2 * ws_ * (stress[a] - target_s[a]);
    }
    if (w->weight_eng > 0 && has_e) {
        double we = w->weight_eng / pow((double)n, w->weight_eng_power) * cc;
        double ff = (energy - target_e) * (energy - target_e);
        metrics[4] += ff / n / n;
        double ll = we * ff;
        *loss += ll;
        metrics[1] += ll;
        dLdE = 2 * we * (energy - target_e);
    }
    const int rsize = m->species_count * m->species_count * m->radial_func_count * m->rb_size;
    double *radial = grad;
    double *species = grad + rsize;
    double *moment = grad + rsize + m->species_count;
    for (int i = a0; i < a1; ++i) {
        int nn = offsets[i + 1] - offsets[i];
        gather_site(i, types, offsets, nbr, rij, jt, dist);
        const double *r = rij + 3 * (size_t)offsets[i];
        if (energy_only) {
            site_parameter_gradient(m, ws, types[i], nn, jt, r, dist, dLdE, NULL, radial, moment);
        } else {
            for (int j = 0; j < nn; ++j) {
                int jn = nbr[offsets[i] + j] - a0;
                for (int a = 0; a < 3; ++a) {
                    ws->w[3 * j + a] = 0;
                    ws->w[3 * j + a] += dLdF[3 * (i - a0) + a];
                    ws->w[3 * j + a] -= dLdF[3 * jn + a];
                }
            }
            for (int j = 0; j < nn; ++j)
                for (int a = 0; a < 3; ++a)
                    for (int b = 0; b < 3; ++b)
                        ws->w[3 * j + a] -= dLdS[a * 3 + b] * r[3 * j + b];
            site_parameter_gradient(m, ws, types[i], nn, jt, r, dist, dLdE, ws->w, radial,
                                    moment);
        }
        species[types[i]] += dLdE;
    }
    free(dLdF);
    return 0;
}

int oracle_loss_grad(const oracle_model *m, const oracle_loss_weights *w, int n_struct,
                     const int *atom_offsets, const int *types, const int *offsets,
                     const int *nbr, const double *rij, const double *target_energy,
                     const double *target_forces, const double *target_stress,
                     const int *has_energy, const int *has_forces, const int *has_stress,
                     double *loss, double *metrics, double *grad)
{
    const int natoms = atom_offsets[n_struct];
    const int ncoef = m->species_count * m->species_count * m->radial_func_count * m->rb_size +
                      m->species_count + m->alpha_scalar_moments;
    int nmax = max_degree(natoms, offsets);
    site_ws ws;
    if (ws_init(&ws, m, nmax, 1))
        return -1;
    double *dedr = (double *)malloc(sizeof(double) * 3 * (size_t)(nmax + 1));
    int *jt = (int *)malloc(sizeof(int) * (size_t)(nmax + 1));
    double *dist = (double *)malloc(sizeof(double) * (size_t)(nmax + 1));
    double *forces = (double *)calloc(3 * (size_t)(natoms + 1), sizeof(double));
    int rc = 0;
    if (!dedr || !jt || !dist || !forces)
        rc = -1;
    *loss = 0;
    for (int k = 0; k < 7; ++k)
        metrics[k] = 0;
    memset(grad, 0, sizeof(double) * ncoef);
    for (int s = 0; s < n_struct && rc == 0; ++s) {
        rc = structure_loss_grad(
            m, w, atom_offsets[s], atom_offsets[s + 1], types, offsets, nbr, rij,
            target_energy ? target_energy[s] : 0.0, target_forces,
            target_stress ? target_stress + 9 * (size_t)s : NULL,
            target_energy && (!has_energy || has_energy[s]),
            target_forces && (!has_forces || has_forces[s]),
            target_stress && (!has_stress || has_stress[s]), loss, metrics, grad, &ws, dedr, jt,
            dist, forces);
    }
    metrics[0] = *loss;
    if (rc == 0 && n_struct > 0) {
        *loss /= n_struct;
        for (int i = 0; i < ncoef; ++i)
            grad[i] = grad[i] / n_struct;
    }
    free(dedr);
    free(jt);
    free(dist);
    free(forces);
    ws_free(&ws);
    return rc;
}

int oracle_efs_batch(const oracle_model *m, int n_struct, const int *atom_offsets,
                     const int *types, const int *offsets, const int *nbr, const double *rij,
                     double *energy, double *forces, double *stress, int threads)
{
    int err = 0;
    const int natoms = atom_offsets[n_struct];
    int nmax = max_degree(natoms, offsets);
#ifdef _OPENMP
    if (threads > 0)
        omp_set_num_threads(threads);
#pragma omp parallel reduction(| : err)
#endif
    {
        site_ws ws;
        double *dedr = NULL, *dist = NULL;
        int *jt = NULL;
        if (ws_init(&ws, m, nmax, 0) == 0) {
            dedr = (double *)malloc(sizeof(double) * 3 * (size_t)(nmax + 1));
            jt = (int *)malloc(sizeof(int) * (size_t)(nmax + 1));
            dist = (double *)malloc(sizeof(double) * (size_t)(nmax + 1));
            if (dedr && jt && dist) {
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
                for (int s = 0; s < n_struct; ++s)
                    efs_range(m, atom_offsets[s], atom_offsets[s + 1], types, offsets, nbr, rij,
                              energy + s, NULL, forces, stress + 9 * (size_t)s, &ws, dedr, jt,
                              dist);
            } else {
                err |= 1;
            }
            ws_free(&ws);
        } else {
            err |= 1;
        }
        free(dedr);
        free(jt);
        free(dist);
    }
    return err ? -1 : 0;
}
