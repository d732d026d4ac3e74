/*
 * hawk_oracle.c -- TEST INFRASTRUCTURE ONLY (see hawk_oracle.h): the CPU
 * restatement of the reference's host target for the five benchmark kernels.
 *
 * Built with -O3 -march=native -ffp-contract=off (no FMA contraction), the
 * reference's `native` host profile (hawk/compile/toolchain.py:897-900).  Each kernel
 * function below states the body the reference renderer writes for the kernel
 * (hawk/emit/render.py:140; the kernels are the ones in hawk_b200/configs.py),
 * operation for operation, inside the serial host loop of
 * hawk/emit/host.py:1386-1495.  Vector helpers follow the library order the
 * reference restates for its own C export: dot products and sums ascending,
 * hawk/embedded/writer.py:603-625.
 */
#include "hawk_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* glibc's sin and cos: the reference host target's libm */
static double o_sin(double x) { return sin(x); }
static double o_cos(double x) { return cos(x); }

/* ------------------------------------------------------------------ c1 energy */

/* out = (0.5 * v.dot(v)) */
void hko_energy(const double* v, int64_t pitch, double* out, int64_t base, int64_t count) {
    for (int64_t i = base; i < base + count; ++i) {
        const double v0 = v[i], v1 = v[pitch + i], v2 = v[2 * pitch + i];
        const double d = ((v0 * v0) + (v1 * v1)) + (v2 * v2);
        out[i] = 0.5 * d;
    }
}

/* t4 = (bar_out * 0.5) * v;  bar_v = t4 + t4 */
void hko_energy_vjp(const double* v, int64_t pitch, const double* bar_out, double* bar_v, int64_t bar_pitch,
                    int64_t base, int64_t count) {
    for (int64_t i = base; i < base + count; ++i) {
        const double s = bar_out[i] * 0.5;
        for (int k = 0; k < 3; ++k) {
            const double t4 = s * v[k * pitch + i];
            bar_v[k * bar_pitch + i] = t4 + t4;
        }
    }
}

/* dot_out = 0.5 * (dot_v.dot(v) + v.dot(dot_v)) */
void hko_energy_jvp(const double* v, int64_t pitch, const double* dot_v, int64_t dot_pitch, double* dot_out,
                    int64_t base, int64_t count) {
    for (int64_t i = base; i < base + count; ++i) {
        const double v0 = v[i], v1 = v[pitch + i], v2 = v[2 * pitch + i];
        const double d0 = dot_v[i], d1 = dot_v[dot_pitch + i], d2 = dot_v[2 * dot_pitch + i];
        const double a = ((d0 * v0) + (d1 * v1)) + (d2 * v2);
        const double b = ((v0 * d0) + (v1 * d1)) + (v2 * d2);
        dot_out[i] = 0.5 * (a + b);
    }
}

/* --------------------------------------------------------- c2 affine polynomial */

/* t11 = (((((a*x)*x)*x) + (b*x)) + c) - t;  r = t11 * t11 */
#define POLY_BODY(T)                                                               \
    for (int64_t i = base; i < base + count; ++i) {                                \
        const T xi = x[i];                                                         \
        const T t11 = ((((((a * xi) * xi) * xi) + (b * xi)) + c) - t[i]);          \
        r[i] = t11 * t11;                                                          \
    }

void hko_poly_loss_f64(const double* x, const double* t, double a, double b, double c, double* r,
                       int64_t base, int64_t count) {
    POLY_BODY(double)
}

void hko_poly_loss_f32(const float* x, const float* t, float a, float b, float c, float* r,
                       int64_t base, int64_t count) {
    POLY_BODY(float)
}

/*
 * The host sample-sum frame (hawk/emit/host.py:1499-1530) with the row tree of
 * sampleSumRow_ (hawk/emit/wrapper.py:578-592): 32 slots per row, a slot past
 * the last sample holding 0, slot l joined with slot l + off (lower first) for
 * off = 16, 8, 4, 2, 1 by pairCombine_ (hawk/emit/wrapper.py:561-576), whose
 * residual is the two-sum error with the larger magnitude first, +0 for zero
 * (hawk/_cells.py:44-49).
 */
#define DEFINE_PAIR(T, SUF)                                                                \
    static int finite_##SUF(T x) { return (x - x) == (x - x); }                           \
    static T two_sum_err_##SUF(T a, T b, T s) {                                           \
        const int a_big = (a < 0 ? -a : a) >= (b < 0 ? -b : b);                           \
        const T big = a_big ? a : b, small = a_big ? b : a;                                \
        return (small - (s - big)) + (T)0;                                                 \
    }                                                                                      \
    static void pair_##SUF(T* s, T* c, T s2, T c2) {                                      \
        const T t = *s + s2;                                                               \
        const T e = two_sum_err_##SUF(*s, s2, t);                                          \
        *c = finite_##SUF(t) ? (*c + c2) + e : (T)0;                                       \
        *s = t;                                                                            \
    }
DEFINE_PAIR(double, d)
DEFINE_PAIR(float, f)

/* row j: terms of samples 32j .. 32j+31 (0 past n), columns k = 0..2 */
#define POLY_VJP_ROWS(T, SUF)                                                              \
    for (int64_t j = 0; j < nrows; ++j) {                                                  \
        T h[32][3], cc[32][3];                                                             \
        const int64_t row = row0 + j;                                                      \
        for (int l = 0; l < 32; ++l) {                                                     \
            const int64_t i = row * 32 + l;                                                \
            for (int k = 0; k < 3; ++k) { h[l][k] = 0; cc[l][k] = 0; }                     \
            if (i < n) {                                                                   \
                const T xi = x[i];                                                         \
                const T t17 = (bar_r[i] * ((((((a * xi) * xi) * xi) + (b * xi)) + c) - t[i])); \
                const T t18 = t17 + t17;                                                   \
                const T t19 = t18 * xi;                                                    \
                h[l][0] = (t19 * xi) * xi;                                                 \
                h[l][1] = t19;                                                             \
                h[l][2] = t18;                                                             \
            }                                                                              \
        }                                                                                  \
        for (int off = 16; off >= 1; off >>= 1)                                            \
            for (int l = 0; l < off; ++l)                                                  \
                for (int k = 0; k < 3; ++k)                                                \
                    pair_##SUF(&h[l][k], &cc[l][k], h[l + off][k], cc[l + off][k]);        \
        for (int k = 0; k < 3; ++k) {                                                      \
            hi[k * nrows + j] = h[0][k];                                                   \
            comp[k * nrows + j] = cc[0][k];                                                \
        }                                                                                  \
    }

void hko_poly_loss_vjp_rows_f64(const double* x, const double* t, const double* bar_r, double a, double b,
                                double c, int64_t n, int64_t row0, int64_t nrows, double* hi, double* comp) {
    POLY_VJP_ROWS(double, d)
}

void hko_poly_loss_vjp_rows_f32(const float* x, const float* t, const float* bar_r, float a, float b, float c,
                                int64_t n, int64_t row0, int64_t nrows, float* hi, float* comp) {
    POLY_VJP_ROWS(float, f)
}

/* The rows of one column of per-sample terms (the host sample-sum frame,
 * hawk/emit/host.py:1499-1530, around any body): 32 slots per row, a slot
 * past the last sample holding the identity of the op (0, -inf, +inf), the
 * slots joined by sampleSumRow_'s pairs (hawk/emit/wrapper.py:561-592); max
 * and min ignore a NaN operand (ssExtreme_, :544-550). */
static double extreme_d(int op, double a, double b) {
    if (a != a) return b;
    if (b != b) return a;
    return op == HKO_OP_MAX ? (b > a ? b : a) : (b < a ? b : a);
}

void hko_rows_f64(int op, const double* terms, int64_t n, double* hi, double* comp) {
    const int64_t nrows = (n + 31) / 32;
    const double ident = op == HKO_OP_SUM ? 0.0 : (op == HKO_OP_MAX ? -INFINITY : INFINITY);
    for (int64_t j = 0; j < nrows; ++j) {
        double h[32], c[32];
        for (int l = 0; l < 32; ++l) {
            const int64_t i = j * 32 + l;
            h[l] = i < n ? terms[i] : ident;
            c[l] = 0.0;
        }
        for (int off = 16; off >= 1; off >>= 1)
            for (int l = 0; l < off; ++l) {
                if (op == HKO_OP_SUM) pair_d(&h[l], &c[l], h[l + off], c[l + off]);
                else h[l] = extreme_d(op, h[l], h[l + off]);
            }
        hi[j] = h[0];
        comp[j] = c[0];
    }
}

/*
 * hawk/_cells.py:94-119 -- leaves of 4096 rows: slot s of 256 walks rows
 * s, s+256, ... with a Neumaier step (_neumaier, :52-55), then a halving tree
 * over the slots (_pair, :58-60); then pairwise levels over the leaves, an odd
 * last one carried; hi + comp at the root for a sum.  Max/min keep `a > b ? a : b`
 * (`a < b ? a : b`) on both node kinds.
 */
#define DEFINE_FINISH(T, SUF)                                                              \
    static void nadd_##SUF(int op, T* h, T* c, T x, T xc) {                               \
        if (op == HKO_OP_MAX) { *h = (*h > x) ? *h : x; return; }                          \
        if (op == HKO_OP_MIN) { *h = (*h < x) ? *h : x; return; }                          \
        const T s = *h + x;                                                                \
        const int f = finite_##SUF(s);                                                     \
        *c = f ? *c + two_sum_err_##SUF(*h, x, s) : (T)0;                                  \
        *c = f ? *c + xc : (T)0;                                                           \
        *h = s;                                                                            \
    }                                                                                      \
    static void join_##SUF(int op, T* h, T* c, T x, T xc) {                               \
        if (op == HKO_OP_MAX) { *h = (*h > x) ? *h : x; return; }                          \
        if (op == HKO_OP_MIN) { *h = (*h < x) ? *h : x; return; }                          \
        const T s = *h + x;                                                                \
        *c = finite_##SUF(s) ? (*c + xc) + two_sum_err_##SUF(*h, x, s) : (T)0;             \
        *h = s;                                                                            \
    }                                                                                      \
    void hko_cells_leaves_##SUF(int op, const T* hi, const T* comp, int64_t n, T* lh, T* lc) {  \
        const int64_t leaves = (n + 4095) / 4096;                                          \
        for (int64_t L = 0; L < leaves; ++L) {                                             \
            const int64_t r0 = L * 4096;                                                   \
            const int64_t cnt = (n - r0) < 4096 ? (n - r0) : 4096;                         \
            const int live = (int)(cnt < 256 ? cnt : 256);                                 \
            T sh[256], sc[256];                                                            \
            for (int s = 0; s < live; ++s) {                                               \
                sh[s] = hi[r0 + s];                                                        \
                sc[s] = (op == HKO_OP_SUM && comp) ? comp[r0 + s] : (T)0;                  \
                if (!finite_##SUF(sh[s])) sc[s] = 0;                                       \
            }                                                                              \
            for (int k = 1; k < 16; ++k) {                                                 \
                const int64_t rest = cnt - (int64_t)k * 256;                               \
                const int m = (int)(rest < live ? rest : live);                            \
                if (m <= 0) break;                                                         \
                for (int s = 0; s < m; ++s) {                                              \
                    const int64_t r = r0 + (int64_t)k * 256 + s;                           \
                    nadd_##SUF(op, &sh[s], &sc[s], hi[r],                                  \
                               (op == HKO_OP_SUM && comp) ? comp[r] : (T)0);               \
                }                                                                          \
            }                                                                              \
            for (int off = 128; off > 0; off >>= 1) {                                      \
                const int lim = live > off ? (off < live - off ? off : live - off) : 0;    \
                for (int s = 0; s < lim; ++s) join_##SUF(op, &sh[s], &sc[s], sh[s + off], sc[s + off]); \
            }                                                                              \
            lh[L] = sh[0];                                                                 \
            lc[L] = sc[0];                                                                 \
        }                                                                                  \
    }                                                                                      \
    T hko_cells_tree_##SUF(int op, T* lh, T* lc, int64_t leaves) {                        \
        int64_t m = leaves;                                                                \
        while (m > 1) {                                                                    \
            const int64_t pairs = m / 2;                                                   \
            for (int64_t j = 0; j < pairs; ++j) {                                          \
                T h = lh[2 * j], c = lc[2 * j];                                            \
                join_##SUF(op, &h, &c, lh[2 * j + 1], lc[2 * j + 1]);                      \
                lh[j] = h;                                                                 \
                lc[j] = c;                                                                 \
            }                                                                              \
            if (m & 1) { lh[pairs] = lh[m - 1]; lc[pairs] = lc[m - 1]; }                   \
            m = pairs + (m & 1);                                                           \
        }                                                                                  \
        if (op == HKO_OP_SUM) return finite_##SUF(lh[0]) ? lh[0] + lc[0] : lh[0];          \
        return lh[0];                                                                      \
    }                                                                                      \
    T hko_cells_finish_##SUF##_impl(int op, const T* hi, const T* comp, int64_t n) {       \
        const int64_t leaves = (n + 4095) / 4096;                                          \
        T* lh = (T*)malloc(sizeof(T) * (size_t)(leaves > 0 ? leaves : 1));                 \
        T* lc = (T*)malloc(sizeof(T) * (size_t)(leaves > 0 ? leaves : 1));                 \
        hko_cells_leaves_##SUF(op, hi, comp, n, lh, lc);                                   \
        const T root = hko_cells_tree_##SUF(op, lh, lc, leaves);                           \
        free(lh);                                                                          \
        free(lc);                                                                          \
        return root;                                                                       \
    }
DEFINE_FINISH(double, d)
DEFINE_FINISH(float, f)

double hko_cells_finish_f64(int op, const double* hi, const double* comp, int64_t nrows) {
    return hko_cells_finish_d_impl(op, hi, comp, nrows);
}
float hko_cells_finish_f32(int op, const float* hi, const float* comp, int64_t nrows) {
    return hko_cells_finish_f_impl(op, hi, comp, nrows);
}

/* --------------------------------------------------------------- c3 gravity */

static double norm3(const double d[3]) { return sqrt(((d[0] * d[0]) + (d[1] * d[1])) + (d[2] * d[2])); }

/* t4 = (G*m1)*m2; t7 = r2 - r1; t8 = |t7|; f = (t4 / ((t8*t8)*t8)) * t7; u = (-t4) / t8 */
void hko_gravity(const double* r1, const double* r2, int64_t pitch, const double* m1, const double* m2,
                 double G, double* f, int64_t f_pitch, double* u, int64_t base, int64_t count) {
    for (int64_t i = base; i < base + count; ++i) {
        const double t4 = (G * m1[i]) * m2[i];
        double t7[3];
        for (int k = 0; k < 3; ++k) t7[k] = r2[k * pitch + i] - r1[k * pitch + i];
        const double t8 = norm3(t7);
        const double s = t4 / ((t8 * t8) * t8);
        for (int k = 0; k < 3; ++k) f[k * f_pitch + i] = s * t7[k];
        u[i] = (-t4) / t8;
    }
}

/*
 * t15 = dr2 + dr1 * -1;  t17 = t7.dot(t15) / t8;
 * dot_f = (-((t11 * ((((t17*t8) + (t8*t17)) * t8) + (t9*t17))) / t10)) * t7 + t11 * t15
 * dot_u = -((((-t4) / t8) * t17) / t8)
 */
void hko_gravity_jvp(const double* r1, const double* r2, const double* dr1, const double* dr2, int64_t pitch,
                     const double* m1, const double* m2, double G, double* dot_f, int64_t f_pitch,
                     double* dot_u, int64_t base, int64_t count) {
    for (int64_t i = base; i < base + count; ++i) {
        const double t4 = (G * m1[i]) * m2[i];
        double t7[3], t15[3];
        for (int k = 0; k < 3; ++k) {
            t7[k] = r2[k * pitch + i] - r1[k * pitch + i];
            t15[k] = dr2[k * pitch + i] + (dr1[k * pitch + i] * -1.0);
        }
        const double t8 = norm3(t7);
        const double t9 = t8 * t8;
        const double t10 = t9 * t8;
        const double t11 = t4 / t10;
        const double dot = ((t7[0] * t15[0]) + (t7[1] * t15[1])) + (t7[2] * t15[2]);
        const double t17 = dot / t8;
        const double s = -((t11 * ((((t17 * t8) + (t8 * t17)) * t8) + (t9 * t17))) / t10);
        for (int k = 0; k < 3; ++k) dot_f[k * f_pitch + i] = (s * t7[k]) + (t11 * t15[k]);
        dot_u[i] = -((((-t4) / t8) * t17) / t8);
    }
}

/*
 * t24 = -((bar_f.cwiseMul(t8).sum() * t12) / t11);  t28 = (t24*t9)*t9;
 * t33 = bar_f * t12 + ((((((-((bar_u * ((-t5)/t9)) / t9)) + (t24*t10)) + t28) + t28) / t9) * t8;
 * bar_r2 = t33;  bar_r1 = t33 * -1
 */
void hko_gravity_vjp(const double* r1, const double* r2, const double* bar_f, int64_t pitch,
                     const double* bar_u, const double* m1, const double* m2, double G, double* bar_r1,
                     double* bar_r2, int64_t out_pitch, int64_t base, int64_t count) {
    for (int64_t i = base; i < base + count; ++i) {
        double bf[3], t8[3];
        for (int k = 0; k < 3; ++k) {
            bf[k] = bar_f[k * pitch + i];
            t8[k] = r2[k * pitch + i] - r1[k * pitch + i];
        }
        const double t5 = (G * m1[i]) * m2[i];
        const double t9 = norm3(t8);
        const double t10 = t9 * t9;
        const double t11 = t10 * t9;
        const double t12 = t5 / t11;
        const double cs = ((bf[0] * t8[0]) + (bf[1] * t8[1])) + (bf[2] * t8[2]);
        const double t24 = -((cs * t12) / t11);
        const double t28 = (t24 * t9) * t9;
        const double s = (((((-((bar_u[i] * ((-t5) / t9)) / t9)) + (t24 * t10)) + t28) + t28) / t9);
        for (int k = 0; k < 3; ++k) {
            const double t33 = (bf[k] * t12) + (s * t8[k]);
            bar_r2[k * out_pitch + i] = t33;
            bar_r1[k * out_pitch + i] = t33 * -1.0;
        }
    }
}

/* ------------------------------------------------------------ c4 SPD solve */

/* Cholesky of the symmetric part, column by column (hawk/embedded/linalg.py:233-271). */
static int chol6(const double a[6][6], double l[6][6]) {
    int info = 0;
    memset(l, 0, sizeof(double) * 36);
    for (int j = 0; j < 6; ++j) {
        if (info != 0) continue;
        double d = (0.5 * a[j][j]) + (0.5 * a[j][j]);
        for (int k = 0; k < j; ++k) d = d - (l[j][k] * l[j][k]);
        if (d > 0.0) {
            const double ljj = sqrt(d);
            l[j][j] = ljj;
            for (int i = j + 1; i < 6; ++i) {
                double acc = (0.5 * a[i][j]) + (0.5 * a[j][i]);
                for (int k = 0; k < j; ++k) acc = acc - (l[i][k] * l[j][k]);
                l[i][j] = acc / ljj;
            }
        } else {
            info = j + 1;
        }
    }
    return info;
}

/* cho_solve: forward sweep on L, backward on L^T, zeros on a failed factor
 * (hawk/embedded/linalg.py:443-520). */
static void cho_solve6(const double l[6][6], int info, const double b[6], double x[6]) {
    if (info != 0) {
        for (int i = 0; i < 6; ++i) x[i] = 0.0;
        return;
    }
    for (int i = 0; i < 6; ++i) {
        double acc = b[i];
        for (int j = 0; j < i; ++j) acc = acc - (l[i][j] * x[j]);
        x[i] = acc / l[i][i];
    }
    for (int r = 0; r < 6; ++r) {
        const int i = 5 - r;
        double acc = x[i];
        for (int j = i + 1; j < 6; ++j) acc = acc - (l[j][i] * x[j]);
        x[i] = acc / l[i][i];
    }
}

static void load6x6(const double* A, int64_t pitch, int64_t i, double a[6][6]) {
    for (int r = 0; r < 6; ++r)
        for (int c = 0; c < 6; ++c) a[r][c] = A[(r * 6 + c) * pitch + i];
}

void hko_spd_solve(const double* A, const double* b, int64_t pitch, double* x, int64_t x_pitch,
                   int64_t base, int64_t count) {
    for (int64_t i = base; i < base + count; ++i) {
        double a[6][6], l[6][6], bb[6], xx[6];
        load6x6(A, pitch, i, a);
        for (int k = 0; k < 6; ++k) bb[k] = b[k * pitch + i];
        const int info = chol6(a, l);
        cho_solve6(l, info, bb, xx);
        for (int k = 0; k < 6; ++k) x[k * x_pitch + i] = xx[k];
    }
}

/* la1 = cho_solve(L, bar_x) -> bar_b;  la2 = cho_solve(L, b);
 * t6 = outer(la1, la2);  bar_A = ((t6 + t6^T) * 0.5) * -1 */
void hko_spd_solve_vjp(const double* A, const double* b, const double* bar_x, int64_t pitch, double* bar_A,
                       double* bar_b, int64_t out_pitch, int64_t base, int64_t count) {
    for (int64_t i = base; i < base + count; ++i) {
        double a[6][6], l[6][6], bx[6], bb[6], la1[6], la2[6];
        load6x6(A, pitch, i, a);
        const int info = chol6(a, l);
        for (int k = 0; k < 6; ++k) {
            bx[k] = bar_x[k * pitch + i];
            bb[k] = b[k * pitch + i];
        }
        cho_solve6(l, info, bx, la1);
        for (int k = 0; k < 6; ++k) bar_b[k * out_pitch + i] = la1[k];
        cho_solve6(l, info, bb, la2);
        for (int r = 0; r < 6; ++r)
            for (int c = 0; c < 6; ++c) {
                const double t6 = la1[r] * la2[c];
                const double t6t = la1[c] * la2[r];
                bar_A[(r * 6 + c) * out_pitch + i] = ((t6 + t6t) * 0.5) * -1.0;
            }
    }
}

/* ------------------------------------------- team-form linear algebra (any n) */

/* Cholesky of the symmetric part, column by column, for any n (the order of
 * hawk/embedded/linalg.py:233-271); l is row-major n x n, zeroed first; the
 * factor as a matrix is l when info == 0, else zeros. */
static int chol_n(int n, const double* a, double* l) {
    int info = 0;
    memset(l, 0, sizeof(double) * (size_t)n * (size_t)n);
    for (int j = 0; j < n; ++j) {
        if (info != 0) continue;
        double d = (0.5 * a[j * n + j]) + (0.5 * a[j * n + j]);
        for (int k = 0; k < j; ++k) d = d - (l[j * n + k] * l[j * n + k]);
        if (d > 0.0) {
            const double ljj = sqrt(d);
            l[j * n + j] = ljj;
            for (int i = j + 1; i < n; ++i) {
                double acc = (0.5 * a[i * n + j]) + (0.5 * a[j * n + i]);
                for (int k = 0; k < j; ++k) acc = acc - (l[i * n + k] * l[j * n + k]);
                l[i * n + j] = acc / ljj;
            }
        } else {
            info = j + 1;
        }
    }
    return info;
}

/* cho_solve on k right-hand sides (row-major n x k), one column at a time:
 * forward sweep on L, backward on L^T (hawk/embedded/linalg.py:443-520). */
static void cho_solve_n(int n, const double* l, int info, const double* b, double* x, int k) {
    for (int e = 0; e < n * k; ++e) x[e] = info != 0 ? 0.0 : b[e];
    if (info != 0) return;
    for (int c = 0; c < k; ++c) {
        for (int i = 0; i < n; ++i) {
            double acc = x[i * k + c];
            for (int j = 0; j < i; ++j) acc = acc - (l[i * n + j] * x[j * k + c]);
            x[i * k + c] = acc / l[i * n + i];
        }
        for (int r = 0; r < n; ++r) {
            const int i = n - 1 - r;
            double acc = x[i * k + c];
            for (int j = i + 1; j < n; ++j) acc = acc - (l[j * n + i] * x[j * k + c]);
            x[i * k + c] = acc / l[i * n + i];
        }
    }
}

/* P A = L U, Crout, column by column; the pivot is the first row of largest
 * magnitude (hawk/embedded/linalg.py:188-231). */
static int lu_n(int n, const double* a, double* f, int32_t* piv) {
    memcpy(f, a, sizeof(double) * (size_t)n * (size_t)n);
    int info = 0;
    if (n == 1) {
        piv[0] = 0;
        return f[0] != 0.0 ? 0 : 1;
    }
    for (int j = 0; j < n; ++j) {
        for (int i = 0; i < n; ++i) {
            const int m = i < j ? i : j;
            double acc = 0.0;
            for (int k = 0; k < m; ++k) acc = acc + (f[i * n + k] * f[k * n + j]);
            f[i * n + j] = f[i * n + j] - acc;
        }
        int p = j;
        double big = fabs(f[j * n + j]);
        for (int i = j + 1; i < n; ++i) {
            const double mag = fabs(f[i * n + j]);
            if (mag > big) {
                big = mag;
                p = i;
            }
        }
        piv[j] = p;
        if (f[p * n + j] != 0.0) {
            if (p != j)
                for (int c = 0; c < n; ++c) {
                    const double t = f[j * n + c];
                    f[j * n + c] = f[p * n + c];
                    f[p * n + c] = t;
                }
            const double rcp = 1.0 / f[j * n + j];
            for (int i = j + 1; i < n; ++i) f[i * n + j] = f[i * n + j] * rcp;
        } else if (info == 0) {
            info = j + 1;
        }
    }
    return info;
}

/* lu_solve on k right-hand sides: the exchanges in step order, the unit-lower
 * forward sweep, the backward sweep on U; zeros on a failed factor. */
static void lu_solve_n(int n, const double* f, const int32_t* piv, int info, const double* b, double* x, int k) {
    for (int e = 0; e < n * k; ++e) x[e] = info != 0 ? 0.0 : b[e];
    if (info != 0) return;
    if (n > 1)
        for (int s = 0; s < n; ++s) {
            const int p = piv[s];
            if (p != s)
                for (int c = 0; c < k; ++c) {
                    const double t = x[s * k + c];
                    x[s * k + c] = x[p * k + c];
                    x[p * k + c] = t;
                }
        }
    for (int c = 0; c < k; ++c) {
        if (n > 1)
            for (int i = 0; i < n; ++i) {
                double acc = x[i * k + c];
                for (int j = 0; j < i; ++j) acc = acc - (f[i * n + j] * x[j * k + c]);
                x[i * k + c] = acc;
            }
        for (int r = 0; r < n; ++r) {
            const int i = n - 1 - r;
            double acc = x[i * k + c];
            for (int j = i + 1; j < n; ++j) acc = acc - (f[i * n + j] * x[j * k + c]);
            x[i * k + c] = acc / f[i * n + i];
        }
    }
}

/* det from the factor: U's diagonal product, negated per exchange as it is met
 * (hawk/embedded/linalg.py:402-418); 0 on a failed factor. */
static double lu_det_n(int n, const double* f, const int32_t* piv, int info) {
    if (info != 0) return 0.0;
    double d = 1.0;
    for (int k = 0; k < n; ++k) {
        d = d * f[k * n + k];
        if (piv[k] != k) d = -d;
    }
    return d;
}

static void load_nxm(const double* P, int64_t pitch, int64_t i, int r, int c, double* out) {
    for (int e = 0; e < r * c; ++e) out[e] = P[(int64_t)e * pitch + i];
}

static void store_nxm(double* P, int64_t pitch, int64_t i, int r, int c, const double* in) {
    for (int e = 0; e < r * c; ++e) P[(int64_t)e * pitch + i] = in[e];
}

void hko_team_chol(int n, const double* A, const double* b, const double* B, int64_t pitch, double* x, double* X,
                   double* L, int32_t* info, int64_t base, int64_t count) {
    double* a = malloc(sizeof(double) * (size_t)n * (size_t)n);
    double* l = malloc(sizeof(double) * (size_t)n * (size_t)n);
    double* v = malloc(sizeof(double) * (size_t)n * 2);
    double* y = malloc(sizeof(double) * (size_t)n * 2);
    for (int64_t i = base; i < base + count; ++i) {
        load_nxm(A, pitch, i, n, n, a);
        const int inf = chol_n(n, a, l);
        load_nxm(b, pitch, i, n, 1, v);
        cho_solve_n(n, l, inf, v, y, 1);
        store_nxm(x, pitch, i, n, 1, y);
        load_nxm(B, pitch, i, n, 2, v);
        cho_solve_n(n, l, inf, v, y, 2);
        store_nxm(X, pitch, i, n, 2, y);
        if (inf != 0) memset(l, 0, sizeof(double) * (size_t)n * (size_t)n);
        store_nxm(L, pitch, i, n, n, l);
        info[i] = inf;
    }
    free(a);
    free(l);
    free(v);
    free(y);
}

void hko_team_lu(int n, const double* A, const double* b, const double* B, int64_t pitch, double* x, double* X,
                 double* det, int32_t* info, int64_t base, int64_t count) {
    double* a = malloc(sizeof(double) * (size_t)n * (size_t)n);
    double* f = malloc(sizeof(double) * (size_t)n * (size_t)n);
    int32_t* piv = malloc(sizeof(int32_t) * (size_t)n);
    double* v = malloc(sizeof(double) * (size_t)n * 2);
    double* y = malloc(sizeof(double) * (size_t)n * 2);
    for (int64_t i = base; i < base + count; ++i) {
        load_nxm(A, pitch, i, n, n, a);
        const int inf = lu_n(n, a, f, piv);
        load_nxm(b, pitch, i, n, 1, v);
        lu_solve_n(n, f, piv, inf, v, y, 1);
        store_nxm(x, pitch, i, n, 1, y);
        load_nxm(B, pitch, i, n, 2, v);
        lu_solve_n(n, f, piv, inf, v, y, 2);
        store_nxm(X, pitch, i, n, 2, y);
        det[i] = lu_det_n(n, f, piv, inf);
        info[i] = inf;
    }
    free(a);
    free(f);
    free(piv);
    free(v);
    free(y);
}

/* chol_from: the lower triangle of A is the factor; info = first column whose
 * diagonal is not positive and finite (hawk/embedded/linalg.py:274-299). */
void hko_team_chol_from(int n, const double* A, const double* b, int64_t pitch, double* x, double* L,
                        int32_t* info, int64_t base, int64_t count) {
    double* a = malloc(sizeof(double) * (size_t)n * (size_t)n);
    double* l = malloc(sizeof(double) * (size_t)n * (size_t)n);
    double* v = malloc(sizeof(double) * (size_t)n);
    double* y = malloc(sizeof(double) * (size_t)n);
    for (int64_t i = base; i < base + count; ++i) {
        load_nxm(A, pitch, i, n, n, a);
        int inf = 0;
        for (int j = 0; j < n && inf == 0; ++j) {
            const double d = a[j * n + j];
            if ((d <= 0.0) || !isfinite(d)) inf = j + 1;
        }
        for (int r = 0; r < n; ++r)
            for (int c = 0; c < n; ++c) l[r * n + c] = (inf == 0 && c <= r) ? a[r * n + c] : 0.0;
        load_nxm(b, pitch, i, n, 1, v);
        cho_solve_n(n, l, inf, v, y, 1);
        store_nxm(x, pitch, i, n, 1, y);
        store_nxm(L, pitch, i, n, n, l);
        info[i] = inf;
    }
    free(a);
    free(l);
    free(v);
    free(y);
}

/* ---------------------------------------------- symmetric eigenproblem (any n) */

static int eigh_sweeps(int n) { return n <= 2 ? 2 : n <= 4 ? 6 : n <= 8 ? 8 : n <= 16 ? 12 : 15; }

/* Cyclic Jacobi on the symmetric part, hawk/embedded/linalg.py:302-399:
 * w ascending, V's columns the eigenvectors (first largest component
 * positive), info bit 1 / bit 2 as restated there. */
static int eigh_n(int n, const double* a, double* w, double* v) {
    const double eps = 2.220446049250313e-16;
    int info = 0;
    if (n == 1) {
        w[0] = a[0];
        v[0] = 1.0;
        return 0;
    }
    double* s = malloc(sizeof(double) * (size_t)n * (size_t)n);
    double fro2 = 0.0;
    for (int e = 0; e < n * n; ++e) v[e] = 0.0;
    for (int i = 0; i < n; ++i) {
        for (int j = 0; j < n; ++j) {
            if (j >= i) s[i * n + j] = (0.5 * a[i * n + j]) + (0.5 * a[j * n + i]);
            else s[i * n + j] = s[j * n + i];
            fro2 = fro2 + (s[i * n + j] * s[i * n + j]);
        }
        v[i * n + i] = 1.0;
    }
    for (int sweep = 0; sweep < eigh_sweeps(n); ++sweep)
        for (int p = 0; p < n - 1; ++p)
            for (int q = p + 1; q < n; ++q) {
                const double app = s[p * n + p], aqq = s[q * n + q], apq = s[p * n + q];
                if (!(fabs(apq) <= (eps * sqrt(fabs(app * aqq))))) {
                    const double theta = (aqq - app) / (2.0 * apq);
                    const double sg = (theta < 0.0) ? -1.0 : 1.0;
                    const double tn = sg / (fabs(theta) + sqrt((theta * theta) + 1.0));
                    const double cs = 1.0 / sqrt((tn * tn) + 1.0);
                    const double sn = tn * cs;
                    s[p * n + p] = app - (tn * apq);
                    s[q * n + q] = aqq + (tn * apq);
                    s[p * n + q] = 0.0;
                    s[q * n + p] = 0.0;
                    for (int k = 0; k < n; ++k) {
                        if ((k != p) && (k != q)) {
                            const double akp = s[k * n + p], akq = s[k * n + q];
                            const double np = (cs * akp) - (sn * akq);
                            const double nq = (sn * akp) + (cs * akq);
                            s[k * n + p] = np;
                            s[p * n + k] = np;
                            s[k * n + q] = nq;
                            s[q * n + k] = nq;
                        }
                        const double vp = v[k * n + p], vq = v[k * n + q];
                        v[k * n + p] = (cs * vp) - (sn * vq);
                        v[k * n + q] = (sn * vp) + (cs * vq);
                    }
                }
            }
    double off2 = 0.0;
    for (int i = 0; i < n; ++i) {
        w[i] = s[i * n + i];
        for (int j = 0; j < n; ++j)
            if (j != i) off2 = off2 + (s[i * n + j] * s[i * n + j]);
    }
    const double tol = (double)n * eps;
    if (!(off2 <= ((tol * tol) * fro2))) info = 1;
    for (int i = 0; i < n - 1; ++i) {
        int lo = i;
        for (int j = i + 1; j < n; ++j)
            if (w[j] < w[lo]) lo = j;
        if (lo != i) {
            const double tw = w[i];
            w[i] = w[lo];
            w[lo] = tw;
            for (int k = 0; k < n; ++k) {
                const double tv = v[k * n + i];
                v[k * n + i] = v[k * n + lo];
                v[k * n + lo] = tv;
            }
        }
    }
    for (int j = 0; j < n; ++j) {
        int big = 0;
        for (int k = 1; k < n; ++k)
            if (fabs(v[k * n + j]) > fabs(v[big * n + j])) big = k;
        if (v[big * n + j] < 0.0)
            for (int k = 0; k < n; ++k) v[k * n + j] = -v[k * n + j];
    }
    const double gap = tol * sqrt(fro2);
    int tight = 0;
    for (int i = 0; i < n - 1; ++i)
        if (!((w[i + 1] - w[i]) > gap)) tight = 1;
    if (tight) info = info + 2;
    free(s);
    return info;
}

void hko_sym_eigen(int n, const double* A, int64_t pitch, double* w, double* V, int32_t* info, int64_t base,
                   int64_t count) {
    double* a = malloc(sizeof(double) * (size_t)n * (size_t)n);
    double* vv = malloc(sizeof(double) * (size_t)n * (size_t)n);
    double* ww = malloc(sizeof(double) * (size_t)n);
    for (int64_t i = base; i < base + count; ++i) {
        load_nxm(A, pitch, i, n, n, a);
        info[i] = eigh_n(n, a, ww, vv);
        store_nxm(w, pitch, i, n, 1, ww);
        if (V) store_nxm(V, pitch, i, n, n, vv);
    }
    free(a);
    free(vv);
    free(ww);
}

/* ------------------------------------------------- QR least squares (n > 32) */

/* The b200 team-form Householder QR and its solve, restated (hk/team.cuh qr,
 * qrSolve): the reference's own team QR (aether-dsc) is absent, so this order
 * is the build's; the tests pin it against numpy's least squares. */
static int qr_n(int m, int n, double* a, double* tau, double* v0s) {
    int info = 0;
    for (int j = 0; j < n; ++j) {
        double norm2 = 0.0;
        for (int i = j; i < m; ++i) norm2 = norm2 + (a[i * n + j] * a[i * n + j]);
        const double ajj = a[j * n + j];
        if (!(norm2 > 0.0)) {
            if (info == 0) info = j + 1;
            tau[j] = 0.0;
            v0s[j] = 0.0;
            continue;
        }
        const double norm = sqrt(norm2);
        const double alpha = (ajj >= 0.0) ? -norm : norm;
        const double v0 = ajj - alpha;
        double vtv = v0 * v0;
        for (int i = j + 1; i < m; ++i) vtv = vtv + (a[i * n + j] * a[i * n + j]);
        const double tj = 2.0 / vtv;
        for (int c = j + 1; c < n; ++c) {
            double d = v0 * a[j * n + c];
            for (int i = j + 1; i < m; ++i) d = d + (a[i * n + j] * a[i * n + c]);
            const double t = tj * d;
            a[j * n + c] = a[j * n + c] - (t * v0);
            for (int i = j + 1; i < m; ++i) a[i * n + c] = a[i * n + c] - (t * a[i * n + j]);
        }
        a[j * n + j] = alpha;
        tau[j] = tj;
        v0s[j] = v0;
    }
    return info;
}

void hko_lstsq_qr(int m, int n, const double* J, const double* r, int64_t pitch, double* x, int32_t* info,
                  int64_t base, int64_t count) {
    double* a = malloc(sizeof(double) * (size_t)m * (size_t)n);
    double* y = malloc(sizeof(double) * (size_t)m);
    double* tau = malloc(sizeof(double) * (size_t)n);
    double* v0 = malloc(sizeof(double) * (size_t)n);
    double* xx = malloc(sizeof(double) * (size_t)n);
    for (int64_t s = base; s < base + count; ++s) {
        load_nxm(J, pitch, s, m, n, a);
        load_nxm(r, pitch, s, m, 1, y);
        const int inf = qr_n(m, n, a, tau, v0);
        if (inf != 0) {
            for (int i = 0; i < n; ++i) xx[i] = 0.0;
        } else {
            for (int j = 0; j < n; ++j) {
                double d = v0[j] * y[j];
                for (int i = j + 1; i < m; ++i) d = d + (a[i * n + j] * y[i]);
                const double t = tau[j] * d;
                y[j] = y[j] - (t * v0[j]);
                for (int i = j + 1; i < m; ++i) y[i] = y[i] - (t * a[i * n + j]);
            }
            for (int q = 0; q < n; ++q) {
                const int i = n - 1 - q;
                double acc = y[i];
                for (int jj = i + 1; jj < n; ++jj) acc = acc - (a[i * n + jj] * xx[jj]);
                xx[i] = acc / a[i * n + i];
            }
        }
        store_nxm(x, pitch, s, n, 1, xx);
        info[s] = inf;
    }
    free(a);
    free(y);
    free(tau);
    free(v0);
    free(xx);
}

/* ---------------------------------------------------------------- c5 Kepler */

/*
 * E = M, n = 0; up to 32 trips:
 *   tb0 = ((E - (e * sin E)) - M) / (1 - (e * cos E));  E' = E - tb0;  n' = n + 1;
 *   leave after the trip when |tb0| < 1e-14.
 */
/* s = sin(x); c = cos(x) */
void hko_trig(const double* x, double* s, double* c, int64_t base, int64_t count) {
    for (int64_t i = base; i < base + count; ++i) {
        s[i] = o_sin(x[i]);
        c[i] = o_cos(x[i]);
    }
}

void hko_kepler(const double* e, const double* M, double* E, int32_t* iters, int64_t base, int64_t count) {
    for (int64_t i = base; i < base + count; ++i) {
        const double Mi = M[i], ei = e[i];
        double Ek = Mi;
        int32_t n = 0;
        for (int k = 0; k < 32; ++k) {
            const double tb0 = ((Ek - (ei * o_sin(Ek))) - Mi) / (1.0 - (ei * o_cos(Ek)));
            const double tb1 = fabs(tb0);
            const double nE = Ek - tb0;
            const int32_t nn = (int32_t)((uint32_t)n + 1u);
            const int x = tb1 < 1e-14;
            Ek = nE;
            n = nn;
            if (x) break;
        }
        E[i] = Ek;
        iters[i] = n;
    }
}

/*
 * The forward loop with its tape (E at the start of each trip) and trip count
 * c, then the reverse loop over the trips taken, k = c - 1 .. 0, as the
 * reference's reverse_loop renders it (hawk/diff/loops.py:384):
 *   tb2 = -bE; tb3 = tape[k]; tb4 = sin tb3; tb5 = cos tb3; tb6 = 1 - e tb5;
 *   tb7 = -(-((tb2 * (((tb3 - e tb4) - M) / tb6)) / tb6)); tb8 = tb2 / tb6;
 *   tb9 = (bE + ((tb7 e) * (-sin tb3))) + tb8; tb10 = -tb8; tb11 = (tb10 e) cos tb3;
 *   tb13 = (tb7 tb5) + (tb10 tb4); bE = tb9 + tb11; bM += -tb8; be += tb13
 * bar_M = bE + bM, bar_e = be.
 */
void hko_kepler_vjp(const double* e, const double* M, const double* bar_E, double* bar_e, double* bar_M,
                    int64_t base, int64_t count) {
    for (int64_t i = base; i < base + count; ++i) {
        const double Mi = M[i], ei = e[i];
        double tape[32];
        double Ek = Mi;
        int64_t c = 0;
        for (int k = 0; k < 32; ++k) {
            tape[k] = Ek;
            const double tb0 = ((Ek - (ei * o_sin(Ek))) - Mi) / (1.0 - (ei * o_cos(Ek)));
            const double tb1 = fabs(tb0);
            const double nE = Ek - tb0;
            const int x = tb1 < 1e-14;
            Ek = nE;
            ++c;
            if (x) break;
        }
        double bE = bar_E[i], bM = 0.0, be = 0.0;
        for (int k = (int)(31 - (32 - c) * 1); k > -1; --k) {
            const double tb2 = -bE;
            const double tb3 = tape[k];
            const double tb4 = o_sin(tb3);
            const double tb5 = o_cos(tb3);
            const double tb6 = 1.0 - (ei * tb5);
            const double tb7 = -(-((tb2 * (((tb3 - (ei * tb4)) - Mi) / tb6)) / tb6));
            const double tb8 = tb2 / tb6;
            const double tb9 = (bE + ((tb7 * ei) * (-o_sin(tb3)))) + tb8;
            const double tb10 = -tb8;
            const double tb11 = (tb10 * ei) * o_cos(tb3);
            const double tb12 = -tb8;
            const double tb13 = (tb7 * tb5) + (tb10 * tb4);
            bE = tb9 + tb11;
            bM = bM + tb12;
            be = be + tb13;
        }
        bar_M[i] = bE + bM;
        bar_e[i] = be;
    }
}

/* ------------------------------------------------------ stepping kernels
 *
 * An automatic kernel (steps="auto", hawk/trace/steps.py) run by the host
 * target's two-path entry (hawk/emit/wrapper.py:1507-1545): a sample finished
 * on entry is skipped; the fused_steps word 1 runs the single step, any other
 * word max(word, 0) trips (at most INT_MAX, hawk_clamp_count) of the fused loop,
 * leaving after the trip whose finish condition holds (a tail break); the
 * carried values commit to the planes after the loop, and a sample whose
 * carried finish flag is set is marked in the mask and counted (one count per
 * newly finished sample).  The single step and one trip of the fused loop are
 * the same operations, so one trip function serves both.  Each function
 * returns the samples it newly finished in [base, base + count).
 */
static int64_t clamp_trips(int64_t word) {
    if (word == 1) return 1;
    if (word < 0) return 0;
    return word < 2147483647LL ? word : 2147483647LL;
}

/*
 * s1 oscillator, one trip:
 *   t3 = dt * 0.16666666666666666; t7 = 0.5 * dt; t10 = -(w*w); t14 = (2 z) w;
 *   t16 = t10 x - t14 v; t18 = v + t7 t16; t23 = t10 (x + t7 v) - t14 t18;
 *   t25 = v + t7 t23; t33 = t10 (x + t7 t18) - t14 t25; t35 = v + dt t33;
 *   x' = x + t3 ((v + 2 (t18 + t25)) + t35);
 *   v' = v + t3 ((t16 + 2 (t23 + t33)) + (t10 (x + dt t25) - t14 t35));
 *   k' = k + 1; finished when k' >= nstop.
 */
uint32_t hko_oscillator(double* x, double* v, double* k, const double* nstop, const double* omega,
                        const double* zeta, uint8_t* term, double dt, int64_t word, int64_t base,
                        int64_t count) {
    uint32_t fin = 0;
    const int64_t trips = clamp_trips(word);
    const double t3 = dt * 0.16666666666666666, t7 = 0.5 * dt;
    for (int64_t i = base; i < base + count; ++i) {
        if (term[i]) continue;
        const double w = omega[i];
        const double t10 = -(w * w);
        const double t14 = (2.0 * zeta[i]) * w;
        double xs = x[i], vs = v[i], ks = k[i];
        int done = 0;
        for (int64_t trip = 0; trip < trips; ++trip) {
            const double t16 = (t10 * xs) - (t14 * vs);
            const double t18 = vs + (t7 * t16);
            const double t23 = (t10 * (xs + (t7 * vs))) - (t14 * t18);
            const double t25 = vs + (t7 * t23);
            const double t33 = (t10 * (xs + (t7 * t18))) - (t14 * t25);
            const double t35 = vs + (dt * t33);
            const double nx = xs + (t3 * ((vs + (2.0 * (t18 + t25))) + t35));
            const double nv = vs + (t3 * ((t16 + (2.0 * (t23 + t33))) + ((t10 * (xs + (dt * t25))) - (t14 * t35))));
            const double nk = ks + 1.0;
            done = nk >= nstop[i];
            xs = nx;
            vs = nv;
            ks = nk;
            if (done) break;
        }
        x[i] = xs;
        v[i] = vs;
        k[i] = ks;
        if (done) {
            term[i] = 1;
            ++fin;
        }
    }
    return fin;
}

/* Fehlberg's 7(8) pair: stage rows, the 8th-order weights and the error signs
 * (hawk_b200/configs.py states the same table). */
static const double RKF_A[12][12] = {
    {2.0 / 27.0},
    {1.0 / 36.0, 1.0 / 12.0},
    {1.0 / 24.0, 0.0, 1.0 / 8.0},
    {5.0 / 12.0, 0.0, -25.0 / 16.0, 25.0 / 16.0},
    {1.0 / 20.0, 0.0, 0.0, 1.0 / 4.0, 1.0 / 5.0},
    {-25.0 / 108.0, 0.0, 0.0, 125.0 / 108.0, -65.0 / 27.0, 125.0 / 54.0},
    {31.0 / 300.0, 0.0, 0.0, 0.0, 61.0 / 225.0, -2.0 / 9.0, 13.0 / 900.0},
    {2.0, 0.0, 0.0, -53.0 / 6.0, 704.0 / 45.0, -107.0 / 9.0, 67.0 / 90.0, 3.0},
    {-91.0 / 108.0, 0.0, 0.0, 23.0 / 108.0, -976.0 / 135.0, 311.0 / 54.0, -19.0 / 60.0, 17.0 / 6.0, -1.0 / 12.0},
    {2383.0 / 4100.0, 0.0, 0.0, -341.0 / 164.0, 4496.0 / 1025.0, -301.0 / 82.0, 2133.0 / 4100.0, 45.0 / 82.0,
     45.0 / 164.0, 18.0 / 41.0},
    {3.0 / 205.0, 0.0, 0.0, 0.0, 0.0, -6.0 / 41.0, -3.0 / 205.0, -3.0 / 41.0, 3.0 / 41.0, 6.0 / 41.0, 0.0},
    {-1777.0 / 4100.0, 0.0, 0.0, -341.0 / 164.0, 4496.0 / 1025.0, -289.0 / 82.0, 2193.0 / 4100.0, 51.0 / 82.0,
     33.0 / 164.0, 12.0 / 41.0, 0.0, 1.0},
};
static const int RKF_BJ[7] = {5, 6, 7, 8, 9, 11, 12};
static const double RKF_BW[7] = {34.0 / 105.0, 9.0 / 35.0, 9.0 / 35.0, 9.0 / 280.0, 9.0 / 280.0,
                                 41.0 / 840.0, 41.0 / 840.0};

/* The two-body rate (GM = 1): rr = (x x + y y) + z z; w = 1 / (rr sqrt rr). */
static void orbit_rate(const double s[6], double out[6]) {
    const double rr = ((s[0] * s[0]) + (s[1] * s[1])) + (s[2] * s[2]);
    const double w = 1.0 / (rr * sqrt(rr));
    out[0] = s[3];
    out[1] = s[4];
    out[2] = s[5];
    out[3] = -(s[0] * w);
    out[4] = -(s[1] * w);
    out[5] = -(s[2] * w);
}

/*
 * s2 orbit, one trip (an adaptive Fehlberg 7(8) attempt):
 *   rest = t_end - t; final = h >= rest; step = final ? rest : h;
 *   stage j: y = s + step * (sum_l a_jl k_l over the nonzero a_jl, in l order);
 *   s8 = s + step * (sum of the 8th-order weights' terms); err_d = (step 41/840) *
 *   (((1 k0 + 1 k10) + -1 k11) + -1 k12); worst = fmax over d of
 *   |err_d| / (1e-10 + 1e-10 fmax(|s8_d|, |s_d|)); ok = worst < 1;
 *   h' = step fmin(5, fmax(0.2, 0.9 (1 / sqrt(sqrt(sqrt worst)))));
 *   s' = ok ? s8 : s; t' = ok ? (final ? t_end : t + step) : t;
 *   n_acc += ok ? 1 : 0; n_rej += ok ? 0 : 1; finished when t' >= t_end.
 */
static int orbit_trip(double s[6], double* t, double* h, double* na, double* nr, double t_end) {
    const double rest = t_end - *t;
    const int final = *h >= rest;
    const double step = final ? rest : *h;
    double k[13][6], y[6];
    orbit_rate(s, k[0]);
    for (int j = 0; j < 12; ++j) {
        for (int d = 0; d < 6; ++d) {
            double acc = 0.0;
            int any = 0;
            for (int l = 0; l <= j; ++l) {
                if (RKF_A[j][l] == 0.0) continue;
                const double term = RKF_A[j][l] * k[l][d];
                acc = any ? acc + term : term;
                any = 1;
            }
            y[d] = s[d] + (step * acc);
        }
        orbit_rate(y, k[j + 1]);
    }
    double s8[6], worst = 0.0;
    const double he = step * (41.0 / 840.0);
    for (int d = 0; d < 6; ++d) {
        double acc = RKF_BW[0] * k[RKF_BJ[0]][d];
        for (int m = 1; m < 7; ++m) acc = acc + (RKF_BW[m] * k[RKF_BJ[m]][d]);
        s8[d] = s[d] + (step * acc);
        const double e = he * ((((1.0 * k[0][d]) + (1.0 * k[10][d])) + (-1.0 * k[11][d])) + (-1.0 * k[12][d]));
        const double q = fabs(e) / (1e-10 + (1e-10 * fmax(fabs(s8[d]), fabs(s[d]))));
        worst = d == 0 ? q : fmax(worst, q);
    }
    const int ok = worst < 1.0;
    const double shrink = 1.0 / sqrt(sqrt(sqrt(worst)));
    *h = step * fmin(5.0, fmax(0.2, 0.9 * shrink));
    if (ok)
        for (int d = 0; d < 6; ++d) s[d] = s8[d];
    const double tn = ok ? (final ? t_end : *t + step) : *t;
    *t = tn;
    *na = *na + (ok ? 1.0 : 0.0);
    *nr = *nr + (ok ? 0.0 : 1.0);
    return tn >= t_end;
}

uint32_t hko_orbit(double* s, int64_t pitch, double* t, double* h, double* n_acc, double* n_rej,
                   const double* t_end, uint8_t* term, int64_t word, int64_t base, int64_t count) {
    uint32_t fin = 0;
    const int64_t trips = clamp_trips(word);
    for (int64_t i = base; i < base + count; ++i) {
        if (term[i]) continue;
        double st[6];
        for (int d = 0; d < 6; ++d) st[d] = s[d * pitch + i];
        double ts = t[i], hs = h[i], na = n_acc[i], nr = n_rej[i];
        int done = 0;
        for (int64_t trip = 0; trip < trips; ++trip) {
            done = orbit_trip(st, &ts, &hs, &na, &nr, t_end[i]);
            if (done) break;
        }
        for (int d = 0; d < 6; ++d) s[d * pitch + i] = st[d];
        t[i] = ts;
        h[i] = hs;
        n_acc[i] = na;
        n_rej[i] = nr;
        if (done) {
            term[i] = 1;
            ++fin;
        }
    }
    return fin;
}
