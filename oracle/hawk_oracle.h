/*
 * hawk_oracle.h -- TEST INFRASTRUCTURE ONLY: the CPU restatement of the
 * reference's host target for the five benchmark kernels.
 *
 * Only the test suite, the smoke check and the benchmark's CPU-baseline leg
 * use this library, as the checker; the b200 product never links or calls it.
 *
 * Every function computes what the reference's emitted host unit computes for
 * the kernel (the serial loop of hawk/emit/host.py:1386-1495 around the body
 * the reference renderer writes, hawk/emit/render.py:140), in the same order of
 * floating-point operations, over samples [base, base + count).  Planes are
 * component-major: component k of sample i of a vector plane is v[k * pitch + i].
 *
 * Math: the reference's host build calls glibc's sin/cos (its host profile
 * equals glibc bit for bit, tests/test_math_parity.py:4-14), and so does this
 * library: the host's own libm, the reference host target's math exactly.
 */
#ifndef HAWK_ORACLE_H
#define HAWK_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HKO_OP_SUM 0
#define HKO_OP_MAX 1
#define HKO_OP_MIN 2

/* c1: out = 0.5 * dot(v, v) */
void hko_energy(const double* v, int64_t pitch, double* out, int64_t base, int64_t count);
void hko_energy_vjp(const double* v, int64_t pitch, const double* bar_out, double* bar_v, int64_t bar_pitch,
                    int64_t base, int64_t count);
void hko_energy_jvp(const double* v, int64_t pitch, const double* dot_v, int64_t dot_pitch, double* dot_out,
                    int64_t base, int64_t count);

/* c2: r = (a x^3 + b x + c - t)^2, and the row terms of its Param VJP */
void hko_poly_loss_f64(const double* x, const double* t, double a, double b, double c, double* r,
                       int64_t base, int64_t count);
void hko_poly_loss_f32(const float* x, const float* t, float a, float b, float c, float* r,
                       int64_t base, int64_t count);
/* rows (hi, comp) of the 3 gradient columns for rows [row0, row0 + nrows): hi[k * nrows + j] */
void hko_poly_loss_vjp_rows_f64(const double* x, const double* t, const double* bar_r, double a, double b,
                                double c, int64_t n, int64_t row0, int64_t nrows, double* hi, double* comp);
void hko_poly_loss_vjp_rows_f32(const float* x, const float* t, const float* bar_r, float a, float b, float c,
                                int64_t n, int64_t row0, int64_t nrows, float* hi, float* comp);

/* the ordered finish of hawk/_cells.py over nrows rows; and its two stages: one
 * (hi, comp) partial per leaf of 4096 rows, then the pairwise levels (the leaf
 * arrays are overwritten) and hi + comp */
void hko_cells_leaves_d(int op, const double* hi, const double* comp, int64_t nrows, double* leaf_hi,
                        double* leaf_comp);
double hko_cells_tree_d(int op, double* leaf_hi, double* leaf_comp, int64_t leaves);
double hko_cells_finish_f64(int op, const double* hi, const double* comp, int64_t nrows);
float hko_cells_finish_f32(int op, const float* hi, const float* comp, int64_t nrows);

/* c3: two-body gravity, its JVP and VJP */
void hko_gravity(const double* r1, const double* r2, int64_t pitch, const double* m1, const double* m2,
                 double G, double* f, int64_t f_pitch, double* u, int64_t base, int64_t count);
void hko_gravity_jvp(const double* r1, const double* r2, const double* dr1, const double* dr2, int64_t pitch,
                     const double* m1, const double* m2, double G, double* dot_f, int64_t f_pitch,
                     double* dot_u, int64_t base, int64_t count);
void hko_gravity_vjp(const double* r1, const double* r2, const double* bar_f, int64_t pitch,
                     const double* bar_u, const double* m1, const double* m2, double G, double* bar_r1,
                     double* bar_r2, int64_t out_pitch, int64_t base, int64_t count);

/* c4: x = cho_solve(cholesky(A), b) for 6x6 A, and its VJP */
void hko_spd_solve(const double* A, const double* b, int64_t pitch, double* x, int64_t x_pitch,
                   int64_t base, int64_t count);
void hko_spd_solve_vjp(const double* A, const double* b, const double* bar_x, int64_t pitch, double* bar_A,
                       double* bar_b, int64_t out_pitch, int64_t base, int64_t count);

/* c5: Kepler's equation by Newton, and its VJP through the loop */
void hko_kepler(const double* e, const double* M, double* E, int32_t* iters, int64_t base, int64_t count);
/* trig: s = sin(x), c = cos(x) (the host target's libm) */
void hko_trig(const double* x, double* s, double* c, int64_t base, int64_t count);
void hko_kepler_vjp(const double* e, const double* M, const double* bar_E, double* bar_e, double* bar_M,
                    int64_t base, int64_t count);

/* Stepping kernels (automatic: the fused_steps word `word`; hawk/trace/steps.py):
 * advance the samples of [base, base + count) not finished on entry, mark and
 * count the ones that finish; returns that count. */
uint32_t hko_oscillator(double* x, double* v, double* k, const double* nstop, const double* omega,
                        const double* zeta, uint8_t* term, double dt, int64_t word, int64_t base,
                        int64_t count);
uint32_t hko_orbit(double* s, int64_t pitch, double* t, double* h, double* n_acc, double* n_rej,
                   const double* t_end, uint8_t* term, int64_t word, int64_t base, int64_t count);

/* The 32-sample rows (sum, compensation) of one column of per-sample terms,
 * any op: what a kernel's sample sum stores before the finish. */
void hko_rows_f64(int op, const double* terms, int64_t n, double* hi, double* comp);

/* Team-form linear algebra (n x n per sample, any n): what the reference's
 * stages compute per lane -- the one-thread form's operation order for every
 * n (hawk/embedded/linalg.py:188-520).  Planes are component-major: A is
 * (n, n, pitch), b and x (n, pitch), B and X (n, 2, pitch), L (n, n, pitch);
 * info is int32 per sample.
 *   team_chol:      L, info = cholesky(A); x = cho_solve(L, b); X = cho_solve(L, B)
 *   team_lu:        f, info = lu(A); x = lu_solve(f, b); X = lu_solve(f, B); det = det(A)
 *   team_chol_from: f, info = chol_from(A); x = cho_solve(f, b); L = f */
void hko_team_chol(int n, const double* A, const double* b, const double* B, int64_t pitch, double* x, double* X,
                   double* L, int32_t* info, int64_t base, int64_t count);
void hko_team_lu(int n, const double* A, const double* b, const double* B, int64_t pitch, double* x, double* X,
                 double* det, int32_t* info, int64_t base, int64_t count);
void hko_team_chol_from(int n, const double* A, const double* b, int64_t pitch, double* x, double* L,
                        int32_t* info, int64_t base, int64_t count);

/* w, V, info = eigh(A) per sample (A (n, n, pitch), w (n, pitch), V (n, n, pitch)
 * or null for the values-only kernel): cyclic Jacobi in the order of
 * hawk/embedded/linalg.py:302-399. */
void hko_sym_eigen(int n, const double* A, int64_t pitch, double* w, double* V, int32_t* info, int64_t base,
                   int64_t count);

/* x, info = lstsq(J, r) per sample for n > 32 (J (m, n, pitch), r (m, pitch),
 * x (n, pitch)): the b200 team-form Householder QR and its solve. */
void hko_lstsq_qr(int m, int n, const double* J, const double* r, int64_t pitch, double* x, int32_t* info,
                  int64_t base, int64_t count);

#ifdef __cplusplus
}
#endif

#endif
