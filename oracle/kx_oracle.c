/*
 * kx_oracle.c -- CPU restatement of Kernix's dense-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the oracle: the tests, the smoke
 * check and the CPU-baseline leg of bench.py call it as the checker.  The
 * product (libkernix_b200.so and the kernix_b200 package) never links or calls
 * it.  It is compiled with -ffp-contract=off so every `acc += a * b` rounds the
 * product and the sum separately, as Rust does (Rust never contracts to FMA).
 *
 * Each function cites the reference code it restates (paths inside the kernix
 * repository, Kernix 0.13.0).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* SplitMix64 SeededRng (crates/kernix/src/training.rs:132-171)              */
/* ------------------------------------------------------------------------ */
uint64_t kxo_splitmix_next(uint64_t *state) {
    *state += 0x9e3779b97f4a7c15ULL;
    uint64_t x = *state;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
    return x ^ (x >> 31);
}

/* uniform(): low + (high - low) * ((u >> 11) * 2^-53), computed in f64, then
 * converted to the element type.  Returns the stream state after n draws. */
uint64_t kxo_uniform_f64(uint64_t state, uint64_t n, double low, double high, double *out) {
    for (uint64_t i = 0; i < n; ++i) {
        double fraction = (double)(kxo_splitmix_next(&state) >> 11) * (1.0 / 9007199254740992.0);
        out[i] = low + (high - low) * fraction;
    }
    return state;
}
uint64_t kxo_uniform_f32(uint64_t state, uint64_t n, double low, double high, float *out) {
    for (uint64_t i = 0; i < n; ++i) {
        double fraction = (double)(kxo_splitmix_next(&state) >> 11) * (1.0 / 9007199254740992.0);
        out[i] = (float)(low + (high - low) * fraction);
    }
    return state;
}

/* ------------------------------------------------------------------------ */
/* Ordered dense matmul (crates/kernix-ops/src/ops/linalg.rs:236-316)        */
/* 4x4 register tiles, each output accumulated in increasing k with          */
/* `acc += a * b`; tail rows/columns by the same scalar recurrence.          */
/* ------------------------------------------------------------------------ */
#define DENSE_MATMUL(NAME, T)                                                             \
    void NAME(const T *a, const T *b, T *out, uint64_t m, uint64_t k, uint64_t n) {       \
        for (uint64_t i = 0; i < m * n; ++i) out[i] = (T)0;                               \
        const uint64_t rows = m / 4 * 4, cols = n / 4 * 4;                                \
        for (uint64_t col = 0; col < cols; col += 4)                                      \
            for (uint64_t row = 0; row < rows; row += 4) {                                \
                T acc[4][4] = {{0}};                                                      \
                for (uint64_t p = 0; p < k; ++p) {                                        \
                    const T *br = b + p * n + col;                                        \
                    for (int r = 0; r < 4; ++r) {                                         \
                        const T av = a[(row + r) * k + p];                                \
                        acc[r][0] += av * br[0];                                          \
                        acc[r][1] += av * br[1];                                          \
                        acc[r][2] += av * br[2];                                          \
                        acc[r][3] += av * br[3];                                          \
                    }                                                                     \
                }                                                                         \
                for (int r = 0; r < 4; ++r)                                               \
                    for (int c = 0; c < 4; ++c) out[(row + r) * n + col + c] = acc[r][c]; \
            }                                                                             \
        for (uint64_t row = 0; row < m; ++row)                                            \
            for (uint64_t col = cols; col < n; ++col) {                                   \
                T v = (T)0;                                                               \
                for (uint64_t p = 0; p < k; ++p) v += a[row * k + p] * b[p * n + col];    \
                out[row * n + col] = v;                                                   \
            }                                                                             \
        for (uint64_t row = rows; row < m; ++row)                                         \
            for (uint64_t col = 0; col < cols; ++col) {                                   \
                T v = (T)0;                                                               \
                for (uint64_t p = 0; p < k; ++p) v += a[row * k + p] * b[p * n + col];    \
                out[row * n + col] = v;                                                   \
            }                                                                             \
    }
DENSE_MATMUL(kxo_dense_matmul_f32, float)
DENSE_MATMUL(kxo_dense_matmul_f64, double)

/* ------------------------------------------------------------------------ */
/* Ordered strided GEMM: one matrix of the general checked fallback          */
/* (linalg.rs:176-213): out(i,j) = sum_{p increasing} A(i,p) * B(p,j),       */
/* value starts at zero, `value += a * b`.  Same per-output operation        */
/* sequence as dense_matmul, so both give identical bits.  Signed strides.   */
/* The 4x4 tiling only changes memory order, never the per-output order.     */
/* ------------------------------------------------------------------------ */
#define STRIDED_GEMM(NAME, T)                                                                          \
    void NAME(const T *A, int64_t a_rs, int64_t a_cs, const T *B, int64_t b_rs, int64_t b_cs, T *Cm,   \
              int64_t c_rs, int64_t c_cs, int64_t m, int64_t n, int64_t k) {                          \
        const int64_t rows = m / 4 * 4, cols = n / 4 * 4;                                             \
        for (int64_t row = 0; row < rows; row += 4)                                                   \
            for (int64_t col = 0; col < cols; col += 4) {                                             \
                T acc[4][4] = {{0}};                                                                  \
                for (int64_t p = 0; p < k; ++p) {                                                     \
                    T bv[4];                                                                          \
                    for (int c = 0; c < 4; ++c) bv[c] = B[p * b_rs + (col + c) * b_cs];               \
                    for (int r = 0; r < 4; ++r) {                                                     \
                        const T av = A[(row + r) * a_rs + p * a_cs];                                  \
                        for (int c = 0; c < 4; ++c) acc[r][c] += av * bv[c];                          \
                    }                                                                                 \
                }                                                                                     \
                for (int r = 0; r < 4; ++r)                                                           \
                    for (int c = 0; c < 4; ++c) Cm[(row + r) * c_rs + (col + c) * c_cs] = acc[r][c]; \
            }                                                                                         \
        for (int64_t row = 0; row < m; ++row)                                                         \
            for (int64_t col = (row < rows ? cols : 0); col < n; ++col) {                             \
                T v = (T)0;                                                                           \
                for (int64_t p = 0; p < k; ++p) v += A[row * a_rs + p * a_cs] * B[p * b_rs + col * b_cs]; \
                Cm[row * c_rs + col * c_cs] = v;                                                      \
            }                                                                                         \
    }
STRIDED_GEMM(kxo_gemm_ordered_f32, float)
STRIDED_GEMM(kxo_gemm_ordered_f64, double)

/* Row-parallel ordered GEMM for the CPU baseline: rows are split into chunks
 * of a multiple of 64 (CpuExecutor::matmul_into, execution.rs:188-233), each
 * chunk running the same ordered recurrence, so results equal the serial ones. */
#define PAR_GEMM(NAME, SER, T)                                                                        \
    void NAME(const T *A, int64_t a_rs, int64_t a_cs, const T *B, int64_t b_rs, int64_t b_cs, T *Cm,  \
              int64_t c_rs, int64_t c_cs, int64_t m, int64_t n, int64_t k, int threads) {            \
        if (threads < 1) threads = 1;                                                                \
        int64_t chunk = (m / threads / 64);                                                          \
        if (chunk < 1) chunk = 1;                                                                    \
        chunk *= 64;                                                                                 \
        const int64_t nchunks = (m + chunk - 1) / chunk;                                             \
        _Pragma("omp parallel for schedule(dynamic, 1) num_threads(threads)")                         \
        for (int64_t c = 0; c < nchunks; ++c) {                                                       \
            const int64_t r0 = c * chunk;                                                            \
            const int64_t rr = (m - r0) < chunk ? (m - r0) : chunk;                                  \
            SER(A + r0 * a_rs, a_rs, a_cs, B, b_rs, b_cs, Cm + r0 * c_rs, c_rs, c_cs, rr, n, k);     \
        }                                                                                            \
    }
PAR_GEMM(kxo_gemm_ordered_par_f32, kxo_gemm_ordered_f32, float)
PAR_GEMM(kxo_gemm_ordered_par_f64, kxo_gemm_ordered_f64, double)

/* ------------------------------------------------------------------------ */
/* Compensated f64 reference (Ogita, Rump, Oishi 2005, "Accurate sum and     */
/* dot product", algorithm Dot2: TwoProduct via fma + TwoSum).  Inputs are   */
/* read as f64; f32 products are exact in f64.  Also returns sum |a*b| for   */
/* scaled error bounds (small_matmul_tests.rs:153-186 style).                */
/* ------------------------------------------------------------------------ */
static inline void two_sum(double a, double b, double *s, double *e) {
    double x = a + b;
    double z = x - a;
    *e = (a - (x - z)) + (b - z);
    *s = x;
}
static inline void two_prod(double a, double b, double *p, double *e) {
    double x = a * b;
    *e = fma(a, b, -x);
    *p = x;
}
#define DOT2_GEMM(NAME, T)                                                                           \
    void NAME(const T *A, int64_t a_rs, int64_t a_cs, const T *B, int64_t b_rs, int64_t b_cs,        \
              double *Cm, double *absm, int64_t m, int64_t n, int64_t k, int threads) {             \
        if (threads < 1) threads = 1;                                                               \
        _Pragma("omp parallel for schedule(dynamic, 4) num_threads(threads)")                        \
        for (int64_t i = 0; i < m; ++i)                                                              \
            for (int64_t j = 0; j < n; ++j) {                                                        \
                double s = 0.0, c = 0.0, ab = 0.0;                                                   \
                for (int64_t p = 0; p < k; ++p) {                                                    \
                    double h, r, q;                                                                  \
                    two_prod((double)A[i * a_rs + p * a_cs], (double)B[p * b_rs + j * b_cs], &h, &r); \
                    ab += fabs(h);                                                                   \
                    two_sum(s, h, &s, &q);                                                           \
                    c += q + r;                                                                      \
                }                                                                                    \
                Cm[i * n + j] = s + c;                                                               \
                if (absm) absm[i * n + j] = ab;                                                      \
            }                                                                                        \
    }
DOT2_GEMM(kxo_gemm_dot2_f32, float)
DOT2_GEMM(kxo_gemm_dot2_f64, double)

/* ------------------------------------------------------------------------ */
/* conv2d ordered scalar path (crates/kernix-ops/src/neural.rs:341-357 with  */
/* ConvGeometry::position :126-132): for each output, sum over ci, ky, kx    */
/* increasing, skipping taps outside the image, `sum += x * w`.              */
/* Strides are signed element strides of 4-d NCHW / OIHW descriptors.        */
/* ------------------------------------------------------------------------ */
#define CONV_REF(NAME, T)                                                                               \
    void NAME(const T *x, const int64_t *xd, const int64_t *xs, const T *w, const int64_t *wd,          \
              const int64_t *wsd, T *y, const int64_t *yd, const int64_t *opt) {                        \
        /* opt = {sy, sx, py, px, dy, dx, groups} */                                                    \
        const int64_t n = yd[0], co = yd[1], oh = yd[2], ow = yd[3];                                    \
        const int64_t cg = wd[1], kh = wd[2], kw = wd[3];                                               \
        const int64_t cog = wd[0] / opt[6];                                                             \
        for (int64_t b = 0; b < n; ++b)                                                                 \
            for (int64_t c = 0; c < co; ++c)                                                            \
                for (int64_t oy = 0; oy < oh; ++oy)                                                     \
                    for (int64_t ox = 0; ox < ow; ++ox) {                                               \
                        const int64_t grp = c / cog;                                                    \
                        T sum = (T)0;                                                                   \
                        for (int64_t ci = 0; ci < cg; ++ci)                                             \
                            for (int64_t ky = 0; ky < kh; ++ky)                                         \
                                for (int64_t kx = 0; kx < kw; ++kx) {                                   \
                                    const int64_t yy = oy * opt[0] + ky * opt[4] - opt[2];              \
                                    const int64_t xx = ox * opt[1] + kx * opt[5] - opt[3];              \
                                    if (yy < 0 || xx < 0 || yy >= xd[2] || xx >= xd[3]) continue;       \
                                    sum += x[b * xs[0] + (grp * cg + ci) * xs[1] + yy * xs[2] + xx * xs[3]] * \
                                           w[c * wsd[0] + ci * wsd[1] + ky * wsd[2] + kx * wsd[3]];     \
                                }                                                                       \
                        y[((b * co + c) * oh + oy) * ow + ox] = sum;                                    \
                    }                                                                                   \
    }
CONV_REF(kxo_conv2d_reference_f32, float)
CONV_REF(kxo_conv2d_reference_f64, double)

/* Compensated conv (Dot2 over the same taps) for tolerance checks. */
#define CONV_DOT2(NAME, T)                                                                              \
    void NAME(const T *x, const int64_t *xd, const int64_t *xs, const T *w, const int64_t *wd,          \
              const int64_t *wsd, double *y, double *absy, const int64_t *yd, const int64_t *opt,       \
              int threads) {                                                                            \
        const int64_t n = yd[0], co = yd[1], oh = yd[2], ow = yd[3];                                    \
        const int64_t cg = wd[1], kh = wd[2], kw = wd[3];                                               \
        const int64_t cog = wd[0] / opt[6];                                                             \
        if (threads < 1) threads = 1;                                                                   \
        _Pragma("omp parallel for collapse(2) schedule(dynamic, 1) num_threads(threads)")               \
        for (int64_t b = 0; b < n; ++b)                                                                 \
            for (int64_t c = 0; c < co; ++c)                                                            \
                for (int64_t oy = 0; oy < oh; ++oy)                                                     \
                    for (int64_t ox = 0; ox < ow; ++ox) {                                               \
                        const int64_t grp = c / cog;                                                    \
                        double s = 0.0, cc = 0.0, ab = 0.0;                                             \
                        for (int64_t ci = 0; ci < cg; ++ci)                                             \
                            for (int64_t ky = 0; ky < kh; ++ky)                                         \
                                for (int64_t kx = 0; kx < kw; ++kx) {                                   \
                                    const int64_t yy = oy * opt[0] + ky * opt[4] - opt[2];              \
                                    const int64_t xx = ox * opt[1] + kx * opt[5] - opt[3];              \
                                    if (yy < 0 || xx < 0 || yy >= xd[2] || xx >= xd[3]) continue;       \
                                    double h, r, q;                                                     \
                                    two_prod((double)x[b * xs[0] + (grp * cg + ci) * xs[1] + yy * xs[2] + xx * xs[3]], \
                                             (double)w[c * wsd[0] + ci * wsd[1] + ky * wsd[2] + kx * wsd[3]], &h, &r); \
                                    ab += fabs(h);                                                      \
                                    two_sum(s, h, &s, &q);                                              \
                                    cc += q + r;                                                        \
                                }                                                                       \
                        const int64_t o = ((b * co + c) * oh + oy) * ow + ox;                           \
                        y[o] = s + cc;                                                                  \
                        if (absy) absy[o] = ab;                                                         \
                    }                                                                                   \
    }
CONV_DOT2(kxo_conv2d_dot2_f32, float)
CONV_DOT2(kxo_conv2d_dot2_f64, double)

/* ------------------------------------------------------------------------ */
/* softmax_temperature over contiguous rows (math_extra.rs:394-401, 425-500): */
/* first nonfinite -> return its flat index; max with strict `>` from the    */
/* first element; sequential sum of exp((x-max)/T) (or x/T - max/T when the  */
/* difference overflows); out = exp(delta) / sum.  Returns -1 on success.    */
/* ------------------------------------------------------------------------ */
#define SOFTMAX(NAME, T, EXP, ISF)                                                  \
    int64_t NAME(const T *x, T *out, int64_t rows, int64_t len, T t) {              \
        for (int64_t r = 0; r < rows; ++r) {                                        \
            const T *xr = x + r * len;                                              \
            T mx = xr[0];                                                           \
            for (int64_t j = 0; j < len; ++j) {                                     \
                if (!ISF(xr[j])) return r * len + j;                                \
                if (j == 0 || xr[j] > mx) mx = xr[j];                               \
            }                                                                       \
            T sum = (T)0;                                                           \
            for (int64_t j = 0; j < len; ++j) {                                     \
                T d = xr[j] - mx;                                                   \
                T delta = ISF(d) ? d / t : xr[j] / t - mx / t;                      \
                sum = sum + EXP(delta);                                             \
            }                                                                       \
            for (int64_t j = 0; j < len; ++j) {                                     \
                T d = xr[j] - mx;                                                   \
                T delta = ISF(d) ? d / t : xr[j] / t - mx / t;                      \
                out[r * len + j] = EXP(delta) / sum;                                \
            }                                                                       \
        }                                                                           \
        return -1;                                                                  \
    }
static inline int isf_f(float v) { return isfinite(v); }
static inline int isf_d(double v) { return isfinite(v); }
SOFTMAX(kxo_softmax_rows_f32, float, expf, isf_f)
SOFTMAX(kxo_softmax_rows_f64, double, exp, isf_d)

int kxo_openmp_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------------------------------ */
/* conv2d_backward (crates/kernix-ops/src/neural.rs:379-430): for every       */
/* output gradient element in C order (n, co, oy, ox) and every tap          */
/* (ci, ky, kx) inside the padded input, dx[n, g*cg+ci, y, x] += dy * w and   */
/* dw[co, ci, ky, kx] += dy * x, separately rounded (no FMA).  Same geometry  */
/* arguments as kxo_conv2d_reference; dx and dw must be zeroed by the caller. */
/* ------------------------------------------------------------------------ */
#define CONV_BWD(NAME, T)                                                                               \
    void NAME(const T *x, const int64_t *xd, const int64_t *xs, const T *w, const int64_t *wd,             \
              const int64_t *ws, const T *dy, const int64_t *yd, T *dx, T *dw, const int64_t *opt) {      \
        const int64_t sy = opt[0], sx = opt[1], py = opt[2], px = opt[3], dly = opt[4], dlx = opt[5];     \
        const int64_t groups = opt[6], cg = wd[1], kh = wd[2], kw = wd[3];                                \
        const int64_t cpg = yd[1] / groups;                                                               \
        for (int64_t n = 0; n < yd[0]; ++n)                                                               \
            for (int64_t co = 0; co < yd[1]; ++co)                                                        \
                for (int64_t oy = 0; oy < yd[2]; ++oy)                                                    \
                    for (int64_t ox = 0; ox < yd[3]; ++ox) {                                              \
                        const T g = dy[((n * yd[1] + co) * yd[2] + oy) * yd[3] + ox];                     \
                        const int64_t grp = co / cpg;                                                     \
                        for (int64_t ci = 0; ci < cg; ++ci)                                               \
                            for (int64_t ky = 0; ky < kh; ++ky)                                           \
                                for (int64_t kx = 0; kx < kw; ++kx) {                                     \
                                    const int64_t y = oy * sy + ky * dly - py, xx = ox * sx + kx * dlx - px; \
                                    if (y < 0 || y >= xd[2] || xx < 0 || xx >= xd[3]) continue;           \
                                    const int64_t c = grp * cg + ci;                                      \
                                    const int64_t ai = ((n * xd[1] + c) * xd[2] + y) * xd[3] + xx;        \
                                    const int64_t wi = ((co * wd[1] + ci) * kh + ky) * kw + kx;           \
                                    const T wv = w[co * ws[0] + ci * ws[1] + ky * ws[2] + kx * ws[3]];    \
                                    const T xv = x[n * xs[0] + c * xs[1] + y * xs[2] + xx * xs[3]];       \
                                    dx[ai] = dx[ai] + g * wv;                                             \
                                    dw[wi] = dw[wi] + g * xv;                                             \
                                }                                                                         \
                    }                                                                                     \
    }
CONV_BWD(kxo_conv2d_backward_f32, float)
CONV_BWD(kxo_conv2d_backward_f64, double)
