/*
 * kx_engine.c -- CPU restatement of the blocked GEMM engines Kernix calls.
 *
 * TEST INFRASTRUCTURE ONLY: the CPU baseline that bench.py times (its
 * cpu_baseline leg and the reference arm) and a second CPU result the tests
 * and the bench compare against the compensated oracle.  The product never
 * links or calls it.
 *
 * Kernix hands its native products to two third-party crates that are not
 * vendored in the kernix repository: gemm-f32 / gemm-f64 0.19.0 (contiguous
 * operands, m,k,n >= 64; ops/matmul_element.rs:178-209) and matrixmultiply
 * 0.3.11 (signed strides, ops/matmul_element.rs:119-136).  Both implement the
 * published BLIS loop nest (Goto & van de Geijn, "Anatomy of high-performance
 * matrix multiplication", TOMS 2008; Van Zee & van de Geijn, "BLIS", TOMS
 * 2015), restated here:
 *
 *   for jc over N by NC:                       B panel stays in L3
 *     for pc over K by KC:
 *       pack B[pc:pc+KC, jc:jc+NC] into NR-wide column panels
 *       for ic over M by MC:                   A block stays in L2
 *         pack A[ic:ic+MC, pc:pc+KC] into MR-tall row panels
 *         for jr, ir: C[ir:ir+MR, jr:jr+NR] += Apanel * Bpanel
 *                     (register micro-tile, one fused multiply-add per
 *                      element and k, fp32 accumulation for f32)
 *
 * Operands are read through signed element strides while packing (what
 * matrixmultiply does), so strided A (the 8192 x 8704 slice) costs nothing
 * extra.  The micro-tile (6 x 16 f32 / 6 x 8 f64 on 256-bit AVX2 registers)
 * and the block sizes are this port's choices for x86-64-v3, not constants
 * read from either crate.  Each call is serial, as Kernix calls both crates
 * (Parallelism::None, matmul_element.rs:109,206); the threaded entry splits
 * output rows into chunks the way CpuExecutor::matmul_into does
 * (execution.rs:188-233: chunks of (m / threads / 64).max(1) * 64 rows, each
 * chunk one serial engine call with its own packing).
 */
#include <immintrin.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define KC 256
#define MC 96
#define NC_F32 3072
#define NC_F64 1536

/* ---------------------------------------------------------------- f32 --- */
#define MR 6
#define NR32 16

static void pack_a_f32(const float *a, int64_t rs, int64_t cs, int64_t mc, int64_t kc, float *dst) {
    for (int64_t i0 = 0; i0 < mc; i0 += MR) {
        const int64_t mr = mc - i0 < MR ? mc - i0 : MR;
        for (int64_t p = 0; p < kc; ++p) {
            for (int64_t i = 0; i < mr; ++i) dst[i] = a[(i0 + i) * rs + p * cs];
            for (int64_t i = mr; i < MR; ++i) dst[i] = 0.0f;
            dst += MR;
        }
    }
}

static void pack_b_f32(const float *b, int64_t rs, int64_t cs, int64_t kc, int64_t nc, float *dst) {
    for (int64_t j0 = 0; j0 < nc; j0 += NR32) {
        const int64_t nr = nc - j0 < NR32 ? nc - j0 : NR32;
        for (int64_t p = 0; p < kc; ++p) {
            const float *row = b + p * rs + j0 * cs;
            if (cs == 1 && nr == NR32) {
                memcpy(dst, row, NR32 * sizeof(float));
            } else {
                for (int64_t j = 0; j < nr; ++j) dst[j] = row[j * cs];
                for (int64_t j = nr; j < NR32; ++j) dst[j] = 0.0f;
            }
            dst += NR32;
        }
    }
}

/* C[0:mr, 0:nr] (+)= Apanel[MR x kc] * Bpanel[kc x NR32]; `first` stores
 * instead of adding (the first k block of C). */
static void micro_f32(int64_t kc, const float *ap, const float *bp, float *c, int64_t ldc, int64_t mr, int64_t nr,
                      int first) {
    __m256 acc[MR][2];
    for (int i = 0; i < MR; ++i) acc[i][0] = acc[i][1] = _mm256_setzero_ps();
    for (int64_t p = 0; p < kc; ++p) {
        const __m256 b0 = _mm256_loadu_ps(bp), b1 = _mm256_loadu_ps(bp + 8);
        for (int i = 0; i < MR; ++i) {
            const __m256 av = _mm256_broadcast_ss(ap + i);
            acc[i][0] = _mm256_fmadd_ps(av, b0, acc[i][0]);
            acc[i][1] = _mm256_fmadd_ps(av, b1, acc[i][1]);
        }
        ap += MR;
        bp += NR32;
    }
    if (mr == MR && nr == NR32) {
        for (int i = 0; i < MR; ++i) {
            float *cr = c + i * ldc;
            if (first) {
                _mm256_storeu_ps(cr, acc[i][0]);
                _mm256_storeu_ps(cr + 8, acc[i][1]);
            } else {
                _mm256_storeu_ps(cr, _mm256_add_ps(_mm256_loadu_ps(cr), acc[i][0]));
                _mm256_storeu_ps(cr + 8, _mm256_add_ps(_mm256_loadu_ps(cr + 8), acc[i][1]));
            }
        }
        return;
    }
    float tile[MR][NR32];
    for (int i = 0; i < MR; ++i) {
        _mm256_storeu_ps(tile[i], acc[i][0]);
        _mm256_storeu_ps(tile[i] + 8, acc[i][1]);
    }
    for (int64_t i = 0; i < mr; ++i)
        for (int64_t j = 0; j < nr; ++j) c[i * ldc + j] = first ? tile[i][j] : c[i * ldc + j] + tile[i][j];
}

/* Serial engine call: out[m x n] (row stride ldc) = A * B. */
static void engine_f32(const float *a, int64_t ars, int64_t acs, const float *b, int64_t brs, int64_t bcs, float *c,
                       int64_t ldc, int64_t m, int64_t n, int64_t k, float *abuf, float *bbuf) {
    if (k == 0) {
        for (int64_t i = 0; i < m; ++i) memset(c + i * ldc, 0, (size_t)n * sizeof(float));
        return;
    }
    for (int64_t jc = 0; jc < n; jc += NC_F32) {
        const int64_t nc = n - jc < NC_F32 ? n - jc : NC_F32;
        for (int64_t pc = 0; pc < k; pc += KC) {
            const int64_t kc = k - pc < KC ? k - pc : KC;
            pack_b_f32(b + pc * brs + jc * bcs, brs, bcs, kc, nc, bbuf);
            for (int64_t ic = 0; ic < m; ic += MC) {
                const int64_t mc = m - ic < MC ? m - ic : MC;
                pack_a_f32(a + ic * ars + pc * acs, ars, acs, mc, kc, abuf);
                for (int64_t jr = 0; jr < nc; jr += NR32)
                    for (int64_t ir = 0; ir < mc; ir += MR)
                        micro_f32(kc, abuf + ir * kc, bbuf + jr * kc, c + (ic + ir) * ldc + jc + jr, ldc,
                                  mc - ir < MR ? mc - ir : MR, nc - jr < NR32 ? nc - jr : NR32, pc == 0);
            }
        }
    }
}

/* ---------------------------------------------------------------- f64 --- */
#define NR64 8

static void pack_a_f64(const double *a, int64_t rs, int64_t cs, int64_t mc, int64_t kc, double *dst) {
    for (int64_t i0 = 0; i0 < mc; i0 += MR) {
        const int64_t mr = mc - i0 < MR ? mc - i0 : MR;
        for (int64_t p = 0; p < kc; ++p) {
            for (int64_t i = 0; i < mr; ++i) dst[i] = a[(i0 + i) * rs + p * cs];
            for (int64_t i = mr; i < MR; ++i) dst[i] = 0.0;
            dst += MR;
        }
    }
}

static void pack_b_f64(const double *b, int64_t rs, int64_t cs, int64_t kc, int64_t nc, double *dst) {
    for (int64_t j0 = 0; j0 < nc; j0 += NR64) {
        const int64_t nr = nc - j0 < NR64 ? nc - j0 : NR64;
        for (int64_t p = 0; p < kc; ++p) {
            const double *row = b + p * rs + j0 * cs;
            for (int64_t j = 0; j < nr; ++j) dst[j] = row[j * cs];
            for (int64_t j = nr; j < NR64; ++j) dst[j] = 0.0;
            dst += NR64;
        }
    }
}

static void micro_f64(int64_t kc, const double *ap, const double *bp, double *c, int64_t ldc, int64_t mr, int64_t nr,
                      int first) {
    __m256d acc[MR][2];
    for (int i = 0; i < MR; ++i) acc[i][0] = acc[i][1] = _mm256_setzero_pd();
    for (int64_t p = 0; p < kc; ++p) {
        const __m256d b0 = _mm256_loadu_pd(bp), b1 = _mm256_loadu_pd(bp + 4);
        for (int i = 0; i < MR; ++i) {
            const __m256d av = _mm256_broadcast_sd(ap + i);
            acc[i][0] = _mm256_fmadd_pd(av, b0, acc[i][0]);
            acc[i][1] = _mm256_fmadd_pd(av, b1, acc[i][1]);
        }
        ap += MR;
        bp += NR64;
    }
    double tile[MR][NR64];
    for (int i = 0; i < MR; ++i) {
        _mm256_storeu_pd(tile[i], acc[i][0]);
        _mm256_storeu_pd(tile[i] + 4, acc[i][1]);
    }
    for (int64_t i = 0; i < mr; ++i)
        for (int64_t j = 0; j < nr; ++j) c[i * ldc + j] = first ? tile[i][j] : c[i * ldc + j] + tile[i][j];
}

static void engine_f64(const double *a, int64_t ars, int64_t acs, const double *b, int64_t brs, int64_t bcs,
                       double *c, int64_t ldc, int64_t m, int64_t n, int64_t k, double *abuf, double *bbuf) {
    if (k == 0) {
        for (int64_t i = 0; i < m; ++i) memset(c + i * ldc, 0, (size_t)n * sizeof(double));
        return;
    }
    for (int64_t jc = 0; jc < n; jc += NC_F64) {
        const int64_t nc = n - jc < NC_F64 ? n - jc : NC_F64;
        for (int64_t pc = 0; pc < k; pc += KC) {
            const int64_t kc = k - pc < KC ? k - pc : KC;
            pack_b_f64(b + pc * brs + jc * bcs, brs, bcs, kc, nc, bbuf);
            for (int64_t ic = 0; ic < m; ic += MC) {
                const int64_t mc = m - ic < MC ? m - ic : MC;
                pack_a_f64(a + ic * ars + pc * acs, ars, acs, mc, kc, abuf);
                for (int64_t jr = 0; jr < nc; jr += NR64)
                    for (int64_t ir = 0; ir < mc; ir += MR)
                        micro_f64(kc, abuf + ir * kc, bbuf + jr * kc, c + (ic + ir) * ldc + jc + jr, ldc,
                                  mc - ir < MR ? mc - ir : MR, nc - jr < NR64 ? nc - jr : NR64, pc == 0);
            }
        }
    }
}

/* ------------------------------------------------------ threaded entries --- */
/* out[m x n] C-order = A * B with signed element strides, row chunks over
 * `threads` host threads (CpuExecutor::matmul_into's split); threads <= 1 is
 * one serial engine call (kernix::matmul's path).  Returns 0, or -1 when the
 * packing buffers cannot be allocated. */
#define ENGINE_ENTRY(NAME, T, ENGINE, NC, NR)                                                              \
    int NAME(const T *a, int64_t ars, int64_t acs, const T *b, int64_t brs, int64_t bcs, T *out, int64_t m,  \
             int64_t n, int64_t k, int threads) {                                                          \
        if (m <= 0 || n <= 0) return 0;                                                                    \
        if (threads < 1) threads = 1;                                                                      \
        int64_t chunk = m;                                                                                 \
        if (threads > 1) {                                                                                 \
            chunk = (m / threads / 64) * 64;                                                               \
            if (chunk < 64) chunk = 64;                                                                    \
        }                                                                                                  \
        const int64_t nchunks = (m + chunk - 1) / chunk;                                                   \
        int failed = 0;                                                                                    \
        _Pragma("omp parallel for num_threads(threads) schedule(dynamic, 1) reduction(|| : failed)")       \
        for (int64_t q = 0; q < nchunks; ++q) {                                                            \
            T *abuf = (T *)aligned_alloc(64, sizeof(T) * (size_t)(MC + MR) * KC);                          \
            T *bbuf = (T *)aligned_alloc(64, sizeof(T) * (size_t)(NC + NR) * KC);                          \
            if (!abuf || !bbuf) {                                                                          \
                failed = 1;                                                                                \
            } else {                                                                                       \
                const int64_t r0 = q * chunk, rows = m - r0 < chunk ? m - r0 : chunk;                      \
                ENGINE(a + r0 * ars, ars, acs, b, brs, bcs, out + r0 * n, n, rows, n, k, abuf, bbuf);      \
            }                                                                                              \
            free(abuf);                                                                                    \
            free(bbuf);                                                                                    \
        }                                                                                                  \
        return failed ? -1 : 0;                                                                            \
    }
ENGINE_ENTRY(kxo_engine_gemm_f32, float, engine_f32, NC_F32, NR32)
ENGINE_ENTRY(kxo_engine_gemm_f64, double, engine_f64, NC_F64, NR64)
