// f64 GEMM on the FP64 tensor pipe (DMMA, mma.sync m16n8k4 .f64) for sm_100a.
//
// C[b](i,j) = sum_p A[b](i,p) * B[b](p,j) in double precision with f64
// accumulation, for operands with unit stride along k or along m/n (the c2
// workload: row-major A, B a transposed view); every other layout keeps the
// SIMT DFMA kernel (gemm_simt.cuh).  Kernix reaches gemm-f64 or matrixmultiply
// for these layouts through MatmulElement::try_dense_matmul / try_strided_matmul
// (crates/kernix-ops/src/ops/matmul_element.rs:53-251).
//
// Why DMMA: a DFMA outer-product kernel with 8x8 outputs per thread reads 16
// doubles of shared memory per 64 FMAs, which is the whole shared-memory
// bandwidth at the FP64 rate; an m16n8k4 MMA takes 2 + 1 doubles per thread for
// 512 FMAs per warp, so the FP64 pipe, not shared memory, sets the pace.
//
// CTA: 128 x 128 outputs, 8 warps as 2 (m) x 4 (n), warp tile 64 x 32 (4 x 4
// MMAs per k-step of 4), k depth 32 per stage, 3-stage cp.async ring (one
// barrier per 32 k); each k-step's fragments are read while the previous
// step's MMAs run, and a stage's copies are issued after its first k-step.
// Shared layouts follow the operand's contiguous axis so that cp.async copies
// stay contiguous; row pitches are padded so the fragment loads of a warp hit
// each bank at most twice (the minimum for 32 doubles).
#include <cstring>

#include "gemm_simt.cuh"
#include "kx_internal.hpp"

namespace kx {
namespace dmma {

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3, NT = 256;
constexpr int PK = BK + 4;     // pitch of a k-contiguous tile row (m or n major index)
constexpr int PMN = BM + 8;    // pitch of an m/n-contiguous tile row (k major index)
static_assert(BM == BN, "one pitch for both operands");
constexpr int TILE_DOUBLES = BM * PK > BK * PMN ? BM * PK : BK * PMN;   // 4608
constexpr int SMEM_BYTES = STAGES * 2 * TILE_DOUBLES * 8;                 // 221184
static_assert(SMEM_BYTES <= 232448, "shared memory");

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// 8- or 16-byte asynchronous copy; `bytes` = 0 zero-fills (src is not read).
__device__ __forceinline__ void cp8(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 8 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void mma_f64(double (&d)[4], double a0, double a1, double b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a0), "d"(a1), "d"(b0));
}

// One operand's tile copy: rows r in [0, 128) along m (A) or n (B), k in
// [0, 16).  KC: unit stride along k, shared [r][PK]; otherwise unit stride
// along r, shared [k][PMN].  V2: pairs of doubles (16 bytes) along the
// contiguous axis, valid when that extent is even and the base is aligned.
template <bool KC, bool V2>
__device__ __forceinline__ void load_tile(double *s, const double *g, int64_t s_r, int64_t s_k, int r0, int R,
                                          int k0, int K, int tid) {
    if constexpr (KC) {
        constexpr int PER = V2 ? 2 : 1;
        constexpr int CH = BK / PER;                       // chunks per row
        constexpr int ITERS = BM * CH / NT;
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
            const int c = tid + it * NT;
            const int r = c / CH, kk = (c % CH) * PER;
            const bool ok = (r0 + r < R) && (k0 + kk < K);
            const double *src = ok ? g + (int64_t)(r0 + r) * s_r + (int64_t)(k0 + kk) : g;
            if constexpr (V2) cp16(s + r * PK + kk, src, ok);
            else cp8(s + r * PK + kk, src, ok);
        }
    } else {
        constexpr int PER = V2 ? 2 : 1;
        constexpr int CH = BM / PER;                       // chunks per k row
        constexpr int ITERS = BK * CH / NT;
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
            const int c = tid + it * NT;
            const int kk = c / CH, r = (c % CH) * PER;
            const bool ok = (r0 + r < R) && (k0 + kk < K);
            const double *src = ok ? g + (int64_t)(r0 + r) + (int64_t)(k0 + kk) * s_k : g;
            if constexpr (V2) cp16(s + kk * PMN + r, src, ok);
            else cp8(s + kk * PMN + r, src, ok);
        }
    }
}

template <bool KC>
__device__ __forceinline__ double frag(const double *s, int r, int k) {
    if constexpr (KC) return s[r * PK + k];
    else return s[k * PMN + r];
}

template <bool A_KC, bool B_KC, bool V2>
__global__ void __launch_bounds__(NT, 1) gemm_dmma_kernel(const __grid_constant__ GemmParams<double> p) {
    extern __shared__ __align__(16) double smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int wm = (warp >> 2) * 64, wn = (warp & 3) * 32;
    const int tiles_m = (p.M + BM - 1) / BM, tiles_n = (p.N + BN - 1) / BN;
    int tm, tn;
    raster(blockIdx.x, tiles_m, tiles_n, 8, tm, tn);
    const int m0 = tm * BM, n0 = tn * BN;
    const int ktiles = (p.K + BK - 1) / BK;
    // A(i, p) = A[i*a_rs + p*a_cs]: r along m; B(p, j) = B[p*b_rs + j*b_cs]: r along n
    const int64_t a_sr = p.a_rs, a_sk = p.a_cs, b_sr = p.b_cs, b_sk = p.b_rs;

    for (int64_t batch = blockIdx.y; batch < p.nbatch; batch += gridDim.y) {
        int64_t oa, ob, oc;
        batch_offsets(p.batch, batch, oa, ob, oc);
        const double *A = p.A + oa;
        const double *B = p.B + ob;
        auto sA = [&](int st) { return smem + st * 2 * TILE_DOUBLES; };
        auto sB = [&](int st) { return smem + st * 2 * TILE_DOUBLES + TILE_DOUBLES; };

        double acc[4][4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0;

#pragma unroll
        for (int st = 0; st < STAGES - 1; ++st) {
            if (st < ktiles) {
                load_tile<A_KC, V2>(sA(st), A, a_sr, a_sk, m0, p.M, st * BK, p.K, tid);
                load_tile<B_KC, V2>(sB(st), B, b_sr, b_sk, n0, p.N, st * BK, p.K, tid);
            }
            cp_commit();
        }
        for (int kt = 0; kt < ktiles; ++kt) {
            cp_wait<STAGES - 2>();
            __syncthreads();
            const int nxt = kt + STAGES - 1;
            const double *a_s = sA(kt % STAGES), *b_s = sB(kt % STAGES);
            // fragments of k step kk + 4 are read while step kk's MMAs run;
            // the next stage's copies go out after the first step's MMAs, so
            // the tensor pipe restarts right after the barrier
            double af[2][4][2], bf[2][4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                af[0][i][0] = frag<A_KC>(a_s, wm + i * 16 + g, t4);
                af[0][i][1] = frag<A_KC>(a_s, wm + i * 16 + g + 8, t4);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) bf[0][j] = frag<B_KC>(b_s, wn + j * 8 + g, t4);
#pragma unroll
            for (int s4 = 0; s4 < BK / 4; ++s4) {
                const int cur = s4 & 1;
                if (s4 + 1 < BK / 4) {
                    const int kn = (s4 + 1) * 4 + t4;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        af[cur ^ 1][i][0] = frag<A_KC>(a_s, wm + i * 16 + g, kn);
                        af[cur ^ 1][i][1] = frag<A_KC>(a_s, wm + i * 16 + g + 8, kn);
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) bf[cur ^ 1][j] = frag<B_KC>(b_s, wn + j * 8 + g, kn);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) mma_f64(acc[i][j], af[cur][i][0], af[cur][i][1], bf[cur][j]);
                if (s4 == 0) {
                    if (nxt < ktiles) {
                        load_tile<A_KC, V2>(sA(nxt % STAGES), A, a_sr, a_sk, m0, p.M, nxt * BK, p.K, tid);
                        load_tile<B_KC, V2>(sB(nxt % STAGES), B, b_sr, b_sk, n0, p.N, nxt * BK, p.K, tid);
                    }
                    cp_commit();
                }
            }
        }
        cp_wait<0>();
        __syncthreads();   // the next batch's prologue reuses the stages

        double *C = p.C + oc;
        const bool vec = p.c_cs == 1 && (p.c_rs % 2 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = m0 + wm + i * 16 + g + h * 8;
                if (row >= p.M) continue;
                double *crow = C + (int64_t)row * p.c_rs;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int col = n0 + wn + j * 8 + 2 * t4;
                    const double v0 = acc[i][j][2 * h], v1 = acc[i][j][2 * h + 1];
                    if (vec && col + 1 < p.N) {
                        *reinterpret_cast<double2 *>(crow + col) = make_double2(v0, v1);
                    } else {
                        if (col < p.N) crow[(int64_t)col * p.c_cs] = v0;
                        if (col + 1 < p.N) crow[(int64_t)(col + 1) * p.c_cs] = v1;
                    }
                }
            }
        }
    }
}

template <bool A_KC, bool B_KC, bool V2>
cudaError_t launch(const GemmParams<double> &p, cudaStream_t s) {
    auto k = gemm_dmma_kernel<A_KC, B_KC, V2>;
    cudaError_t ce = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (ce != cudaSuccess) return ce;
    const int64_t tiles = (int64_t)((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
    dim3 grid((unsigned)tiles, (unsigned)(p.nbatch < 65535 ? p.nbatch : 65535), 1);
    k<<<grid, NT, SMEM_BYTES, s>>>(p);
    return cudaGetLastError();
}

}  // namespace dmma

// Unit stride along k or along m/n for each operand, positive strides.
bool dmma_eligible(const GemmParams<double> &p, bool *a_kc, bool *b_kc, bool *v2) {
    if (p.M < 1 || p.N < 1 || p.K < 1) return false;
    const bool akc = p.a_cs == 1 && p.a_rs > 0, amn = p.a_rs == 1 && p.a_cs > 0;
    const bool bkc = p.b_rs == 1 && p.b_cs > 0, bmn = p.b_cs == 1 && p.b_rs > 0;
    if (!(akc || amn) || !(bkc || bmn)) return false;
    // For rank-1 extents both strides may be 1: prefer the k-contiguous form.
    *a_kc = akc;
    *b_kc = bkc;
    // 16-byte copies: even contiguous extents and strides, aligned bases and batch strides.
    bool ok2 = ((reinterpret_cast<uintptr_t>(p.A) | reinterpret_cast<uintptr_t>(p.B)) & 15) == 0;
    ok2 = ok2 && (akc ? (p.K % 2 == 0 && p.a_rs % 2 == 0) : (p.M % 2 == 0 && p.a_cs % 2 == 0));
    ok2 = ok2 && (bkc ? (p.K % 2 == 0 && p.b_cs % 2 == 0) : (p.N % 2 == 0 && p.b_rs % 2 == 0));
    for (int d = 0; d < p.batch.ndims; ++d) ok2 = ok2 && p.batch.a_str[d] % 2 == 0 && p.batch.b_str[d] % 2 == 0;
    *v2 = ok2;
    for (int d = 0; d < p.batch.ndims; ++d)
        if (p.batch.a_str[d] < 0 || p.batch.b_str[d] < 0) return false;
    return true;
}

int run_gemm_dmma(Handle *h, const GemmParams<double> &p0, const char **kernel_name) {
    // A stride along an extent-one axis is never used: call it unit so that
    // vectors and single rows/columns qualify.
    GemmParams<double> p = p0;
    // (Singleton strides arrive normalised to zero, as MatrixInput::new does.)
    if (p.K == 1) {
        p.a_cs = (p.a_rs == 1) ? 2 : 1;
        p.b_rs = (p.b_cs == 1) ? 2 : 1;
    }
    if (p.M == 1) p.a_rs = (p.a_cs == 1) ? 2 : 1;
    if (p.N == 1) p.b_cs = (p.b_rs == 1) ? 2 : 1;
    bool akc, bkc, v2;
    if (!dmma_eligible(p, &akc, &bkc, &v2)) return KX_DECLINED;
    cudaError_t ce;
    const int sel = (akc ? 4 : 0) | (bkc ? 2 : 0) | (v2 ? 1 : 0);
    switch (sel) {
        case 0: ce = dmma::launch<false, false, false>(p, h->stream); break;
        case 1: ce = dmma::launch<false, false, true>(p, h->stream); break;
        case 2: ce = dmma::launch<false, true, false>(p, h->stream); break;
        case 3: ce = dmma::launch<false, true, true>(p, h->stream); break;
        case 4: ce = dmma::launch<true, false, false>(p, h->stream); break;
        case 5: ce = dmma::launch<true, false, true>(p, h->stream); break;
        case 6: ce = dmma::launch<true, true, false>(p, h->stream); break;
        default: ce = dmma::launch<true, true, true>(p, h->stream); break;
    }
    *kernel_name = "dmma_128x128";
    ++h->launches;
    return ce == cudaSuccess ? KX_OK : h->cuda_fail(ce);
}

}  // namespace kx
