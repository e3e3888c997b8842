// SIMT (CUDA-core) strided batched GEMM for sm_100a: FFMA for f32, DFMA for f64.
//
// C[b](i,j) = sum_p A[b](i,p) * B[b](p,j) for arbitrarily strided A, B and C,
// with a NumPy-style broadcast batch (zero batch strides).  This is the device
// half of kernix's matmul funnel (crates/kernix-ops/src/ops/linalg.rs:68-214):
// the reference reaches gemm-f32/f64 or matrixmultiply through the
// MatmulElement hooks (ops/matmul_element.rs:53-251); here every layout the
// hooks accept is read in place by a register-staged loader.
//
// Tile pipeline: global -> registers (vectorised when one operand axis has unit
// stride and is aligned, scalar gather otherwise) -> shared memory in one
// canonical k-major layout -> 8x8 (or 4x4) register outer products.  Two shared
// buffers with one barrier per k-tile: the loads of tile t+1 are in flight
// while tile t is multiplied.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

// Compile-time tuning knobs of the f32 SIMT tiles (defaults are the shipped
// configuration): packed FP32 FMA, k depth of the 128x128 tile, and its
// resident-CTA target per SM.
#ifndef KX_FFMA2
#define KX_FFMA2 1
#endif
#ifndef KX_F32_BK
#define KX_F32_BK 8
#endif
#ifndef KX_F32_MINB
#define KX_F32_MINB 2
#endif

namespace kx {

constexpr int kMaxBatchDims = 6;

// Output batch geometry: batch index -> per-operand element offsets.
struct BatchGeom {
    int ndims;                       // number of batch dims (0 = single matrix)
    int64_t dims[kMaxBatchDims];     // output batch dims, outermost first
    int64_t a_str[kMaxBatchDims];    // element stride of A per batch dim (0 = broadcast)
    int64_t b_str[kMaxBatchDims];
    int64_t c_str[kMaxBatchDims];
};

template <typename T>
struct GemmParams {
    const T *A;          // already advanced by the descriptor origin
    const T *B;
    T *C;
    int64_t a_rs, a_cs;  // A(i,p) = A[i*a_rs + p*a_cs]
    int64_t b_rs, b_cs;  // B(p,j) = B[p*b_rs + j*b_cs]
    int64_t c_rs, c_cs;  // C(i,j) = C[i*c_rs + j*c_cs]
    int M, N, K;
    int64_t nbatch;
    BatchGeom batch;
    int splits;          // split-K factor (1 = direct store)
    int k_per_split;     // multiple of BK
    T *ws;               // split-K partials [splits][nbatch][M][N] (C-order)
    T *C_mc;             // NVLink multicast address of C (null: none); C is then C-contiguous
};

// Operand access modes.
enum LoadMode : int {
    kVecK = 0,     // unit stride along k, vector aligned
    kVecMN = 1,    // unit stride along m (A) / n (B), vector aligned
    kGatherMN = 2, // scalar gather, threads walk m (A) / n (B) fastest
    kGatherK = 3   // scalar gather, threads walk k fastest
};

template <typename T> struct Vec;
template <> struct Vec<float> { using type = float4; static constexpr int width = 4; };
template <> struct Vec<double> { using type = double2; static constexpr int width = 2; };

__device__ __forceinline__ void batch_offsets(const BatchGeom &g, int64_t b,
                                              int64_t &oa, int64_t &ob, int64_t &oc) {
    oa = ob = oc = 0;
    for (int d = g.ndims - 1; d >= 0; --d) {
        int64_t coord = b % g.dims[d];
        b /= g.dims[d];
        oa += coord * g.a_str[d];
        ob += coord * g.b_str[d];
        oc += coord * g.c_str[d];
    }
}

// ---------------------------------------------------------------------------
// Tile loader for one operand.  `Rows` is the extent along m (A) or n (B) of the
// tile, `BK` the k extent.  The operand element (r, p) (r along m/n, p along k)
// lives at ptr[r*s_r + p*s_k].  Shared layout: sm[p][r] with row pitch Pitch.
//
// The thread -> element map is fixed for the whole k loop, so init() resolves
// the thread's row (or column) once and load() only adds the k offset; this
// keeps 64-bit address arithmetic out of the inner loop and the register
// budget small enough for two resident CTAs per SM.
//   kVecK     vector of W along k; threads walk rows fastest (transposing store)
//   kVecMN    vector of W along m/n; straight store
//   kGatherMN scalar; threads walk rows fastest
//   kGatherK  scalar; threads walk k fastest
// ---------------------------------------------------------------------------
template <typename T, int Rows, int BK, int NT, int Mode, int Pitch>
struct TileLoader {
    using V = typename Vec<T>::type;
    static constexpr int W = Vec<T>::width;
    static constexpr bool kVector = (Mode == kVecK || Mode == kVecMN);
    static constexpr int kCount = kVector ? (Rows * BK) / (W * NT) : (Rows * BK) / NT;
    static_assert(kCount >= 1, "tile too small for thread count");
    static_assert(kVector ? (Rows * BK) % (W * NT) == 0 : (Rows * BK) % NT == 0, "tile/thread mismatch");
    // Threads per "row" of the walk and the fixed stride between a thread's slots.
    static constexpr int kLanesR = (Mode == kVecK || Mode == kGatherMN) ? Rows : (Mode == kVecMN ? Rows / W : BK);
    static_assert(NT % kLanesR == 0, "thread count must tile the fast axis");
    static constexpr int kStep = NT / kLanesR;

    T reg[kVector ? kCount * W : kCount];
    const T *base;      // element (row of this thread, k = 0)
    int64_t s_k;        // stride along k (gathers, kVecMN)
    int64_t s_rstep;    // kGatherK: stride between this thread's rows
    int fast, slow0;    // thread position on the fast / slow axis
    int rlim;           // rows remaining from this thread's first row (validity)

    __device__ __forceinline__ void init(const T *__restrict__ ptr, int64_t s_r, int64_t sk, int r0, int R,
                                         int tid) {
        fast = tid % kLanesR;
        slow0 = tid / kLanesR;
        s_k = sk;
        if constexpr (Mode == kVecK || Mode == kGatherMN) {
            base = ptr + (int64_t)(r0 + fast) * s_r;
            rlim = R - (r0 + fast);
        } else if constexpr (Mode == kVecMN) {
            base = ptr + (r0 + fast * W);
            rlim = R - (r0 + fast * W);
        } else {
            base = ptr + (int64_t)(r0 + slow0) * s_r;
            s_rstep = (int64_t)kStep * s_r;
            rlim = R - (r0 + slow0);
        }
    }

    // Load k [k0, k0 + BK), zero filled outside the row range and [.., kend).
    __device__ __forceinline__ void load(int k0, int kend) {
        if constexpr (Mode == kVecK) {
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                const int gk = k0 + (slow0 + i * kStep) * W;
                V val = zero_vec();
                if (rlim > 0 && gk < kend) val = __ldg(reinterpret_cast<const V *>(base + gk));
                store_vec(&reg[i * W], val);
            }
        } else if constexpr (Mode == kVecMN) {
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                const int gk = k0 + slow0 + i * kStep;
                V val = zero_vec();
                if (rlim > 0 && gk < kend) val = __ldg(reinterpret_cast<const V *>(base + (int64_t)gk * s_k));
                store_vec(&reg[i * W], val);
            }
        } else if constexpr (Mode == kGatherMN) {
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                const int gk = k0 + slow0 + i * kStep;
                reg[i] = (rlim > 0 && gk < kend) ? __ldg(base + (int64_t)gk * s_k) : T(0);
            }
        } else {
            const int gk = k0 + fast;
            const bool kok = gk < kend;
            const T *p = base + (int64_t)gk * s_k;
#pragma unroll
            for (int i = 0; i < kCount; ++i)
                reg[i] = (kok && rlim > i * kStep) ? __ldg(p + i * s_rstep) : T(0);
        }
    }

    __device__ __forceinline__ void store(T *sm) const {
        if constexpr (Mode == kVecK) {
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                const int kv = slow0 + i * kStep;
#pragma unroll
                for (int j = 0; j < W; ++j) sm[(kv * W + j) * Pitch + fast] = reg[i * W + j];
            }
        } else if constexpr (Mode == kVecMN) {
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                V val;
                load_vec(&reg[i * W], val);
                *reinterpret_cast<V *>(&sm[(slow0 + i * kStep) * Pitch + fast * W]) = val;
            }
        } else if constexpr (Mode == kGatherMN) {
#pragma unroll
            for (int i = 0; i < kCount; ++i) sm[(slow0 + i * kStep) * Pitch + fast] = reg[i];
        } else {
#pragma unroll
            for (int i = 0; i < kCount; ++i) sm[fast * Pitch + slow0 + i * kStep] = reg[i];
        }
    }

  private:
    __device__ __forceinline__ static V zero_vec() {
        V z;
        T *p = reinterpret_cast<T *>(&z);
#pragma unroll
        for (int j = 0; j < W; ++j) p[j] = T(0);
        return z;
    }
    __device__ __forceinline__ static void store_vec(T *dst, const V &v) {
        const T *p = reinterpret_cast<const T *>(&v);
#pragma unroll
        for (int j = 0; j < W; ++j) dst[j] = p[j];
    }
    __device__ __forceinline__ static void load_vec(const T *src, V &v) {
        T *p = reinterpret_cast<T *>(&v);
#pragma unroll
        for (int j = 0; j < W; ++j) p[j] = src[j];
    }
};

// ---------------------------------------------------------------------------
// Register micro-tile: each thread owns TM x TN outputs split into 2x2 blocks of
// (TM/2)x(TN/2), the blocks BM/2 (resp. BN/2) apart.  A warp covers 4 rows x 8
// columns of thread positions so each shared read is at most one wavefront.
// ---------------------------------------------------------------------------
template <typename T> struct Pair;
template <> struct Pair<float> { using type = float2; };
template <> struct Pair<double> { using type = double2; };

template <typename T, int BM, int BN, int TM, int TN>
struct MicroTile {
    static constexpr int HM = TM / 2, HN = TN / 2;
    static constexpr int TY = BM / TM, TX = BN / TN;   // thread grid
    static constexpr int NT = TY * TX;
    static_assert(TX % 8 == 0 && TY % 4 == 0, "warp shape 4x8 requires TX%8==0, TY%4==0");
    static_assert(TN % 2 == 0, "columns are held in pairs");
    using P = typename Pair<T>::type;
    // Accumulators in column pairs: acc(i, j) = accp[i][j/2].{x,y}.  Pairs sit in
    // adjacent registers, the operand shape of the packed FP32 FMA.
    P accp[TM][TN / 2];
    int ty, tx;

    __device__ __forceinline__ T acc(int i, int j) const { return (j & 1) ? accp[i][j >> 1].y : accp[i][j >> 1].x; }

    __device__ __forceinline__ void init(int tid) {
        int warp = tid >> 5, lane = tid & 31;
        constexpr int WN = TX / 8;                 // warps along n
        int wm = warp / WN, wn = warp % WN;
        ty = wm * 4 + (lane >> 3);
        tx = wn * 8 + (lane & 7);
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN / 2; ++j) {
                accp[i][j].x = T(0);
                accp[i][j].y = T(0);
            }
    }
    __device__ __forceinline__ int row(int i) const {  // tile-local row of acc(i, *)
        return (i < HM) ? ty * HM + i : BM / 2 + ty * HM + (i - HM);
    }
    __device__ __forceinline__ int col(int j) const {
        return (j < HN) ? tx * HN + j : BN / 2 + tx * HN + (j - HN);
    }

    // ORD: separately rounded multiply and add (no FMA), which together with the
    // increasing-k order reproduces the reference's ordered recurrence
    // `acc += a * b` (linalg.rs:236-316) bit for bit.
    template <int BK, int PA, int PB, bool ORD = false>
    __device__ __forceinline__ void mma(const T *__restrict__ sa, const T *__restrict__ sb) {
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            T a[TM];
            P b[TN / 2];
            load_frag<HM>(sa + k * PA + ty * HM, a);
            load_frag<HM>(sa + k * PA + BM / 2 + ty * HM, a + HM);
            load_frag<HN>(sb + k * PB + tx * HN, reinterpret_cast<T *>(b));
            load_frag<HN>(sb + k * PB + BN / 2 + tx * HN, reinterpret_cast<T *>(b) + HN);
#pragma unroll
            for (int i = 0; i < TM; ++i) {
#pragma unroll
                for (int j = 0; j < TN / 2; ++j) {
                    if constexpr (ORD) {
                        accp[i][j].x = add_rn(accp[i][j].x, mul_rn(a[i], b[j].x));
                        accp[i][j].y = add_rn(accp[i][j].y, mul_rn(a[i], b[j].y));
                    } else {
                        fma2(accp[i][j], a[i], b[j]);
                    }
                }
            }
        }
    }

  private:
    // Blackwell's packed FP32 FMA: one issue slot for both lanes of a pair,
    // which leaves issue bandwidth for the shared-memory fragment loads.
    __device__ __forceinline__ static void fma2(float2 &c, float a, const float2 &b) {
#if KX_FFMA2
        c = __ffma2_rn(make_float2(a, a), b, c);
#else
        c.x = fmaf(a, b.x, c.x);
        c.y = fmaf(a, b.y, c.y);
#endif
    }
    __device__ __forceinline__ static void fma2(double2 &c, double a, const double2 &b) {
        c.x = fma(a, b.x, c.x);
        c.y = fma(a, b.y, c.y);
    }
    // H consecutive shared elements with the widest aligned vector loads.
    template <int H>
    __device__ __forceinline__ static void load_frag(const T *__restrict__ src, T *dst) {
        constexpr int bytes = H * (int)sizeof(T);
        if constexpr (bytes % 16 == 0) {
#pragma unroll
            for (int v = 0; v < bytes / 16; ++v) {
                const uint4 q = *reinterpret_cast<const uint4 *>(reinterpret_cast<const char *>(src) + 16 * v);
                *reinterpret_cast<uint4 *>(reinterpret_cast<char *>(dst) + 16 * v) = q;
            }
        } else if constexpr (bytes % 8 == 0) {
#pragma unroll
            for (int v = 0; v < bytes / 8; ++v) {
                const uint2 q = *reinterpret_cast<const uint2 *>(reinterpret_cast<const char *>(src) + 8 * v);
                *reinterpret_cast<uint2 *>(reinterpret_cast<char *>(dst) + 8 * v) = q;
            }
        } else {
#pragma unroll
            for (int v = 0; v < H; ++v) dst[v] = src[v];
        }
    }
    __device__ __forceinline__ static float mul_rn(float x, float y) { return __fmul_rn(x, y); }
    __device__ __forceinline__ static double mul_rn(double x, double y) { return __dmul_rn(x, y); }
    __device__ __forceinline__ static float add_rn(float x, float y) { return __fadd_rn(x, y); }
    __device__ __forceinline__ static double add_rn(double x, double y) { return __dadd_rn(x, y); }
};

// Tile configuration.  MinBlocks is the resident-CTA target per SM that bounds
// registers per thread (65536 / (NT * MinBlocks)).
template <typename T, int BM_, int BN_, int BK_, int TM_, int TN_, int MinBlocks_ = 1>
struct TileCfg {
    static constexpr int BM = BM_, BN = BN_, BK = BK_, TM = TM_, TN = TN_;
    static constexpr int MinBlocks = MinBlocks_;
    static constexpr int NT = (BM / TM) * (BN / TN);
    // Pitch keeps 16-byte alignment of every shared row (float4 / double2 reads).
    static constexpr int PA = BM + 16 / (int)sizeof(T);
    static constexpr int PB = BN + 16 / (int)sizeof(T);
};

// Map a linear CTA id to (tile_m, tile_n) with grouped rasterisation so that
// CTAs resident together share A row-panels and B column-panels in L2.
__device__ __forceinline__ void raster(int lin, int tiles_m, int tiles_n, int group,
                                       int &tm, int &tn) {
    int per_group = group * tiles_n;
    int g = lin / per_group;
    int first_m = g * group;
    int gm = min(tiles_m - first_m, group);
    int in = lin - g * per_group;
    tm = first_m + in % gm;
    tn = in / gm;
}

template <typename T, typename Cfg, int AM, int BMODE, bool ORD = false>
__global__ void __launch_bounds__(Cfg::NT, Cfg::MinBlocks)
gemm_simt_kernel(const __grid_constant__ GemmParams<T> p) {
    constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, NT = Cfg::NT;
    constexpr int PA = Cfg::PA, PB = Cfg::PB;
    __shared__ __align__(16) T sa[2][BK * PA];
    __shared__ __align__(16) T sb[2][BK * PB];

    const int tid = threadIdx.x;
    const int tiles_m = (p.M + BM - 1) / BM, tiles_n = (p.N + BN - 1) / BN;
    int tm, tn;
    raster(blockIdx.x, tiles_m, tiles_n, 8, tm, tn);
    const int m0 = tm * BM, n0 = tn * BN;

    const int64_t zcount = p.nbatch * p.splits;
    for (int64_t z = blockIdx.y; z < zcount; z += gridDim.y) {
        const int64_t batch = z / p.splits;
        const int split = (int)(z % p.splits);
        int64_t oa, ob, oc;
        batch_offsets(p.batch, batch, oa, ob, oc);
        const T *A = p.A + oa;
        const T *B = p.B + ob;
        const int kbeg = split * p.k_per_split;
        const int kend = min(p.K, kbeg + p.k_per_split);

        TileLoader<T, BM, BK, NT, AM, PA> la;
        TileLoader<T, BN, BK, NT, BMODE, PB> lb;
        MicroTile<T, BM, BN, Cfg::TM, Cfg::TN> mt;
        mt.init(tid);

        const int ktiles = (kend - kbeg + BK - 1) / BK;
        la.init(A, p.a_rs, p.a_cs, m0, p.M, tid);
        lb.init(B, p.b_cs, p.b_rs, n0, p.N, tid);
        if (ktiles > 0) {
            la.load(kbeg, kend);
            lb.load(kbeg, kend);
            la.store(sa[0]);
            lb.store(sb[0]);
        }
        __syncthreads();
        for (int kt = 0; kt < ktiles; ++kt) {
            const int cur = kt & 1;
            if (kt + 1 < ktiles) {
                const int k0 = kbeg + (kt + 1) * BK;
                la.load(k0, kend);
                lb.load(k0, kend);
            }
            mt.template mma<BK, PA, PB, ORD>(sa[cur], sb[cur]);
            if (kt + 1 < ktiles) {
                la.store(sa[cur ^ 1]);
                lb.store(sb[cur ^ 1]);
            }
            __syncthreads();
        }

        // Epilogue.
        T *C;
        int64_t crs, ccs;
        if (p.splits == 1) {
            C = p.C + oc;
            crs = p.c_rs;
            ccs = p.c_cs;
        } else {
            C = p.ws + ((int64_t)split * p.nbatch + batch) * (int64_t)p.M * p.N;
            crs = p.N;
            ccs = 1;
        }
        constexpr int W = Vec<T>::width;
        constexpr int HN = Cfg::TN / 2;
        // Vector stores need unit column stride, aligned rows, and in-range groups.
        const bool vec_ok = (ccs == 1) && (crs % W == 0) &&
                            ((reinterpret_cast<uintptr_t>(C) % (W * sizeof(T))) == 0) && (HN % W == 0);
#pragma unroll
        for (int i = 0; i < Cfg::TM; ++i) {
            const int gr = m0 + mt.row(i);
            if (gr >= p.M) continue;
            T *crow = C + (int64_t)gr * crs;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int cbase = mt.col(h * HN);
                const int gc = n0 + cbase;
                if (vec_ok && gc + HN <= p.N) {
#pragma unroll
                    for (int v = 0; v < HN; v += W) {
                        typename Vec<T>::type val;
                        T *pv = reinterpret_cast<T *>(&val);
#pragma unroll
                        for (int w = 0; w < W; ++w) pv[w] = mt.acc(i, h * HN + v + w);
                        *reinterpret_cast<typename Vec<T>::type *>(crow + gc + v) = val;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < HN; ++j) {
                        if (gc + j < p.N) crow[(int64_t)(gc + j) * ccs] = mt.acc(i, h * HN + j);
                    }
                }
            }
        }
        __syncthreads();
    }
}

// Deterministic split-K reduction: C(b,i,j) = sum_{s=0..S-1} ws[s][b][i][j],
// added in increasing s.
template <typename T>
__global__ void splitk_reduce_kernel(const __grid_constant__ GemmParams<T> p) {
    const int64_t mn = (int64_t)p.M * p.N;
    const int64_t total = mn * p.nbatch;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t batch = e / mn;
        const int64_t r = e % mn;
        const int i = (int)(r / p.N), j = (int)(r % p.N);
        T s = T(0);
        for (int q = 0; q < p.splits; ++q) s += p.ws[((int64_t)q * p.nbatch + batch) * mn + r];
        int64_t oa, ob, oc;
        batch_offsets(p.batch, batch, oa, ob, oc);
        p.C[oc + (int64_t)i * p.c_rs + (int64_t)j * p.c_cs] = s;
    }
}

}  // namespace kx
