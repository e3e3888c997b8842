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
// ---------------------------------------------------------------------------
template <typename T, int Rows, int BK, int NT, int Mode, int Pitch>
struct TileLoader {
    using V = typename Vec<T>::type;
    static constexpr int W = Vec<T>::width;
    static constexpr bool kVector = (Mode == kVecK || Mode == kVecMN);
    static constexpr int kCount = kVector ? (Rows * BK) / (W * NT) : (Rows * BK) / NT;
    static_assert(kCount >= 1, "tile too small for thread count");
    static_assert(kVector ? (Rows * BK) % (W * NT) == 0 : (Rows * BK) % NT == 0, "tile/thread mismatch");

    T reg[kVector ? kCount * W : kCount];

    // Load tile rows [r0, r0+Rows), k [k0, k0+BK) with zero fill outside
    // [0,R) x [0,kend).
    __device__ __forceinline__ void load(const T *__restrict__ ptr, int64_t s_r, int64_t s_k,
                                         int r0, int R, int k0, int kend, int tid) {
        if constexpr (Mode == kVecK) {
            // vector index v: r = v % Rows, kv = v / Rows (threads walk r fastest)
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                int v = tid + i * NT;
                int r = v % Rows, kv = v / Rows;
                int gr = r0 + r, gk = k0 + kv * W;
                V val;
                if (gr < R && gk < kend) {
                    val = __ldg(reinterpret_cast<const V *>(ptr + (int64_t)gr * s_r + gk));
                } else {
                    val = zero_vec();
                }
                store_vec(&reg[i * W], val);
            }
        } else if constexpr (Mode == kVecMN) {
            constexpr int RV = Rows / W;
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                int v = tid + i * NT;
                int rv = v % RV, kk = v / RV;
                int gr = r0 + rv * W, gk = k0 + kk;
                V val;
                if (gr < R && gk < kend) {
                    val = __ldg(reinterpret_cast<const V *>(ptr + (int64_t)gk * s_k + gr));
                } else {
                    val = zero_vec();
                }
                store_vec(&reg[i * W], val);
            }
        } else if constexpr (Mode == kGatherMN) {
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                int v = tid + i * NT;
                int r = v % Rows, kk = v / Rows;
                int gr = r0 + r, gk = k0 + kk;
                reg[i] = (gr < R && gk < kend) ? __ldg(ptr + (int64_t)gr * s_r + (int64_t)gk * s_k) : T(0);
            }
        } else {
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                int v = tid + i * NT;
                int kk = v % BK, r = v / BK;
                int gr = r0 + r, gk = k0 + kk;
                reg[i] = (gr < R && gk < kend) ? __ldg(ptr + (int64_t)gr * s_r + (int64_t)gk * s_k) : T(0);
            }
        }
    }

    __device__ __forceinline__ void store(T *sm, int tid) const {
        if constexpr (Mode == kVecK) {
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                int v = tid + i * NT;
                int r = v % Rows, kv = v / Rows;
#pragma unroll
                for (int j = 0; j < W; ++j) sm[(kv * W + j) * Pitch + r] = reg[i * W + j];
            }
        } else if constexpr (Mode == kVecMN) {
            constexpr int RV = Rows / W;
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                int v = tid + i * NT;
                int rv = v % RV, kk = v / RV;
                V val;
                load_vec(&reg[i * W], val);
                *reinterpret_cast<V *>(&sm[kk * Pitch + rv * W]) = val;
            }
        } else if constexpr (Mode == kGatherMN) {
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                int v = tid + i * NT;
                int r = v % Rows, kk = v / Rows;
                sm[kk * Pitch + r] = reg[i];
            }
        } else {
#pragma unroll
            for (int i = 0; i < kCount; ++i) {
                int v = tid + i * NT;
                int kk = v % BK, r = v / BK;
                sm[kk * Pitch + r] = reg[i];
            }
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
template <typename T, int BM, int BN, int TM, int TN>
struct MicroTile {
    static constexpr int HM = TM / 2, HN = TN / 2;
    static constexpr int TY = BM / TM, TX = BN / TN;   // thread grid
    static constexpr int NT = TY * TX;
    static_assert(TX % 8 == 0 && TY % 4 == 0, "warp shape 4x8 requires TX%8==0, TY%4==0");
    T acc[TM][TN];
    int ty, tx;

    __device__ __forceinline__ void init(int tid) {
        int warp = tid >> 5, lane = tid & 31;
        constexpr int WN = TX / 8;                 // warps along n
        int wm = warp / WN, wn = warp % WN;
        ty = wm * 4 + (lane >> 3);
        tx = wn * 8 + (lane & 7);
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[i][j] = T(0);
    }
    __device__ __forceinline__ int row(int i) const {  // tile-local row of acc[i][*]
        return (i < HM) ? ty * HM + i : BM / 2 + ty * HM + (i - HM);
    }
    __device__ __forceinline__ int col(int j) const {
        return (j < HN) ? tx * HN + j : BN / 2 + tx * HN + (j - HN);
    }

    template <int BK, int PA, int PB>
    __device__ __forceinline__ void mma(const T *__restrict__ sa, const T *__restrict__ sb) {
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            T a[TM], b[TN];
#pragma unroll
            for (int i = 0; i < HM; ++i) {
                a[i] = sa[k * PA + ty * HM + i];
                a[HM + i] = sa[k * PA + BM / 2 + ty * HM + i];
            }
#pragma unroll
            for (int j = 0; j < HN; ++j) {
                b[j] = sb[k * PB + tx * HN + j];
                b[HN + j] = sb[k * PB + BN / 2 + tx * HN + j];
            }
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
        }
    }
};

// Tile configuration.
template <typename T, int BM_, int BN_, int BK_, int TM_, int TN_>
struct TileCfg {
    static constexpr int BM = BM_, BN = BN_, BK = BK_, TM = TM_, TN = TN_;
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

template <typename T, typename Cfg, int AM, int BMODE>
__global__ void __launch_bounds__(Cfg::NT)
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
        if (ktiles > 0) {
            la.load(A, p.a_rs, p.a_cs, m0, p.M, kbeg, kend, tid);
            lb.load(B, p.b_cs, p.b_rs, n0, p.N, kbeg, kend, tid);
            la.store(sa[0], tid);
            lb.store(sb[0], tid);
        }
        __syncthreads();
        for (int kt = 0; kt < ktiles; ++kt) {
            const int cur = kt & 1;
            if (kt + 1 < ktiles) {
                const int k0 = kbeg + (kt + 1) * BK;
                la.load(A, p.a_rs, p.a_cs, m0, p.M, k0, kend, tid);
                lb.load(B, p.b_cs, p.b_rs, n0, p.N, k0, kend, tid);
            }
            mt.template mma<BK, PA, PB>(sa[cur], sb[cur]);
            if (kt + 1 < ktiles) {
                la.store(sa[cur ^ 1], tid);
                lb.store(sb[cur ^ 1], tid);
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
                        for (int w = 0; w < W; ++w) pv[w] = mt.acc[i][h * HN + v + w];
                        *reinterpret_cast<typename Vec<T>::type *>(crow + gc + v) = val;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < HN; ++j) {
                        if (gc + j < p.N) crow[(int64_t)(gc + j) * ccs] = mt.acc[i][h * HN + j];
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
