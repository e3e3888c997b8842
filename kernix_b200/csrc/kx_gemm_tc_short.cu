// Split-TF32 f32 GEMM for short contractions (K <= 1024), persistent.
//
// With K <= 1024 a tile's hi*hi sum stays within one TMEM accumulation chunk
// (the one-SM kernel folds every 1024 k), so no register folding is needed and
// the epilogue can read both accumulators straight from TMEM.  That frees the
// tile's epilogue from the split warps: each CTA stays resident (one per SM),
// walks tiles round-robin, and keeps two TMEM accumulator pairs so that the
// epilogue of tile t overlaps the loads, splits and MMAs of tile t+1.  This is
// the shape of the attention score product (S = Q K^T: K = head_dim = 128),
// where the one-SM kernel spent as long on per-CTA set-up, pipeline fill and
// epilogue as on its 8 k-tiles of MMAs.
//
// Roles (448 threads):
//   warp 0      TMA producer: A and B tiles of every k-tile of every tile
//   warp 1      TMEM owner (512 columns) and MMA issuer
//   warps 2..5  epilogue: one TMEM lane quarter each (warp % 4), 128 columns,
//               written as 32 x 32 boxes through shared memory and TMA stores
//   warps 6..13 split: lo beside each raw tile (the raw tile is hi)
// TMEM: buffer b in {0, 1} holds hi*hi at columns [256 b, 256 b + 128) and the
// cross terms at [256 b + 128, 256 b + 256).  Same arithmetic, nonfinite
// fallback, bounded waits and plain TMA as the one-SM kernel (kx_gemm_tc.cu).
#include <cstring>

#include "gemm_simt.cuh"
#include "tc_common.cuh"

namespace kx {
namespace tc {
namespace shortk {

constexpr int BN = 128, NST = 6;
constexpr int B_TILE = BN * BK * 4;                   // 8 KB
constexpr int STAGE_BYTES = 2 * A_TILE + 2 * B_TILE;  // 32 KB
// Output staging: per epilogue warp two 32 x 32 f32 boxes (128-byte swizzle)
// that the TMA stores to C.
constexpr int OUT_BOX = 32 * 32 * 4;                  // 4 KB
constexpr int OUT_BYTES = 4 * 2 * OUT_BOX;            // 32 KB
constexpr int SMEM_BYTES = NST * STAGE_BYTES + OUT_BYTES + BAR_BYTES + 1024;
constexpr int NT = 448;
constexpr int EPI_WARP0 = 2, EPI_WARPS = 4;
constexpr int SPLIT_WARP0 = 6, SPLIT_WARPS = 8, SPLIT_THREADS = SPLIT_WARPS * 32;
constexpr int CHUNKS = (A_TILE + B_TILE) / 16;        // 1024 per stage
static_assert(CHUNKS % SPLIT_THREADS == 0, "split work must divide evenly");
static_assert(3 * NST + 6 <= (BAR_BYTES - 8) / 8, "barrier area");
constexpr int MAX_K = KC * BK;                        // 1024: one accumulation chunk

struct Params {
    const float *A;
    int64_t a_rs, a_bs;
    const float *B;
    int64_t b_rs, b_cs, b_bs;
    float *C;
    int64_t c_rs, c_bs;
    int M, N, K;
    int nbatch;
    int a_batched, b_batched;
    int tiles_m, tiles_n;
    int64_t ntiles;       // tiles_m * tiles_n * nbatch
    int c_tma;            // C is stored through the tensor map (else plain stores)
    uint32_t *status;
};

__device__ __forceinline__ void tile_coords(const Params &p, int64_t t, int &m0, int &n0, int &batch) {
    const int64_t per = (int64_t)p.tiles_m * p.tiles_n;
    batch = (int)(t / per);
    int tm, tn;
    raster((int)(t % per), p.tiles_m, p.tiles_n, 8, tm, tn);
    m0 = tm * BM;
    n0 = tn * BN;
}

template <bool B_MN>
__global__ void __launch_bounds__(NT, 1)
gemm_3xtf32_short_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmC, const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *out_stage = smem + NST * STAGE_BYTES;   // [epilogue warp][2] boxes of OUT_BOX bytes
    uint64_t *full = reinterpret_cast<uint64_t *>(out_stage + OUT_BYTES);
    uint64_t *conv = full + NST;
    uint64_t *empty = conv + NST;
    uint64_t *tmem_full = empty + NST;      // [2]
    uint64_t *tmem_empty = tmem_full + 2;   // [2]
    uint64_t *flag_ready = tmem_empty + 2;  // [2] the MMA thread has published the tile's nonfinite flag
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(flag_ready + 2);
    __shared__ int s_fail_storage;
    // nonfinite marks: slot i % 16 holds i + 1 once a split warp met an
    // inf/NaN input of the CTA's tile i (they run at most NST tiles ahead of
    // the MMA thread, which reads the slot after the tile's last conversion
    // and publishes it to the epilogue in tile_flag[i % 2] behind flag_ready)
    __shared__ uint32_t s_nonfinite[16];
    __shared__ uint32_t tile_flag[2];
    volatile int &s_fail = s_fail_storage;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ktiles = (p.K + BK - 1) / BK;
    // this CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...
    const int64_t my_tiles = p.ntiles > blockIdx.x ? (p.ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], SPLIT_WARPS);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], EPI_WARPS);
            mbar_init(&flag_ready[b], 1);
        }
        s_fail = 0;
        for (int i = 0; i < 16; ++i) s_nonfinite[i] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto stage_a = [&](int s) { return smem + s * STAGE_BYTES; };
    auto stage_b = [&](int s) { return smem + s * STAGE_BYTES + 2 * A_TILE; };

    if (warp == 0) {
        // ---- TMA producer: one continuous stream of k-tiles -------------
        if (lane == 0) {
            int64_t g = 0;   // k-tiles issued so far
            for (int64_t i = 0; i < my_tiles && !s_fail; ++i) {
                int m0, n0, batch;
                tile_coords(p, blockIdx.x + i * gridDim.x, m0, n0, batch);
                const int ab = p.a_batched ? batch : 0, bb = p.b_batched ? batch : 0;
                for (int kt = 0; kt < ktiles; ++kt, ++g) {
                    const int s = (int)(g % NST);
                    if (g >= NST && !mbar_wait(&empty[s], (uint32_t)(((g / NST) - 1) & 1))) {
                        s_fail = 1;
                        break;
                    }
                    mbar_expect_tx(&full[s], A_TILE + B_TILE);
                    const int k0 = kt * BK;
                    tma_load_3d(stage_a(s), &tmA, k0, m0, ab, &full[s]);
                    if constexpr (B_MN) {
#pragma unroll
                        for (int j = 0; j < BN / 32; ++j)
                            tma_load_3d(stage_b(s) + j * 2048, &tmB, n0 + 32 * j, k0, bb, &full[s]);
                    } else {
                        tma_load_3d(stage_b(s), &tmB, k0, n0, bb, &full[s]);
                    }
                }
            }
            // drain: the last copy issued into each stage has landed
            for (int s = 0; s < NST && s < g; ++s) {
                const int64_t last = s + NST * ((g - 1 - s) / NST);
                mbar_wait(&full[s], (uint32_t)((last / NST) & 1));
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer ------------------------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32<BN>(B_MN);
            int64_t g = 0;
            for (int64_t i = 0; i < my_tiles && !s_fail; ++i) {
                const int b = (int)(i & 1);
                // the epilogue of tile i - 2 has read this buffer
                if (i >= 2 && !mbar_wait(&tmem_empty[b], (uint32_t)(((i - 2) >> 1) & 1))) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(b * 256), cross = acc + 128;
                for (int kt = 0; kt < ktiles; ++kt, ++g) {
                    const int s = (int)(g % NST);
                    if (!mbar_wait(&conv[s], (uint32_t)((g / NST) & 1))) {
                        s_fail = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_hi = smem_u32(stage_a(s)), a_lo = a_hi + A_TILE;
                    const uint32_t b_hi = smem_u32(stage_b(s)), b_lo = b_hi + B_TILE;
#pragma unroll
                    for (int ks = 0; ks < BK / 8; ++ks) {
                        const uint64_t dah = desc_k_sw64(a_hi + ks * 32), dal = desc_k_sw64(a_lo + ks * 32);
                        uint64_t dbh, dbl;
                        if constexpr (B_MN) {
                            dbh = desc_mn_sw128(b_hi + ks * 1024, 2048, 512);
                            dbl = desc_mn_sw128(b_lo + ks * 1024, 2048, 512);
                        } else {
                            dbh = desc_k_sw64(b_hi + ks * 32);
                            dbl = desc_k_sw64(b_lo + ks * 32);
                        }
                        const uint32_t first = (kt > 0 || ks > 0) ? 1u : 0u;
                        mma_tf32(acc, dah, dbh, idesc, first);
                        mma_tf32(cross, dah, dbl, idesc, first);
                        mma_tf32(cross, dal, dbh, idesc, 1u);
                    }
                    mma_commit(&empty[s]);
                }
                if (s_fail) break;
                mma_commit(&tmem_full[b]);
                // every split warp's mark for this tile precedes its arrives
                tile_flag[b] = s_nonfinite[i & 15] == (uint32_t)(i + 1) ? 1u : 0u;
                mbar_arrive(&flag_ready[b]);
            }
            if (s_fail) {   // release epilogue warps waiting on either buffer
                mma_commit(&tmem_full[0]);
                mma_commit(&tmem_full[1]);
                mbar_arrive(&flag_ready[0]);
                mbar_arrive(&flag_ready[1]);
            }
        }
    } else if (warp >= SPLIT_WARP0) {
        // ---- split warps -----------------------------------------------
        const int wt = threadIdx.x - SPLIT_WARP0 * 32;
        int64_t g = 0;
        for (int64_t i = 0; i < my_tiles && !s_fail; ++i) {
            uint32_t bad = 0;
            for (int kt = 0; kt < ktiles; ++kt, ++g) {
                const int s = (int)(g % NST);
                if (!mbar_wait(&full[s], (uint32_t)((g / NST) & 1))) {
                    s_fail = 1;
                    break;
                }
                bad |= split_stage<CHUNKS / SPLIT_THREADS, SPLIT_THREADS>(smem_u32(stage_a(s)), wt, CHUNKS, A_TILE / 16,
                                                                     2 * A_TILE, A_TILE, B_TILE);
                if (bad) atomicMax(&s_nonfinite[i & 15], (uint32_t)(i + 1));   // before this k-tile's arrive
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(&conv[s]);
            }
        }
    } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + EPI_WARPS) {
        // ---- epilogue warps ----------------------------------------------
        const int quarter = warp & 3;
        uint32_t sc = 0;    // staging boxes filled by this warp (buffer sc % 2)
        for (int64_t i = 0; i < my_tiles && !s_fail; ++i) {
            const int b = (int)(i & 1);
            if (!mbar_wait(&tmem_full[b], (uint32_t)((i >> 1) & 1)) ||
                !mbar_wait(&flag_ready[b], (uint32_t)((i >> 1) & 1))) {
                s_fail = 1;
                break;
            }
            tc_fence_after();
            if (s_fail) break;
            int m0, n0, batch;
            tile_coords(p, blockIdx.x + i * gridDim.x, m0, n0, batch);
            const int row = m0 + quarter * 32 + lane;
            const bool in_rows = row < p.M;
            const bool nonfinite = *reinterpret_cast<volatile uint32_t *>(&tile_flag[b]) != 0;
            const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * 256);
            float *crow = p.C + (int64_t)batch * p.c_bs + (int64_t)(in_rows ? row : 0) * p.c_rs + n0;
            const bool vec = (p.c_rs % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) && (p.c_bs % 4 == 0);
            if (!nonfinite && p.c_tma) {
                // 32-column boxes: this lane's row into the swizzled staging
                // box (16-byte chunk j of row r at chunk j ^ (r % 8): each
                // quarter-warp store covers 32 distinct banks), then one TMA
                // store per box, clipped at the matrix edges.
                const uint32_t sbase = smem_u32(out_stage) + (uint32_t)((warp - EPI_WARP0) * 2 * OUT_BOX);
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t r0[16], r1[16], x0[16], x1[16];
                    tmem_ld16(lane_base + (uint32_t)(c * 32), r0);
                    tmem_ld16(lane_base + (uint32_t)(c * 32 + 16), r1);
                    tmem_ld16(lane_base + 128u + (uint32_t)(c * 32), x0);
                    tmem_ld16(lane_base + 128u + (uint32_t)(c * 32 + 16), x1);
                    tmem_wait_ld();
                    const uint32_t box = sbase + (uint32_t)((sc & 1) * OUT_BOX);
                    if (lane == 0) bulk_wait_read<1>();     // the store that last read this box is done
                    __syncwarp();
                    const uint32_t row = box + (uint32_t)lane * 128;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        sts_v4_f32(row + (uint32_t)((j ^ (lane & 7)) << 4),
                                   __uint_as_float(r0[4 * j]) + __uint_as_float(x0[4 * j]),
                                   __uint_as_float(r0[4 * j + 1]) + __uint_as_float(x0[4 * j + 1]),
                                   __uint_as_float(r0[4 * j + 2]) + __uint_as_float(x0[4 * j + 2]),
                                   __uint_as_float(r0[4 * j + 3]) + __uint_as_float(x0[4 * j + 3]));
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        sts_v4_f32(row + (uint32_t)(((j + 4) ^ (lane & 7)) << 4),
                                   __uint_as_float(r1[4 * j]) + __uint_as_float(x1[4 * j]),
                                   __uint_as_float(r1[4 * j + 1]) + __uint_as_float(x1[4 * j + 1]),
                                   __uint_as_float(r1[4 * j + 2]) + __uint_as_float(x1[4 * j + 2]),
                                   __uint_as_float(r1[4 * j + 3]) + __uint_as_float(x1[4 * j + 3]));
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_3d(&tmC, out_stage + (box - smem_u32(out_stage)), n0 + c * 32, m0 + quarter * 32,
                                     batch);
                        bulk_commit();
                    }
                    ++sc;
                }
            } else if (!nonfinite) {
#pragma unroll 1
                for (int c = 0; c < BN / 16; ++c) {
                    uint32_t r0[16], r1[16];
                    tmem_ld16(lane_base + (uint32_t)(c * 16), r0);
                    tmem_ld16(lane_base + 128u + (uint32_t)(c * 16), r1);
                    tmem_wait_ld();
                    if (!in_rows) continue;
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r0[j]) + __uint_as_float(r1[j]);
                    const int gcol = n0 + c * 16;
                    if (vec && gcol + 16 <= p.N) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            *reinterpret_cast<float4 *>(crow + c * 16 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (gcol + j < p.N) crow[c * 16 + j] = v[j];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[b]);   // TMEM read: the buffer may be reused
            if (nonfinite && in_rows) {
                // inf/NaN among this tile's inputs: f32 FMA in k order (IEEE
                // propagation of the CUDA-core path)
                const int ab = p.a_batched ? batch : 0, bb = p.b_batched ? batch : 0;
                const float *arow = p.A + (int64_t)ab * p.a_bs + (int64_t)row * p.a_rs;
                const float *bbat = p.B + (int64_t)bb * p.b_bs;
                for (int j = 0; j < BN && n0 + j < p.N; ++j) {
                    const float *bcol = bbat + (int64_t)(n0 + j) * p.b_cs;
                    float accv = 0.0f;
                    for (int k = 0; k < p.K; ++k) accv = fmaf(arow[k], bcol[(int64_t)k * p.b_rs], accv);
                    crow[j] = accv;
                }
            }
        }
        if (lane == 0) bulk_wait_all();   // every TMA store of C has completed
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
    if (threadIdx.x == 0 && s_fail) atomicOr(p.status, KX_TIMEOUT_FLAG);
}

}  // namespace shortk
}  // namespace tc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int run_gemm_tc_short(Handle *h, const GemmParams<float> &p, const char **kernel_name) {
    using namespace tc;
    using namespace tc::shortk;
    if (p.K > MAX_K) return KX_DECLINED;
    const bool b_mn = p.b_cs == 1 && (p.b_rs * 4) % 16 == 0 && p.b_rs > 0;
    const int nb = (int)p.nbatch;
    const int64_t a_bs = p.batch.ndims == 1 ? p.batch.a_str[0] : 0;
    const int64_t b_bs = p.batch.ndims == 1 ? p.batch.b_str[0] : 0;
    const int64_t c_bs = p.batch.ndims == 1 ? p.batch.c_str[0] : 0;
    const int a_batched = (nb > 1 && a_bs > 0) ? 1 : 0;
    const int b_batched = (nb > 1 && b_bs > 0) ? 1 : 0;
    const int64_t a_rs = p.M == 1 ? 16 : p.a_rs;
    CUtensorMap ma, mb;
    const uint64_t a_s2 = a_batched ? (uint64_t)a_bs * 4 : (uint64_t)((a_rs * 4 * (int64_t)p.M + 15) / 16 * 16);
    if (!make_map(&ma, p.A, (uint64_t)p.K, (uint64_t)p.M, a_batched ? (uint64_t)nb : 1, (uint64_t)a_rs * 4, a_s2, BK,
                  BM, CU_TENSOR_MAP_SWIZZLE_64B))
        return KX_DECLINED;
    bool okb;
    if (b_mn) {
        const uint64_t s2 = b_batched ? (uint64_t)b_bs * 4 : (uint64_t)((p.b_rs * 4 * (int64_t)p.K + 15) / 16 * 16);
        okb = make_map(&mb, p.B, (uint64_t)p.N, (uint64_t)p.K, b_batched ? (uint64_t)nb : 1, (uint64_t)p.b_rs * 4, s2,
                       32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    } else {
        const uint64_t s2 = b_batched ? (uint64_t)b_bs * 4 : (uint64_t)((p.b_cs * 4 * (int64_t)p.N + 15) / 16 * 16);
        okb = make_map(&mb, p.B, (uint64_t)p.K, (uint64_t)p.N, b_batched ? (uint64_t)nb : 1, (uint64_t)p.b_cs * 4, s2,
                       BK, BN, CU_TENSOR_MAP_SWIZZLE_64B);
    }
    if (!okb) return KX_DECLINED;
    Params pp;
    std::memset(&pp, 0, sizeof(pp));
    pp.A = p.A;
    pp.a_rs = p.a_rs;
    pp.a_bs = a_bs;
    pp.B = p.B;
    pp.b_rs = p.b_rs;
    pp.b_cs = p.b_cs;
    pp.b_bs = b_bs;
    pp.C = p.C;
    pp.c_rs = p.M == 1 ? 0 : p.c_rs;
    pp.c_bs = c_bs;
    pp.M = p.M;
    pp.N = p.N;
    pp.K = p.K;
    pp.nbatch = nb;
    pp.a_batched = a_batched;
    pp.b_batched = b_batched;
    pp.tiles_m = (p.M + BM - 1) / BM;
    pp.tiles_n = (p.N + BN - 1) / BN;
    pp.ntiles = (int64_t)pp.tiles_m * pp.tiles_n * nb;
    pp.status = h->flags + kStatusWord;
    // C through a tensor map (dims N, M, batch): 16-byte aligned base and strides
    CUtensorMap mc;
    std::memset(&mc, 0, sizeof(mc));
    const bool c_batched = nb > 1;
    pp.c_tma = p.M > 1 && p.c_rs > 0 && (p.c_rs * 4) % 16 == 0 && (reinterpret_cast<uintptr_t>(p.C) & 15) == 0 &&
               (!c_batched || (c_bs > 0 && (c_bs * 4) % 16 == 0)) &&
               make_map(&mc, p.C, (uint64_t)p.N, (uint64_t)p.M, (uint64_t)nb, (uint64_t)p.c_rs * 4,
                        c_batched ? (uint64_t)c_bs * 4 : (uint64_t)((p.c_rs * 4 * (int64_t)p.M + 15) / 16 * 16), 32, 32,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    const int64_t grid = pp.ntiles < h->sm_count ? pp.ntiles : h->sm_count;
    cudaError_t ce;
    if (b_mn) {
        auto k = gemm_3xtf32_short_kernel<true>;
        ce = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (ce == cudaSuccess) {
            k<<<(unsigned)grid, NT, SMEM_BYTES, h->stream>>>(ma, mb, mc, pp);
            ce = cudaGetLastError();
        }
        *kernel_name = "tc_3xtf32_short_128x128_bmn";
    } else {
        auto k = gemm_3xtf32_short_kernel<false>;
        ce = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (ce == cudaSuccess) {
            k<<<(unsigned)grid, NT, SMEM_BYTES, h->stream>>>(ma, mb, mc, pp);
            ce = cudaGetLastError();
        }
        *kernel_name = "tc_3xtf32_short_128x128_bk";
    }
    ++h->launches;
    return ce == cudaSuccess ? KX_OK : h->cuda_fail(ce);
}

}  // namespace kx
