// Split-TF32 f32 GEMM on CTA pairs: tcgen05.mma.cta_group::2 computes a
// 256 x 256 (or 256 x 224) tile on two SMs of a cluster, each SM staging only
// its half of A (128 rows) and its half of B (128 or 112 columns).
//
// Same arithmetic as the one-SM kernel (kx_gemm_tc.cu): hi = the raw tile (the
// tensor core reads f32 as tf32 by truncation), lo = x - hi written by the
// worker warps, C = A_hi B_hi + A_hi B_lo + A_lo B_hi, the hi*hi sum folded
// into f32 registers every 1024 k, cross terms in one TMEM accumulator.
// Why pairs: per k-tile and CTA the one-SM kernel moves 24 KB by TMA, splits
// 24 KB and feeds 72 KB of operands to the tensor core; a pair CTA moves 16 KB,
// splits 16 KB and feeds 48 KB for the same FLOPs, which relieves shared
// memory (the limiter of the one-SM kernel) by a third.
//
// Roles in each CTA of the pair (384 threads):
//   warp 0      TMA: this CTA's A half and B half into stage s (own barrier)
//   warp 1      TMEM owner (cta_group::2 alloc in both CTAs); in the leader
//               (cluster rank 0) also the MMA issuer for the pair
//   warps 4..11 workers: lo split of this CTA's halves, then an arrive on the
//               LEADER's conversion barrier (remote for the peer); chunk folds
//               from this CTA's TMEM rows; epilogue of this CTA's 128 rows.
// The leader's MMA completions are committed to the barriers of both CTAs
// (one commit per CTA, addressed through the cluster window).  Cluster
// barriers order the start (barriers initialised before any remote arrive),
// the epilogue (both CTAs' nonfinite flags final) and the exit (no CTA leaves
// while the pair's MMAs may still read its shared memory).  Every mbarrier
// wait is bounded; TMA loads are plain (no cluster multicast) and read this
// GPU's memory only.
#include <cstring>

#include "gemm_simt.cuh"
#include "tc_common.cuh"

namespace kx {
namespace tc {
namespace pair {

constexpr int BMP = 256;                       // pair tile rows
constexpr int B_TILE = 128 * BK * 4;           // 8 KB of B staging per CTA and stage
constexpr int NST = 6;                         // stages
constexpr int STAGE_BYTES = 2 * A_TILE + 2 * B_TILE;   // 32 KB
constexpr int SMEM_BYTES = NST * STAGE_BYTES + BAR_BYTES + 1024;
static_assert(3 * NST + 2 <= (BAR_BYTES - 8) / 8, "barrier area");

// Pair tile width 2 * HB: 256, or 224 when that packs the pairs into whole
// waves (a 512 x 8192 piece: 74 pairs = 148 CTAs).  Each CTA's B half is HB
// columns; MN-major B is loaded as four 32-column boxes (128 columns, the
// last 16 unused at HB = 112), K-major B as an HB-row box.
template <int HB> struct Pair {
    static_assert(HB == 128 || HB == 112, "pair half width");
    static constexpr int BNP = 2 * HB;
    static constexpr int HALF_COLS = HB;       // accumulator columns per worker thread
    static constexpr int B_BYTES_MN = B_TILE;          // four 32-column boxes
    static constexpr int B_BYTES_K = HB * BK * 4;      // one HB-row box
};

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
    uint32_t *status;
};

template <bool B_MN, int HB>
__global__ void __launch_bounds__(NTHREADS, 1)
gemm_3xtf32_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ Params p) {
    using PT = Pair<HB>;
    constexpr int BNP = PT::BNP, HALF_COLS = PT::HALF_COLS;
    constexpr int B_BYTES = B_MN ? PT::B_BYTES_MN : PT::B_BYTES_K;
    constexpr int CHUNKS = (A_TILE + B_BYTES) / 16;
    constexpr int CONV_ITERS = (CHUNKS + WORK_THREADS - 1) / WORK_THREADS;
    extern __shared__ uint8_t smem_raw[];
    // The same dynamic offsets in both CTAs: the MMA reads the peer's halves
    // at the addresses the leader's descriptors name.
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + NST * STAGE_BYTES);
    uint64_t *conv = full + NST;
    uint64_t *empty = conv + NST;
    uint64_t *chunk_full = empty + NST;
    uint64_t *chunk_empty = chunk_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(chunk_empty + 1);
    __shared__ int s_fail_storage;
    __shared__ uint32_t s_nonfinite_storage;
    volatile int &s_fail = s_fail_storage;
    volatile uint32_t &s_nonfinite = s_nonfinite_storage;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const uint32_t peer = rank ^ 1u;
    const int tiles_m = (p.M + BMP - 1) / BMP, tiles_n = (p.N + BNP - 1) / BNP;
    int tm, tn;
    raster((int)(blockIdx.x >> 1), tiles_m, tiles_n, 8, tm, tn);
    const int m0 = tm * BMP + (int)rank * BM;        // this CTA's 128 rows
    const int n0 = tn * BNP;                         // the pair's columns
    const int nb0 = n0 + (int)rank * HB;             // this CTA's staged B columns
    const int batch = blockIdx.y;
    const int ab = p.a_batched ? batch : 0, bb = p.b_batched ? batch : 0;
    const int ktiles = (p.K + BK - 1) / BK;
    const int nchunks = (ktiles + KC - 1) / KC;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 2 * WORK_WARPS);     // both CTAs' workers (used in the leader)
            mbar_init(&empty[s], 1);
        }
        mbar_init(chunk_full, 1);
        mbar_init(chunk_empty, 2 * WORK_WARPS);
        s_fail = 0;
        s_nonfinite = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync_any();       // both CTAs' barriers initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto stage_a = [&](int s) { return smem + s * STAGE_BYTES; };
    auto stage_b = [&](int s) { return smem + s * STAGE_BYTES + 2 * A_TILE; };

    if (warp == 0) {
        // ---- TMA producer: this CTA's halves ---------------------------
        if (lane == 0) {
            int issued = 0;
            for (int kt = 0; kt < ktiles && !s_fail; ++kt) {
                const int s = kt % NST;
                if (kt >= NST && !mbar_wait(&empty[s], ((kt / NST) - 1) & 1)) {
                    s_fail = 1;
                    break;
                }
                mbar_expect_tx(&full[s], A_TILE + B_BYTES);
                const int k0 = kt * BK;
                tma_load_3d(stage_a(s), &tmA, k0, m0, ab, &full[s]);
                if constexpr (B_MN) {
#pragma unroll
                    for (int j = 0; j < B_TILE / 2048; ++j)
                        tma_load_3d(stage_b(s) + j * 2048, &tmB, nb0 + 32 * j, k0, bb, &full[s]);
                } else {
                    tma_load_3d(stage_b(s), &tmB, k0, nb0, bb, &full[s]);
                }
                issued = kt + 1;
            }
            for (int s = 0; s < NST && s < issued; ++s) {
                const int last = s + NST * ((issued - 1 - s) / NST);
                mbar_wait(&full[s], (last / NST) & 1);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer (leader only) ----------------------------------
        if (leader && lane == 0) {
            constexpr uint32_t idesc = idesc_pair(B_MN, BNP);
            const uint32_t chunk_full_peer = map_to(smem_u32(chunk_full), peer);
            for (int kt = 0; kt < ktiles; ++kt) {
                const int s = kt % NST;
                const int chunk = kt / KC, kin = kt % KC;
                if (kin == 0 && chunk > 0 && (s_fail || !mbar_wait_cluster(chunk_empty, (chunk - 1) & 1))) {
                    s_fail = 1;
                    break;
                }
                if (s_fail || !mbar_wait_cluster(&conv[s], (kt / NST) & 1)) {
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
                    mma_pair(tmem, dah, dbh, idesc, (kin > 0 || ks > 0) ? 1u : 0u);
                    mma_pair(tmem + XCOL, dah, dbl, idesc, (kt > 0 || ks > 0) ? 1u : 0u);
                    mma_pair(tmem + XCOL, dal, dbh, idesc, 1u);
                }
                const uint32_t e_local = smem_u32(&empty[s]);
                commit_pair(e_local);
                commit_pair(map_to(e_local, peer));
                if (kin == KC - 1 || kt == ktiles - 1) {
                    commit_pair(smem_u32(chunk_full));
                    commit_pair(chunk_full_peer);
                }
            }
            if (s_fail) {   // release workers of both CTAs waiting on a chunk
                commit_pair(smem_u32(chunk_full));
                commit_pair(chunk_full_peer);
            }
        }
    } else if (warp >= WORK_WARP0) {
        // ---- workers: split, fold, epilogue ----------------------------
        const int wt = threadIdx.x - WORK_WARP0 * 32;
        const int quarter = warp & 3;
        const int col0 = ((warp - WORK_WARP0) >> 2) * HALF_COLS;
        const uint32_t conv_leader0 = map_to(smem_u32(&conv[0]), 0);
        const uint32_t chunk_empty_leader = map_to(smem_u32(chunk_empty), 0);
        float sum[HALF_COLS];
#pragma unroll
        for (int j = 0; j < HALF_COLS; ++j) sum[j] = 0.0f;
        int chunk = 0;
        for (int kt = 0; kt < ktiles; ++kt) {
            const int s = kt % NST;
            if (s_fail || !mbar_wait(&full[s], (kt / NST) & 1)) {
                s_fail = 1;
                break;
            }
            uint32_t bad = 0;
            uint8_t *base = stage_a(s);
#pragma unroll
            for (int j = 0; j < CONV_ITERS; ++j) {
                const int c = wt + j * WORK_THREADS;
                if (CHUNKS % WORK_THREADS != 0 && c >= CHUNKS) break;   // only what the TMA wrote
                const bool in_a = c < A_TILE / 16;
                float4 *hp = reinterpret_cast<float4 *>(base + (in_a ? c * 16 : 2 * A_TILE + (c - A_TILE / 16) * 16));
                float4 *lp = reinterpret_cast<float4 *>(reinterpret_cast<uint8_t *>(hp) + (in_a ? A_TILE : B_TILE));
                const float4 v = *hp;
                float4 l;
                l.x = v.x - tf32_trunc(v.x);
                l.y = v.y - tf32_trunc(v.y);
                l.z = v.z - tf32_trunc(v.z);
                l.w = v.w - tf32_trunc(v.w);
                bad |= nonfinite_bits(v.x) | nonfinite_bits(v.y) | nonfinite_bits(v.z) | nonfinite_bits(v.w);
                *lp = l;
            }
            if (bad) s_nonfinite = 1u;
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(conv_leader0 + (uint32_t)(s * 8));
            if (kt % KC == KC - 1 || kt == ktiles - 1) {
                if (!mbar_wait(chunk_full, chunk & 1)) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                if (s_fail) break;
                tmem_accumulate(tmem, quarter, col0, sum);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(chunk_empty_leader);
                ++chunk;
            }
        }
        // Pair-wide barrier: both CTAs' nonfinite flags are final after it.
        tc_fence_before();
        cluster_sync_any();
        tc_fence_after();
        const uint32_t nonfinite = s_nonfinite | ld_cluster_u32(map_to(smem_u32((const void *)&s_nonfinite_storage), peer));
        const int row = m0 + quarter * 32 + lane;
        if (!s_fail && chunk == nchunks) {
            if (nonfinite) {
                // inf/NaN in the pair's inputs: this CTA's rows by f32 FMA in k order
                if (row < p.M) {
                    const float *arow = p.A + (int64_t)ab * p.a_bs + (int64_t)row * p.a_rs;
                    const float *bbat = p.B + (int64_t)bb * p.b_bs;
                    float *crow = p.C + (int64_t)batch * p.c_bs + (int64_t)row * p.c_rs;
                    for (int j = 0; j < HALF_COLS && n0 + col0 + j < p.N; ++j) {
                        const float *bcol = bbat + (int64_t)(n0 + col0 + j) * p.b_cs;
                        float acc = 0.0f;
                        for (int k = 0; k < p.K; ++k) acc = fmaf(arow[k], bcol[(int64_t)k * p.b_rs], acc);
                        crow[n0 + col0 + j] = acc;
                    }
                }
            } else {
                const bool in_rows = row < p.M;
                float *crow = p.C + (int64_t)batch * p.c_bs + (int64_t)(in_rows ? row : 0) * p.c_rs + n0 + col0;
                const bool vec = (p.c_rs % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                                 (p.c_bs % 4 == 0);
#pragma unroll
                for (int c = 0; c < HALF_COLS / 16; ++c) {
                    uint32_t r[16];
                    tmem_ld16(tmem + XCOL + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(col0 + c * 16), r);
                    tmem_wait_ld();
                    if (!in_rows) continue;
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = sum[c * 16 + j] + __uint_as_float(r[j]);
                    const int gcol = n0 + col0 + c * 16;
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
        }
    }
    if (warp < WORK_WARP0) cluster_sync_any();   // the non-worker threads meet the workers' pair-wide barrier
    tc_fence_before();
    cluster_sync_any();       // no CTA leaves while the pair's MMAs or peer arrives may touch it
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
    if (threadIdx.x == 0 && s_fail) atomicOr(p.status, KX_TIMEOUT_FLAG);
}

}  // namespace pair
}  // namespace tc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

template <bool B_MN, int HB>
cudaError_t launch_pair(Handle *h, const CUtensorMap &ma, const CUtensorMap &mb, const tc::pair::Params &pp,
                        int64_t pair_tiles, int nb) {
    using namespace tc;
    using namespace tc::pair;
    auto k = gemm_3xtf32_pair_kernel<B_MN, HB>;
    cudaError_t ce = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (ce != cudaSuccess) return ce;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * pair_tiles), (unsigned)nb, 1);
    cfg.blockDim = dim3(NTHREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = h->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ce = cudaLaunchKernelEx(&cfg, k, ma, mb, pp);
    if (ce != cudaSuccess) return ce;
    return cudaGetLastError();
}

}  // namespace

// Pair kernel for products large enough to fill the SMs with 256 x 256 tiles;
// same operand rules as the one-SM kernel (tc_eligible).
int run_gemm_tc_pair(Handle *h, const GemmParams<float> &p, const char **kernel_name) {
    using namespace tc;
    using namespace tc::pair;
    const bool b_mn = p.b_cs == 1 && (p.b_rs * 4) % 16 == 0 && p.b_rs > 0;
    const int nb = (int)p.nbatch;
    const int64_t a_bs = p.batch.ndims == 1 ? p.batch.a_str[0] : 0;
    const int64_t b_bs = p.batch.ndims == 1 ? p.batch.b_str[0] : 0;
    const int64_t c_bs = p.batch.ndims == 1 ? p.batch.c_str[0] : 0;
    const int a_batched = (nb > 1 && a_bs > 0) ? 1 : 0;
    const int b_batched = (nb > 1 && b_bs > 0) ? 1 : 0;
    if (p.M < 2 * BM) return KX_DECLINED;
    // pair width by the wave model (as the one-SM kernel's tile width)
    const int64_t pm = (p.M + BMP - 1) / BMP;
    // (the 224-wide pair stages 128 B columns for 112: weighted 5 % heavier)
    auto cost = [&](int bnp) {
        const int64_t ctas = 2 * pm * ((p.N + bnp - 1) / bnp) * nb;
        return (double)((ctas + h->sm_count - 1) / h->sm_count) * (bnp + 32) * (bnp == 224 ? 1.05 : 1.0);
    };
    const int hb = cost(224) < cost(256) ? 112 : 128;
    CUtensorMap ma, mb;
    const uint64_t a_s2 = a_batched ? (uint64_t)a_bs * 4 : (uint64_t)((p.a_rs * 4 * (int64_t)p.M + 15) / 16 * 16);
    if (!make_map(&ma, p.A, (uint64_t)p.K, (uint64_t)p.M, a_batched ? (uint64_t)nb : 1, (uint64_t)p.a_rs * 4, a_s2,
                  BK, BM, CU_TENSOR_MAP_SWIZZLE_64B))
        return KX_DECLINED;
    bool okb;
    if (b_mn) {
        const uint64_t s2 = b_batched ? (uint64_t)b_bs * 4 : (uint64_t)((p.b_rs * 4 * (int64_t)p.K + 15) / 16 * 16);
        okb = make_map(&mb, p.B, (uint64_t)p.N, (uint64_t)p.K, b_batched ? (uint64_t)nb : 1, (uint64_t)p.b_rs * 4, s2,
                       32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    } else {
        const uint64_t s2 = b_batched ? (uint64_t)b_bs * 4 : (uint64_t)((p.b_cs * 4 * (int64_t)p.N + 15) / 16 * 16);
        okb = make_map(&mb, p.B, (uint64_t)p.K, (uint64_t)p.N, b_batched ? (uint64_t)nb : 1, (uint64_t)p.b_cs * 4, s2,
                       BK, (uint32_t)hb, CU_TENSOR_MAP_SWIZZLE_64B);
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
    pp.c_rs = p.c_rs;
    pp.c_bs = c_bs;
    pp.M = p.M;
    pp.N = p.N;
    pp.K = p.K;
    pp.nbatch = nb;
    pp.a_batched = a_batched;
    pp.b_batched = b_batched;
    pp.status = h->flags + kStatusWord;
    const int bnp = 2 * hb;
    const int64_t pair_tiles = pm * ((p.N + bnp - 1) / bnp);
    if (2 * pair_tiles > INT32_MAX) return KX_DECLINED;
    cudaError_t ce;
    if (b_mn)
        ce = hb == 128 ? launch_pair<true, 128>(h, ma, mb, pp, pair_tiles, nb)
                       : launch_pair<true, 112>(h, ma, mb, pp, pair_tiles, nb);
    else
        ce = hb == 128 ? launch_pair<false, 128>(h, ma, mb, pp, pair_tiles, nb)
                       : launch_pair<false, 112>(h, ma, mb, pp, pair_tiles, nb);
    *kernel_name = hb == 128 ? (b_mn ? "tc_3xtf32_pair_256x256_bmn" : "tc_3xtf32_pair_256x256_bk")
                             : (b_mn ? "tc_3xtf32_pair_256x224_bmn" : "tc_3xtf32_pair_256x224_bk");
    ++h->launches;
    return ce == cudaSuccess ? KX_OK : h->cuda_fail(ce);
}

}  // namespace kx
