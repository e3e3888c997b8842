// conv2d on the 5th-generation tensor cores: split-TF32 implicit GEMM whose
// B operand (the im2col columns) is gathered straight from the NCHW input by
// the worker warps, so no column buffer ever exists.
//
// GEMM view (kernix-ops neural.rs:200-302, conv_impl's native branch): per
// group, out[co][(img,oy,ox)] = sum_k weight[co][k] * col[k][(img,oy,ox)] with
// k = (ci, ky, kx) in the reference's im2col order and col[k][pixel] the
// input element under tap k, zero on padding.  M = output channels of the
// group, N = batch * oh * ow pixels, K = cin/groups * kh * kw.
//
// Per CTA: 128 output channels x 128 pixels, 384 threads.
//   warp 0       TMA producer: the weight tile (K-major, 64-byte swizzle)
//   warp 1       TMEM owner and MMA issuer (3 x 2 tcgen05.mma kind::tf32 per stage)
//   warps 4..11  workers: gather the B tile for stage s (one pixel and 8 taps
//                per thread, loads for stage s+1 issued before stage s is
//                written), write its hi (raw) and lo parts in the canonical
//                K-major no-swizzle layout, split the weight tile's lo part,
//                fold hi*hi chunks into registers, and store the NCHW output
// A per-CTA table of (ci, ky, kx) offsets in shared memory and a per-pixel
// mask of in-bounds taps turn each gathered element into one table read, one
// bit test and one 4-byte cp.async (zero-filled on padding).  Split-TF32 arithmetic, chunked folding and
// the nonfinite fallback are those of the GEMM kernel (kx_gemm_tc.cu): with
// inf/NaN in a tile's inputs the tile is recomputed with f32 FMA in k order,
// as the SIMT implicit GEMM does.  Every mbarrier wait is bounded.
#include <algorithm>
#include <cstring>

#include "gemm_simt.cuh"
#include "tc_common.cuh"

namespace kx {
namespace tc {
namespace conv {

// Pixels per tile: 256, or 128 when that packs the tiles into fewer waves.
template <int BN> struct Tile {
    static constexpr int B_TILE = BN * BK * 4;                   // 16 KB at 256
    static constexpr int STAGE_BYTES = 2 * A_TILE + 2 * B_TILE;  // 48 KB at 256
    static constexpr int HALF_COLS = BN / 2;                     // columns per worker thread
    // Stage ring: the gather for k-tile kt + LOOKAHEAD goes into the stage of
    // k-tile kt + LOOKAHEAD - NST, so LOOKAHEAD stages cover the gather latency
    // and NST - LOOKAHEAD MMA groups may be in flight when a worker reuses a stage.
    static constexpr int NST = BN == 128 ? 6 : 4;
    static constexpr int LOOKAHEAD = NST / 2;
    static constexpr int FIXED_SMEM = NST * STAGE_BYTES + BAR_BYTES + 1024;
};
constexpr int SMEM_LIMIT = 227 * 1024;

struct Params {
    const float *x;       // input at its origin
    const float *w;       // weights at their origin (used by the nonfinite fallback)
    float *y;             // output at its origin, C-contiguous NCHW
    int64_t xs[4];        // input strides (elements)
    int64_t ws0;          // weight stride between output channels; taps are contiguous
    int64_t ih, iw, oh, ow, hw;
    int64_t co_total, cog, cg;
    int kh, kw, sy, sx, py, px, dy, dx;
    int kk;               // cg * kh * kw
    int64_t ncols;        // batch * oh * ow
    uint32_t *status;
};

struct Tap {
    int64_t x_off;        // ci*xs1 + ky*dy*xs2 + kx*dx*xs3
    int32_t r;            // ky*kw + kx: bit of the pixel's in-bounds mask; 63 past the last tap
    int32_t unused;
};
constexpr int PAD_TAP = 63;

// B tiles (BN pixels x 16 taps) use the canonical K-major no-swizzle layout:
// 8x4 core matrices of 128 contiguous bytes, the four along k adjacent (LBO
// 128 B), row groups 512 B apart (SBO); element (r, k) of core matrix
// 4*(r/8) + k/4 sits at byte 16*(r%8) + 4*(k%4) within it.
// 4-byte asynchronous copy into shared memory; `valid` false zero-fills
// (the source is not read).
__device__ __forceinline__ void cp4(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int BN>
__global__ void __launch_bounds__(NTHREADS, 1)
conv_3xtf32_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ Params p) {
    using TL = Tile<BN>;
    constexpr int B_TILE = TL::B_TILE, STAGE_BYTES = TL::STAGE_BYTES, HALF_COLS = TL::HALF_COLS;
    constexpr int NST = TL::NST, LOOKAHEAD = TL::LOOKAHEAD;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + NST * STAGE_BYTES);
    uint64_t *conv = full + NST;
    uint64_t *empty = conv + NST;
    uint64_t *chunk_full = empty + NST;
    uint64_t *chunk_empty = chunk_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(chunk_empty + 1);
    Tap *taps = reinterpret_cast<Tap *>(smem + NST * STAGE_BYTES + BAR_BYTES);
    __shared__ int s_fail_storage, s_nonfinite_storage;
    volatile int &s_fail = s_fail_storage;
    volatile int &s_nonfinite = s_nonfinite_storage;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = (int)((p.cog + BM - 1) / BM), tiles_n = (int)((p.ncols + BN - 1) / BN);
    int tm, tn;
    raster(blockIdx.x, tiles_m, tiles_n, 8, tm, tn);
    const int m0 = tm * BM;
    const int64_t n0 = (int64_t)tn * BN;
    const int grp = blockIdx.y;
    const int ktiles = (p.kk + BK - 1) / BK;
    const int nchunks = (ktiles + KC - 1) / KC;

    for (int k = threadIdx.x; k < ktiles * BK; k += NTHREADS) {
        Tap t;
        t.unused = 0;
        if (k < p.kk) {
            const int khw = p.kh * p.kw;
            const int ci = k / khw, r = k % khw;
            const int ky = r / p.kw, kx = r % p.kw;
            t.r = r;
            t.x_off = (int64_t)ci * p.xs[1] + (int64_t)(ky * p.dy) * p.xs[2] + (int64_t)(kx * p.dx) * p.xs[3];
        } else {
            t.r = PAD_TAP;
            t.x_off = 0;
        }
        taps[k] = t;
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], WORK_WARPS);
            mbar_init(&empty[s], 1);
        }
        mbar_init(chunk_full, 1);
        mbar_init(chunk_empty, WORK_WARPS);
        s_fail = 0;
        s_nonfinite = 0;
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
        // ---- TMA producer: weight tiles ---------------------------------
        if (lane == 0) {
            int issued = 0;
            for (int kt = 0; kt < ktiles && !s_fail; ++kt) {
                const int s = kt % NST;
                if (kt >= NST && !mbar_wait(&empty[s], ((kt / NST) - 1) & 1)) {
                    s_fail = 1;
                    break;
                }
                mbar_expect_tx(&full[s], A_TILE);
                tma_load_3d(stage_a(s), &tmW, kt * BK, m0, grp, &full[s]);
                issued = kt + 1;
            }
            for (int s = 0; s < NST && s < issued; ++s) {
                const int last = s + NST * ((issued - 1 - s) / NST);
                mbar_wait(&full[s], (last / NST) & 1);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----------------------------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32<BN>(false);
            for (int kt = 0; kt < ktiles; ++kt) {
                const int s = kt % NST;
                const int chunk = kt / KC, kin = kt % KC;
                if (kin == 0 && chunk > 0 && (s_fail || !mbar_wait(chunk_empty, (chunk - 1) & 1))) {
                    s_fail = 1;
                    break;
                }
                if (s_fail || !mbar_wait(&conv[s], (kt / NST) & 1)) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t a_hi = smem_u32(stage_a(s)), a_lo = a_hi + A_TILE;
                const uint32_t b_hi = smem_u32(stage_b(s)), b_lo = b_hi + B_TILE;
#pragma unroll
                for (int ks = 0; ks < BK / 8; ++ks) {
                    const uint64_t dah = desc_k_sw64(a_hi + ks * 32), dal = desc_k_sw64(a_lo + ks * 32);
                    const uint64_t dbh = desc_k_none(b_hi + ks * 256, 128, 512);
                    const uint64_t dbl = desc_k_none(b_lo + ks * 256, 128, 512);
                    mma_tf32(tmem, dah, dbh, idesc, (kin > 0 || ks > 0) ? 1u : 0u);
                    mma_tf32(tmem + XCOL, dah, dbl, idesc, (kt > 0 || ks > 0) ? 1u : 0u);
                    mma_tf32(tmem + XCOL, dal, dbh, idesc, 1u);
                }
                mma_commit(&empty[s]);
                if (kin == KC - 1 || kt == ktiles - 1) mma_commit(chunk_full);
            }
            if (s_fail) mma_commit(chunk_full);
        }
    } else if (warp >= WORK_WARP0) {
        // ---- workers: gather B, split, fold, epilogue --------------------
        const int wt = threadIdx.x - WORK_WARP0 * 32;           // 0..255
        const int quarter = warp & 3;
        const int col0 = ((warp - WORK_WARP0) >> 2) * HALF_COLS;
        // Gather ownership: worker warp ww owns the CM core matrices
        // [ww*CM, (ww+1)*CM) of every B stage (core matrix cm = row group cm/4,
        // k group cm%4, 8 pixels x 4 taps = 128 contiguous bytes); lane l of a
        // warp instruction fetches pixel 8*(cm/4) + l/4, tap 4*(cm%4) + l%4, so
        // one instruction fills one core matrix with 32 bank-distinct 4-byte
        // copies.  A thread therefore gathers for NPIX pixels, 4 taps each.
        constexpr int CM = BN / 16;                 // core matrices per warp per stage
        constexpr int NPIX = CM / 4;
        const int ww = warp - WORK_WARP0;
        const int ih = (int)p.ih, iw = (int)p.iw;
        const float *xpix[NPIX];
        uint64_t inb[NPIX];      // bit r: tap r = ky*kw + kx of the pixel lands inside the input
#pragma unroll
        for (int q = 0; q < NPIX; ++q) {
            const int prow = 8 * (ww * CM / 4 + q) + (lane >> 2);
            const int64_t gcol = n0 + prow;
            xpix[q] = p.x;
            inb[q] = 0;
            if (gcol < p.ncols) {
                const int64_t img = gcol / p.hw, pix = gcol % p.hw;
                const int64_t oy = pix / p.ow, ox = pix % p.ow;
                const int iy0 = (int)(oy * p.sy - p.py), ix0 = (int)(ox * p.sx - p.px);
                xpix[q] = p.x + img * p.xs[0] + (int64_t)grp * p.cg * p.xs[1] + (int64_t)iy0 * p.xs[2] +
                          (int64_t)ix0 * p.xs[3];
                for (int r = 0; r < p.kh * p.kw; ++r) {
                    const int iy = iy0 + (r / p.kw) * p.dy, ix = ix0 + (r % p.kw) * p.dx;
                    if (iy >= 0 && iy < ih && ix >= 0 && ix < iw) inb[q] |= 1ull << r;
                }
            }
        }
        // Gather k-tile kt into its stage with 4-byte asynchronous copies
        // (zero on padding and past the last tap).
        auto gather = [&](int kt) {
            uint8_t *bh = stage_b(kt % NST) + ww * CM * 128 + lane * 4;
            const Tap *tk = taps + kt * BK + (lane & 3);
#pragma unroll
            for (int i = 0; i < CM; ++i) {
                const Tap t = tk[4 * (i & 3)];
                const bool ok = (inb[i >> 2] >> t.r) & 1;
                cp4(bh + i * 128, ok ? xpix[i >> 2] + t.x_off : p.x, ok);
            }
        };
        float sum[HALF_COLS];
#pragma unroll
        for (int j = 0; j < HALF_COLS; ++j) sum[j] = 0.0f;
        // the first LOOKAHEAD stages start free
#pragma unroll
        for (int j = 0; j < LOOKAHEAD; ++j) {
            if (j < ktiles) gather(j);
            cp_commit();
        }
        int chunk = 0;
        for (int kt = 0; kt < ktiles; ++kt) {
            const int s = kt % NST;
            cp_wait<LOOKAHEAD - 1>();                 // this thread's copies for k-tile kt have landed
            __syncwarp();                             // ... and those of the rest of its warp
            if (s_fail || !mbar_wait(&full[s], (kt / NST) & 1)) {
                s_fail = 1;
                break;
            }
            uint32_t bad = 0;
            // lo of the warp's own core matrices: CM * 8 chunks of 16 bytes
            uint8_t *bh = stage_b(s) + ww * CM * 128, *bl = bh + B_TILE;
#pragma unroll
            for (int jc = 0; jc < CM / 4; ++jc) {
                const uint32_t off = (uint32_t)(lane + 32 * jc) * 16;
                const float4 v = *reinterpret_cast<const float4 *>(bh + off);   // hi: the gathered values
                float4 l;
                l.x = v.x - tf32_trunc(v.x);
                l.y = v.y - tf32_trunc(v.y);
                l.z = v.z - tf32_trunc(v.z);
                l.w = v.w - tf32_trunc(v.w);
                bad |= nonfinite_bits(v.x) | nonfinite_bits(v.y) | nonfinite_bits(v.z) | nonfinite_bits(v.w);
                *reinterpret_cast<float4 *>(bl + off) = l;
            }
            // weight tile: 512 16-byte chunks, two per thread, lo beside hi
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float4 *hp = reinterpret_cast<float4 *>(stage_a(s) + (wt + j * WORK_THREADS) * 16);
                float4 *lp = reinterpret_cast<float4 *>(reinterpret_cast<uint8_t *>(hp) + A_TILE);
                const float4 v = *hp;
                float4 l;
                l.x = v.x - tf32_trunc(v.x);
                l.y = v.y - tf32_trunc(v.y);
                l.z = v.z - tf32_trunc(v.z);
                l.w = v.w - tf32_trunc(v.w);
                bad |= nonfinite_bits(v.x) | nonfinite_bits(v.y) | nonfinite_bits(v.z) | nonfinite_bits(v.w);
                *lp = l;
            }
            if (bad) s_nonfinite = 1;
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(&conv[s]);
            // Gather k-tile kt + LOOKAHEAD into the stage of k-tile
            // kt + LOOKAHEAD - NST, once the MMAs that read that stage have completed.
            const int ahead = kt + LOOKAHEAD, prev = ahead - NST;
            if (ahead < ktiles) {
                if (prev >= 0 && !mbar_wait(&empty[prev % NST], (prev / NST) & 1)) {
                    s_fail = 1;
                    break;
                }
                gather(ahead);
            }
            cp_commit();
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
                if (lane == 0) mbar_arrive(chunk_empty);
                ++chunk;
            }
        }
        cp_wait<0>();    // no copy of this thread may land after the CTA's shared memory is released
        // ---- epilogue: row = output channel, columns = pixels -----------
        const int co = m0 + quarter * 32 + lane;
        const bool row_ok = co < p.cog;
        const int64_t co_abs = (int64_t)grp * p.cog + co;
        if (!s_fail && chunk == nchunks) {
            if (s_nonfinite) {
                // inf/NaN among this tile's inputs: f32 FMA in k order
                if (row_ok) {
                    const float *wrow = p.w + co_abs * p.ws0;
                    for (int j = 0; j < HALF_COLS; ++j) {
                        const int64_t c = n0 + col0 + j;
                        if (c >= p.ncols) break;
                        const int64_t img = c / p.hw, pix = c % p.hw;
                        const int64_t oy = pix / p.ow, ox = pix % p.ow;
                        const int y0 = (int)(oy * p.sy - p.py), x0 = (int)(ox * p.sx - p.px);
                        const int64_t base = img * p.xs[0] + (int64_t)grp * p.cg * p.xs[1] + (int64_t)y0 * p.xs[2] +
                                             (int64_t)x0 * p.xs[3];
                        float acc = 0.0f;
                        for (int k = 0; k < p.kk; ++k) {
                            const Tap t = taps[k];
                            const int iy = y0 + (t.r / p.kw) * p.dy, ix = x0 + (t.r % p.kw) * p.dx;
                            const float xv = (iy >= 0 && iy < ih && ix >= 0 && ix < iw) ? p.x[base + t.x_off] : 0.0f;
                            acc = fmaf(wrow[k], xv, acc);
                        }
                        p.y[(img * p.co_total + co_abs) * p.hw + pix] = acc;
                    }
                }
            } else {
                const bool vec_ok = (p.hw % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.y) & 15) == 0);
#pragma unroll
                for (int c = 0; c < HALF_COLS / 16; ++c) {
                    uint32_t r[16];
                    tmem_ld16(tmem + XCOL + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(col0 + c * 16), r);
                    tmem_wait_ld();
                    if (!row_ok) continue;
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = sum[c * 16 + j] + __uint_as_float(r[j]);
                    const int64_t c0 = n0 + col0 + c * 16;
                    const int64_t img = c0 / p.hw, pix = c0 % p.hw;
                    if (vec_ok && c0 + 16 <= p.ncols && pix + 16 <= p.hw) {
                        float *dst = p.y + (img * p.co_total + co_abs) * p.hw + pix;
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            *reinterpret_cast<float4 *>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int64_t cc = c0 + j;
                            if (cc < p.ncols) p.y[((cc / p.hw) * p.co_total + co_abs) * p.hw + cc % p.hw] = v[j];
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
    if (threadIdx.x == 0 && s_fail) atomicOr(p.status, KX_TIMEOUT_FLAG);
}


// ---------------------------------------------------------------------------
// CTA pairs: tcgen05.mma.cta_group::2 on a 256-channel x 256-pixel tile.  Each
// CTA takes 128 output channels of weights (TMA) and gathers 128 pixels of the
// B tile, so every input element is gathered once per 256 channels instead of
// once per 128, and each SM feeds the tensor core a third less operand data.
// Pair protocol as in kx_gemm_tc2.cu: remote arrives on the leader's barriers,
// the leader's completions committed to both CTAs, three cluster barriers.
// ---------------------------------------------------------------------------
constexpr int PAIR_NST = 6;
constexpr int PAIR_B_TILE = 128 * BK * 4;                          // 8 KB
constexpr int PAIR_STAGE = 2 * A_TILE + 2 * PAIR_B_TILE;           // 32 KB
constexpr int PAIR_FIXED_SMEM = PAIR_NST * PAIR_STAGE + BAR_BYTES + 1024;
static_assert(3 * PAIR_NST + 2 <= (BAR_BYTES - 8) / 8, "barrier area");

__global__ void __launch_bounds__(NTHREADS, 1)
conv_3xtf32_pair_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ Params p) {
    constexpr int NST = PAIR_NST, LOOKAHEAD = NST / 2, B_TILE = PAIR_B_TILE, STAGE_BYTES = PAIR_STAGE;
    constexpr int BNP = 256, HALF_COLS = 128;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + NST * STAGE_BYTES);
    uint64_t *conv = full + NST;
    uint64_t *empty = conv + NST;
    uint64_t *chunk_full = empty + NST;
    uint64_t *chunk_empty = chunk_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(chunk_empty + 1);
    Tap *taps = reinterpret_cast<Tap *>(smem + NST * STAGE_BYTES + BAR_BYTES);
    __shared__ int s_fail_storage;
    __shared__ uint32_t s_nonfinite_storage;
    volatile int &s_fail = s_fail_storage;
    volatile uint32_t &s_nonfinite = s_nonfinite_storage;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const uint32_t peer = rank ^ 1u;
    const int tiles_m = (int)((p.cog + 255) / 256), tiles_n = (int)((p.ncols + BNP - 1) / BNP);
    int tm, tn;
    raster((int)(blockIdx.x >> 1), tiles_m, tiles_n, 8, tm, tn);
    const int m0 = tm * 256 + (int)rank * BM;            // this CTA's output channels
    const int64_t n0 = (int64_t)tn * BNP;                // the pair's pixels
    const int64_t nb0 = n0 + (int64_t)rank * 128;        // this CTA's gathered pixels
    const int grp = blockIdx.y;
    const int ktiles = (p.kk + BK - 1) / BK;
    const int nchunks = (ktiles + KC - 1) / KC;

    for (int k = threadIdx.x; k < ktiles * BK; k += NTHREADS) {
        Tap t;
        t.unused = 0;
        if (k < p.kk) {
            const int khw = p.kh * p.kw;
            const int ci = k / khw, r = k % khw;
            const int ky = r / p.kw, kx = r % p.kw;
            t.r = r;
            t.x_off = (int64_t)ci * p.xs[1] + (int64_t)(ky * p.dy) * p.xs[2] + (int64_t)(kx * p.dx) * p.xs[3];
        } else {
            t.r = PAD_TAP;
            t.x_off = 0;
        }
        taps[k] = t;
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 2 * WORK_WARPS);
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
    cluster_sync_any();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto stage_a = [&](int s) { return smem + s * STAGE_BYTES; };
    auto stage_b = [&](int s) { return smem + s * STAGE_BYTES + 2 * A_TILE; };

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            for (int kt = 0; kt < ktiles && !s_fail; ++kt) {
                const int s = kt % NST;
                if (kt >= NST && !mbar_wait(&empty[s], ((kt / NST) - 1) & 1)) {
                    s_fail = 1;
                    break;
                }
                mbar_expect_tx(&full[s], A_TILE);
                tma_load_3d(stage_a(s), &tmW, kt * BK, m0, grp, &full[s]);
                issued = kt + 1;
            }
            for (int s = 0; s < NST && s < issued; ++s) {
                const int last = s + NST * ((issued - 1 - s) / NST);
                mbar_wait(&full[s], (last / NST) & 1);
            }
        }
    } else if (warp == 1) {
        if (leader && lane == 0) {
            constexpr uint32_t idesc = idesc_pair(false, BNP);
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
                    const uint64_t dbh = desc_k_none(b_hi + ks * 256, 128, 512);
                    const uint64_t dbl = desc_k_none(b_lo + ks * 256, 128, 512);
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
            if (s_fail) {
                commit_pair(smem_u32(chunk_full));
                commit_pair(chunk_full_peer);
            }
        }
    } else if (warp >= WORK_WARP0) {
        const int wt = threadIdx.x - WORK_WARP0 * 32;
        const int quarter = warp & 3;
        const int col0 = ((warp - WORK_WARP0) >> 2) * HALF_COLS;
        const uint32_t conv_leader0 = map_to(smem_u32(&conv[0]), 0);
        const uint32_t chunk_empty_leader = map_to(smem_u32(chunk_empty), 0);
        // gather ownership as the one-SM kernel at 128 pixels: 8 core
        // matrices per warp, two pixels per thread
        constexpr int CM = 8, NPIX = 2;
        const int ww = warp - WORK_WARP0;
        const int ih = (int)p.ih, iw = (int)p.iw;
        const float *xpix[NPIX];
        uint64_t inb[NPIX];
#pragma unroll
        for (int q = 0; q < NPIX; ++q) {
            const int prow = 8 * (ww * CM / 4 + q) + (lane >> 2);
            const int64_t gcol = nb0 + prow;
            xpix[q] = p.x;
            inb[q] = 0;
            if (gcol < p.ncols) {
                const int64_t img = gcol / p.hw, pix = gcol % p.hw;
                const int64_t oy = pix / p.ow, ox = pix % p.ow;
                const int iy0 = (int)(oy * p.sy - p.py), ix0 = (int)(ox * p.sx - p.px);
                xpix[q] = p.x + img * p.xs[0] + (int64_t)grp * p.cg * p.xs[1] + (int64_t)iy0 * p.xs[2] +
                          (int64_t)ix0 * p.xs[3];
                for (int r = 0; r < p.kh * p.kw; ++r) {
                    const int iy = iy0 + (r / p.kw) * p.dy, ix = ix0 + (r % p.kw) * p.dx;
                    if (iy >= 0 && iy < ih && ix >= 0 && ix < iw) inb[q] |= 1ull << r;
                }
            }
        }
        auto gather = [&](int kt) {
            uint8_t *bh = stage_b(kt % NST) + ww * CM * 128 + lane * 4;
            const Tap *tk = taps + kt * BK + (lane & 3);
#pragma unroll
            for (int i = 0; i < CM; ++i) {
                const Tap t = tk[4 * (i & 3)];
                const bool ok = (inb[i >> 2] >> t.r) & 1;
                cp4(bh + i * 128, ok ? xpix[i >> 2] + t.x_off : p.x, ok);
            }
        };
        float sum[HALF_COLS];
#pragma unroll
        for (int j = 0; j < HALF_COLS; ++j) sum[j] = 0.0f;
#pragma unroll
        for (int j = 0; j < LOOKAHEAD; ++j) {
            if (j < ktiles) gather(j);
            cp_commit();
        }
        int chunk = 0;
        for (int kt = 0; kt < ktiles; ++kt) {
            const int s = kt % NST;
            cp_wait<LOOKAHEAD - 1>();
            __syncwarp();
            if (s_fail || !mbar_wait(&full[s], (kt / NST) & 1)) {
                s_fail = 1;
                break;
            }
            uint32_t bad = 0;
            uint8_t *bh = stage_b(s) + ww * CM * 128, *bl = bh + B_TILE;
#pragma unroll
            for (int jc = 0; jc < CM / 4; ++jc) {
                const uint32_t off = (uint32_t)(lane + 32 * jc) * 16;
                const float4 v = *reinterpret_cast<const float4 *>(bh + off);
                float4 l;
                l.x = v.x - tf32_trunc(v.x);
                l.y = v.y - tf32_trunc(v.y);
                l.z = v.z - tf32_trunc(v.z);
                l.w = v.w - tf32_trunc(v.w);
                bad |= nonfinite_bits(v.x) | nonfinite_bits(v.y) | nonfinite_bits(v.z) | nonfinite_bits(v.w);
                *reinterpret_cast<float4 *>(bl + off) = l;
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float4 *hp = reinterpret_cast<float4 *>(stage_a(s) + (wt + j * WORK_THREADS) * 16);
                float4 *lp = reinterpret_cast<float4 *>(reinterpret_cast<uint8_t *>(hp) + A_TILE);
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
            const int ahead = kt + LOOKAHEAD, prev = ahead - NST;
            if (ahead < ktiles) {
                if (prev >= 0 && !mbar_wait(&empty[prev % NST], (prev / NST) & 1)) {
                    s_fail = 1;
                    break;
                }
                gather(ahead);
            }
            cp_commit();
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
        cp_wait<0>();
        tc_fence_before();
        cluster_sync_any();     // pair-wide: both CTAs' nonfinite flags are final
        tc_fence_after();
        const uint32_t nonfinite = s_nonfinite | ld_cluster_u32(map_to(smem_u32((const void *)&s_nonfinite_storage), peer));
        const int co = m0 + quarter * 32 + lane;
        const bool row_ok = co < p.cog;
        const int64_t co_abs = (int64_t)grp * p.cog + co;
        if (!s_fail && chunk == nchunks) {
            if (nonfinite) {
                if (row_ok) {
                    const float *wrow = p.w + co_abs * p.ws0;
                    for (int j = 0; j < HALF_COLS; ++j) {
                        const int64_t c = n0 + col0 + j;
                        if (c >= p.ncols) break;
                        const int64_t img = c / p.hw, pix = c % p.hw;
                        const int64_t oy = pix / p.ow, ox = pix % p.ow;
                        const int y0 = (int)(oy * p.sy - p.py), x0 = (int)(ox * p.sx - p.px);
                        const int64_t base = img * p.xs[0] + (int64_t)grp * p.cg * p.xs[1] + (int64_t)y0 * p.xs[2] +
                                             (int64_t)x0 * p.xs[3];
                        float acc = 0.0f;
                        for (int k = 0; k < p.kk; ++k) {
                            const Tap t = taps[k];
                            const int iy = y0 + (t.r / p.kw) * p.dy, ix = x0 + (t.r % p.kw) * p.dx;
                            const float xv = (iy >= 0 && iy < ih && ix >= 0 && ix < iw) ? p.x[base + t.x_off] : 0.0f;
                            acc = fmaf(wrow[k], xv, acc);
                        }
                        p.y[(img * p.co_total + co_abs) * p.hw + pix] = acc;
                    }
                }
            } else {
                const bool vec_ok = (p.hw % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.y) & 15) == 0);
#pragma unroll
                for (int c = 0; c < HALF_COLS / 16; ++c) {
                    uint32_t r[16];
                    tmem_ld16(tmem + XCOL + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(col0 + c * 16), r);
                    tmem_wait_ld();
                    if (!row_ok) continue;
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = sum[c * 16 + j] + __uint_as_float(r[j]);
                    const int64_t c0 = n0 + col0 + c * 16;
                    const int64_t img = c0 / p.hw, pix = c0 % p.hw;
                    if (vec_ok && c0 + 16 <= p.ncols && pix + 16 <= p.hw) {
                        float *dst = p.y + (img * p.co_total + co_abs) * p.hw + pix;
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            *reinterpret_cast<float4 *>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int64_t cc = c0 + j;
                            if (cc < p.ncols) p.y[((cc / p.hw) * p.co_total + co_abs) * p.hw + cc % p.hw] = v[j];
                        }
                    }
                }
            }
        }
    }
    if (warp < WORK_WARP0) cluster_sync_any();
    tc_fence_before();
    cluster_sync_any();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
    if (threadIdx.x == 0 && s_fail) atomicOr(p.status, KX_TIMEOUT_FLAG);
}

// ---------------------------------------------------------------------------
// Patch-staged CTA pair: 256 output channels x 224 pixels of one image.
//
// The gathered kernels above read every input element once per tap from L2
// (nine times for a 3x3 filter).  Here each CTA stages, per 16 input
// channels, the input rows under its 112 output pixels with ONE TMA box
// (zero-filled outside the image, which is the padding), and the worker warps
// build each k-tile's im2col tile from shared memory.  16 channels are
// exactly kh*kw k-tiles, so the k-tiles of a chunk never straddle two chunks;
// two chunk buffers let the next chunk's box land while this one is used.
// Needs a unit inner input stride, the other strides 16-byte multiples, and
// a patch row (the output row's input columns, widened to 16-byte bounds) of
// at most 256 floats.
//   warp 0   weight tiles by TMA (as above)
//   warp 1   TMEM owner; the pair leader's lane 0 issues the MMAs (N = 224)
//   warp 2   patch boxes by TMA
//   warps 4..11  build B hi/lo from the patch, fold the hi*hi chunks, store
//            the output
// The weights' lo parts are split once per call (split_weights_kernel) and
// come by TMA beside the hi tile.  Persistent: one CTA pair per two SMs walks
// the tiles; the TMEM accumulators of a tile are read into registers before
// the next tile's MMAs start, so its stores overlap the next tile's loads.
// ---------------------------------------------------------------------------
// HB pixels per CTA (half the pair's width).
constexpr int PP_HB = 112;
template <int HB> struct PatchTile {
    static constexpr int B_TILE = HB * BK * 4;                   // 8 KB at 128
    static constexpr int STAGE = 2 * A_TILE + 2 * B_TILE;        // 32 KB at 128
    static_assert(STAGE % 1024 == 0, "stage alignment");
    static_assert(HB % 16 == 0 && HB >= 96 && HB <= 128 && WORK_WARPS == 8,
                  "B build: 8 warps = 4 tap groups x 2 halves of HB/2 pixels, 32 < HB/2 <= 64");
};
constexpr int PP_NST = 6;                                // most stages; fewer when the patch buffers are large
constexpr int PP_CH = 16;                                // input channels per patch chunk
static_assert(3 * PP_NST + 2 + 4 + 1 <= BAR_BYTES / 8, "barrier area");

struct PatchGeom {
    int x0;                  // first input column of every patch (a multiple of 4; negative on left padding)
    int pitch;               // floats per patch row (a multiple of 4, at most 256)
    int prows;               // input rows per patch
    int tpi;                 // pair tiles per image
    int nimg;                // images
    uint32_t patch_bytes;    // one chunk: PP_CH * prows * pitch * 4
    uint32_t patch_stride;   // patch_bytes rounded up to 1 KB
};

template <int NST, int HB>
__global__ void __launch_bounds__(NTHREADS, 1)
conv_3xtf32_patch_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmWlo,
                         const __grid_constant__ CUtensorMap tmX, const __grid_constant__ Params p,
                         const __grid_constant__ PatchGeom g) {
    constexpr int BNP = 2 * HB, B_TILE = PatchTile<HB>::B_TILE, STAGE_BYTES = PatchTile<HB>::STAGE;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *patch = smem + NST * STAGE_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(patch + 2 * g.patch_stride);
    uint64_t *conv = full + NST;
    uint64_t *empty = conv + NST;
    uint64_t *chunk_full = empty + NST;
    uint64_t *chunk_empty = chunk_full + 1;
    uint64_t *pfull = chunk_empty + 1;      // [2]: patch chunk landed
    uint64_t *pempty = pfull + 2;           // [2]: patch chunk read by every worker warp
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pempty + 2);
    int32_t *tap_off = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(full) + BAR_BYTES);
    __shared__ int s_fail_storage;
    volatile int &s_fail = s_fail_storage;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const uint32_t peer = rank ^ 1u;
    const int tiles_m = (int)(p.cog / 256), tiles_n = g.nimg * g.tpi;
    const int ntiles = tiles_m * tiles_n;
    const int pair0 = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
    const int hw = (int)p.hw, ow = (int)p.ow;
    const int grp = blockIdx.y;
    const int khw = p.kh * p.kw;
    const int ktiles = (p.kk + BK - 1) / BK;
    const int npatch = (ktiles + khw - 1) / khw;
    const int ch_floats = g.prows * g.pitch;
    // tile -> this CTA's output channels m0, image, the pair's first pixel p0
    // and this CTA's first pixel q0 (112 pixels from it)
    auto tile_of = [&](int t, int &m0, int &img, int &p0, int &q0) {
        int tm, tn;
        raster(t, tiles_m, tiles_n, 8, tm, tn);
        m0 = tm * 256 + (int)rank * BM;
        img = tn / g.tpi;
        p0 = (tn % g.tpi) * BNP;
        q0 = p0 + (int)rank * HB;
    };

    // patch offset of chunk-local tap kl = (ci, ky, kx)
    for (int kl = threadIdx.x; kl < PP_CH * khw; kl += NTHREADS) {
        const int ci = kl / khw, r = kl % khw;
        tap_off[kl] = ci * ch_floats + (r / p.kw) * p.dy * g.pitch + (r % p.kw) * p.dx;
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 2 * WORK_WARPS);
            mbar_init(&empty[s], 1);
        }
        mbar_init(chunk_full, 1);
        mbar_init(chunk_empty, 2 * WORK_WARPS);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&pfull[b], 1);
            mbar_init(&pempty[b], WORK_WARPS);
        }
        s_fail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync_any();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto stage_a = [&](int s) { return smem + s * STAGE_BYTES; };

    // Every role walks the same tiles (pair0, pair0 + npairs, ...) with
    // stage, patch-buffer and TMEM-chunk counters that run on across tiles.
    if (warp == 0) {
        if (lane == 0) {
            uint32_t gkt = 0;
            for (int t = pair0; t < ntiles && !s_fail; t += npairs) {
                int m0, img, p0, q0;
                tile_of(t, m0, img, p0, q0);
                for (int kt = 0; kt < ktiles; ++kt, ++gkt) {
                    const uint32_t s = gkt % NST;
                    if (gkt >= NST && !mbar_wait(&empty[s], ((gkt / NST) - 1) & 1)) {
                        s_fail = 1;
                        break;
                    }
                    mbar_expect_tx(&full[s], 2 * A_TILE);
                    tma_load_3d(stage_a(s), &tmW, kt * BK, m0, grp, &full[s]);
                    tma_load_3d(stage_a(s) + A_TILE, &tmWlo, kt * BK, m0, grp, &full[s]);
                }
            }
            // no TMA write may still be in flight when the CTA exits
            for (uint32_t s = 0; s < NST && s < gkt; ++s) {
                const uint32_t last = s + NST * ((gkt - 1 - s) / NST);
                mbar_wait(&full[s], (last / NST) & 1);
            }
        }
    } else if (warp == 1) {
        if (leader && lane == 0) {
            constexpr uint32_t idesc = idesc_pair(false, BNP);
            const uint32_t chunk_full_peer = map_to(smem_u32(chunk_full), peer);
            uint32_t gkt = 0, gc = 0;
            for (int t = pair0; t < ntiles && !s_fail; t += npairs) {
                for (int kt = 0; kt < ktiles; ++kt, ++gkt) {
                    const uint32_t s = gkt % NST;
                    const int kin = kt % KC;
                    // the workers have folded the previous chunk (and, at a
                    // tile's first k-tile, read the last tile's accumulators)
                    if (kin == 0 && gc > 0 && (s_fail || !mbar_wait_cluster(chunk_empty, (gc - 1) & 1))) {
                        s_fail = 1;
                        break;
                    }
                    if (s_fail || !mbar_wait_cluster(&conv[s], (gkt / NST) & 1)) {
                        s_fail = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_hi = smem_u32(stage_a(s)), a_lo = a_hi + A_TILE;
                    const uint32_t b_hi = a_hi + 2 * A_TILE, b_lo = b_hi + B_TILE;
#pragma unroll
                    for (int ks = 0; ks < BK / 8; ++ks) {
                        const uint64_t dah = desc_k_sw64(a_hi + ks * 32), dal = desc_k_sw64(a_lo + ks * 32);
                        const uint64_t dbh = desc_k_sw64(b_hi + ks * 32), dbl = desc_k_sw64(b_lo + ks * 32);
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
                        ++gc;
                    }
                }
            }
            if (s_fail) {
                commit_pair(smem_u32(chunk_full));
                commit_pair(chunk_full_peer);
            }
        }
    } else if (warp == 2) {
        if (lane == 0) {
            uint32_t gj = 0;
            const int c0 = grp * (int)p.cg;
            for (int t = pair0; t < ntiles && !s_fail; t += npairs) {
                int m0, img, p0, q0;
                tile_of(t, m0, img, p0, q0);
                const int iy0 = (min(q0, hw - 1) / ow) * p.sy - p.py;   // the patch's first input row
                for (int j = 0; j < npatch; ++j, ++gj) {
                    const uint32_t b = gj & 1;
                    if (gj >= 2 && !mbar_wait(&pempty[b], ((gj >> 1) - 1) & 1)) {
                        s_fail = 1;
                        break;
                    }
                    mbar_expect_tx(&pfull[b], g.patch_bytes);
                    tma_load_4d(patch + b * g.patch_stride, &tmX, g.x0, iy0, c0 + PP_CH * j, img, &pfull[b]);
                }
            }
            for (uint32_t b = 0; b < 2 && b < gj; ++b) {
                const uint32_t last = b + 2 * ((gj - 1 - b) / 2);
                mbar_wait(&pfull[b], (last >> 1) & 1);
            }
        }
    } else if (warp >= WORK_WARP0) {
        const int ww = warp - WORK_WARP0;
        const int quarter = warp & 3;
        const int col0 = (ww >> 2) * HB;
        const uint32_t conv_leader0 = map_to(smem_u32(&conv[0]), 0);
        const uint32_t chunk_empty_leader = map_to(smem_u32(chunk_empty), 0);
        // B build: lane = pixel, thread = 4 consecutive taps, i.e. one 16-byte
        // row segment of the K-major tile with the 64-byte swizzle (as the TMA
        // writes A): pixel r, taps 4g..4g+3 at byte 64 r + 16 (g ^ ((r/2)%4)).
        // Warp ww writes tap group g = ww%4 of pixels HB/2 (ww/4) + [0, HB/2):
        // lanes 0..31, then lanes 0..HB/2-33.  Each quarter-warp store covers 32
        // distinct banks; the patch reads of a warp are consecutive pixels.
        // Rows of pixels past the image read the last pixel (their outputs are
        // never stored) and taps past the group read whatever the patch holds
        // there (their weights are zero).  Neither reaches a stored result:
        // an inf or NaN anywhere in a product makes the accumulated output
        // nonfinite (the lo part of an inf is NaN, and 0 * inf is NaN), and
        // an output row segment with a nonfinite value is recomputed with f32
        // FMA in tap order, as the SIMT implicit GEMM computes it.
        const int kg = ww & 3;
        const int r0 = (HB / 2) * (ww >> 2) + lane, r1 = r0 + 32;
        const bool two = lane < HB / 2 - 32;
        const uint32_t bo0 = (uint32_t)r0 * 64 + ((uint32_t)(kg ^ ((r0 >> 1) & 3)) << 4);
        const uint32_t bo1 = (uint32_t)r1 * 64 + ((uint32_t)(kg ^ ((r1 >> 1) & 3)) << 4);
        const uint32_t smem_s = smem_u32(smem), patch_s = smem_u32(patch), tap_s = smem_u32(tap_off);
        const int ih = (int)p.ih, iw = (int)p.iw;
        const bool vec_ok = (p.hw % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.y) & 15) == 0);
        uint32_t gkt = 0, gj = 0, gc = 0;
        for (int t = pair0; t < ntiles && !s_fail; t += npairs) {
            int m0, img, p0, q0;
            tile_of(t, m0, img, p0, q0);
            const int oy_a = min(q0, hw - 1) / ow;
            auto pix_of = [&](int r) {
                const int q = min(q0 + r, hw - 1);
                const int oy = q / ow, ox = q % ow;
                return (oy - oy_a) * p.sy * g.pitch + (ox * p.sx - p.px - g.x0);
            };
            // lanes without a second pixel read their first one again (stores skipped)
            const int pix0 = pix_of(r0), pix1 = two ? pix_of(r1) : pix0;
            float sum[HB];
#pragma unroll
            for (int j = 0; j < HB; ++j) sum[j] = 0.0f;
            int kin_p = 0;          // k-tile within the current patch chunk
            bool done = false;      // the tile's accumulators are in sum[]
            for (int kt = 0; kt < ktiles; ++kt, ++gkt) {
                const uint32_t s = gkt % NST;
                if (gkt >= NST && (s_fail || !mbar_wait(&empty[s], ((gkt / NST) - 1) & 1))) {
                    s_fail = 1;
                    break;
                }
                if (kin_p == 0 && (s_fail || !mbar_wait(&pfull[gj & 1], (gj >> 1) & 1))) {
                    s_fail = 1;
                    break;
                }
                // shared addresses in bytes; all eight loads go out before any store
                const uint32_t pt = patch_s + (gj & 1) * g.patch_stride;
                const int4 t4 = lds_v4_s32(tap_s + (uint32_t)(kin_p * 4 + kg) * 16);
                const uint32_t bt = smem_s + s * STAGE_BYTES + 2 * A_TILE;
                float v[8];
                v[0] = lds_f32(pt + 4u * (uint32_t)(t4.x + pix0));
                v[1] = lds_f32(pt + 4u * (uint32_t)(t4.y + pix0));
                v[2] = lds_f32(pt + 4u * (uint32_t)(t4.z + pix0));
                v[3] = lds_f32(pt + 4u * (uint32_t)(t4.w + pix0));
                v[4] = lds_f32(pt + 4u * (uint32_t)(t4.x + pix1));
                v[5] = lds_f32(pt + 4u * (uint32_t)(t4.y + pix1));
                v[6] = lds_f32(pt + 4u * (uint32_t)(t4.z + pix1));
                v[7] = lds_f32(pt + 4u * (uint32_t)(t4.w + pix1));
                sts_v4_f32(bt + bo0, v[0], v[1], v[2], v[3]);
                sts_v4_f32(bt + B_TILE + bo0, v[0] - tf32_trunc(v[0]), v[1] - tf32_trunc(v[1]),
                           v[2] - tf32_trunc(v[2]), v[3] - tf32_trunc(v[3]));
                if (two) {
                    sts_v4_f32(bt + bo1, v[4], v[5], v[6], v[7]);
                    sts_v4_f32(bt + B_TILE + bo1, v[4] - tf32_trunc(v[4]), v[5] - tf32_trunc(v[5]),
                               v[6] - tf32_trunc(v[6]), v[7] - tf32_trunc(v[7]));
                }
                __syncwarp();
                const bool chunk_end = kin_p == khw - 1 || kt == ktiles - 1;
                if (lane == 0 && chunk_end) mbar_arrive(&pempty[gj & 1]);
                if (s_fail || !mbar_wait(&full[s], (gkt / NST) & 1)) {
                    s_fail = 1;
                    break;
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(conv_leader0 + s * 8);
                if (chunk_end) {
                    kin_p = 0;
                    ++gj;
                } else {
                    ++kin_p;
                }
                if (kt % KC == KC - 1 || kt == ktiles - 1) {
                    if (!mbar_wait(chunk_full, gc & 1)) {
                        s_fail = 1;
                        break;
                    }
                    tc_fence_after();
                    if (s_fail) break;
                    tmem_accumulate(tmem, quarter, col0, sum);
                    if (kt == ktiles - 1) {
                        // the cross terms too, before the MMAs of the next tile overwrite them
                        tmem_accumulate(tmem + XCOL, quarter, col0, sum);
                        done = true;
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(chunk_empty_leader);
                    ++gc;
                }
            }
            if (!done) break;
            // store this thread's output row segment (channel co, pixels p0 + col0 + [0, 112))
            const int co = m0 + quarter * 32 + lane;
            const int64_t co_abs = (int64_t)grp * p.cog + co;
            float *yrow = p.y + ((int64_t)img * p.co_total + co_abs) * p.hw;
            float probe = 0.0f;     // NaN iff some sum is inf or NaN
#pragma unroll
            for (int jj = 0; jj < HB; ++jj) probe = fmaf(sum[jj], 0.0f, probe);
            if (probe != probe) {
                const float *wrow = p.w + co_abs * p.ws0;
                const float *ximg = p.x + (int64_t)img * p.xs[0] + (int64_t)grp * p.cg * p.xs[1];
                for (int jj = 0; jj < HB; ++jj) {
                    const int q = p0 + col0 + jj;
                    if (q >= hw) break;
                    const int y0 = (q / ow) * p.sy - p.py, x0 = (q % ow) * p.sx - p.px;
                    float acc = 0.0f;
                    for (int k = 0; k < p.kk; ++k) {
                        const int ci = k / khw, r = k % khw;
                        const int iy = y0 + (r / p.kw) * p.dy, ix = x0 + (r % p.kw) * p.dx;
                        const float xv = (iy >= 0 && iy < ih && ix >= 0 && ix < iw)
                                             ? ximg[(int64_t)ci * p.xs[1] + (int64_t)iy * p.xs[2] + (int64_t)ix * p.xs[3]]
                                             : 0.0f;
                        acc = fmaf(wrow[k], xv, acc);
                    }
                    yrow[q] = acc;
                }
            } else {
#pragma unroll
                for (int c = 0; c < HB / 16; ++c) {
                    const int q = p0 + col0 + c * 16;
                    if (vec_ok && q + 16 <= hw) {
#pragma unroll
                        for (int jj = 0; jj < 16; jj += 4)
                            *reinterpret_cast<float4 *>(yrow + q + jj) =
                                make_float4(sum[c * 16 + jj], sum[c * 16 + jj + 1], sum[c * 16 + jj + 2],
                                            sum[c * 16 + jj + 3]);
                    } else {
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj)
                            if (q + jj < hw) yrow[q + jj] = sum[c * 16 + jj];
                    }
                }
            }
        }
    }
    tc_fence_before();
    cluster_sync_any();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
    if (threadIdx.x == 0 && s_fail) atomicOr(p.status, KX_TIMEOUT_FLAG);
}

// Weights [co][cg][kh][kw] under any strides -> dense rows of `pitch` floats
// in the reference's tap order (ci, ky, kx), zero beyond the taps: the layout
// the weight tensor map reads (16-byte aligned rows).
__global__ void pack_weights_kernel(const float *__restrict__ w, int64_t ws0, int64_t ws1, int64_t ws2, int64_t ws3,
                                    int64_t co, int kh, int kw, int kk, int pitch, float *__restrict__ out) {
    const int64_t total = co * pitch;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = e / pitch;
        const int k = (int)(e % pitch);
        float v = 0.0f;
        if (k < kk) {
            const int khw = kh * kw;
            const int ci = k / khw, r = k % khw;
            v = w[o * ws0 + ci * ws1 + (r / kw) * ws2 + (r % kw) * ws3];
        }
        out[e] = v;
    }
}

// The patch-staged kernel's weights: dense hi rows (when `hi` is given; the
// caller's rows are used in place otherwise) and their lo parts w - tf32(w),
// `pitch` floats per output channel in tap order, zero beyond the taps (the
// lo part of an infinite weight is NaN, which the kernel's epilogue catches).
__global__ void split_weights_kernel(const float *__restrict__ w, int64_t ws0, int64_t ws1, int64_t ws2, int64_t ws3,
                                     int64_t co, int kh, int kw, int kk, int pitch, float *__restrict__ hi,
                                     float *__restrict__ lo) {
    const int64_t total = co * pitch;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = e / pitch;
        const int k = (int)(e % pitch);
        float v = 0.0f;
        if (k < kk) {
            const int khw = kh * kw;
            const int ci = k / khw, r = k % khw;
            v = w[o * ws0 + ci * ws1 + (r / kw) * ws2 + (r % kw) * ws3];
        }
        if (hi) hi[e] = v;
        lo[e] = v - tf32_trunc(v);
    }
}

}  // namespace conv
}  // namespace tc

// The tensor-core conv reads each group's weights as dense [cog, cg*kh*kw]
// rows with 16-byte aligned pitch (repacked into the handle's workspace when
// the caller's layout is not that), at least one k-tile, a tap table that fits
// in shared memory beside the stages, and geometry whose pixel and tap
// coordinates fit int32.
int run_conv_tc(Handle *h, const float *x, const int64_t *xs, const float *w, const int64_t *ws, float *y,
                int64_t n, int64_t c, int64_t ih, int64_t iw, int64_t co, int64_t cg, int64_t kh, int64_t kw,
                int64_t oh, int64_t ow, int64_t groups, int64_t sy, int64_t sx, int64_t py, int64_t px, int64_t dy,
                int64_t dx, const char **kernel_name) {
    using namespace tc;
    using namespace tc::conv;
    (void)c;
    const int64_t kk = cg * kh * kw;
    const int64_t cog = co / groups;
    if (kk < 16 || groups > 65535) return KX_DECLINED;
    const bool taps_dense = (kw == 1 || ws[3] == 1) && (kh == 1 || ws[2] == kw) && (cg == 1 || ws[1] == kh * kw);
    // dense, 16-byte aligned tap rows are read in place; anything else is repacked
    const bool repack = !taps_dense || ws[0] < kk || (ws[0] * 4) % 16 || (reinterpret_cast<uintptr_t>(w) & 15);
    const int64_t ncols = n * oh * ow;
    Params p;
    auto fill = [&](const float *wp, int64_t pitch) {
        std::memset(&p, 0, sizeof(p));
        p.x = x;
        p.w = wp;
        p.y = y;
        for (int i = 0; i < 4; ++i) p.xs[i] = xs[i];
        p.ws0 = pitch;
        p.ih = ih;
        p.iw = iw;
        p.oh = oh;
        p.ow = ow;
        p.hw = oh * ow;
        p.co_total = co;
        p.cog = cog;
        p.cg = cg;
        p.kh = (int)kh;
        p.kw = (int)kw;
        p.sy = (int)sy;
        p.sx = (int)sx;
        p.py = (int)py;
        p.px = (int)px;
        p.dy = (int)dy;
        p.dx = (int)dx;
        p.kk = (int)kk;
        p.ncols = ncols;
        p.status = h->flags + kStatusWord;
    };
    // Patch-staged CTA pairs (256 channels x 224 pixels of one image) when
    // TMA can box the input rows: unit column stride, 16-byte row, channel and
    // image strides, a patch row of at most 256 floats, both chunk buffers
    // beside the stages in shared memory.
    // Size-1 dimensions arrive with stride 0; the map gets any 16-byte
    // multiple there (only coordinate 0 is read).
    int64_t ts[3] = {xs[2], xs[1], xs[0]};   // row, channel, image strides
    if (ih <= 1 && ts[0] == 0) ts[0] = (iw + 3) / 4 * 4;
    if (c <= 1 && ts[1] == 0) ts[1] = ts[0] * ih;
    if (n <= 1 && ts[2] == 0) ts[2] = ts[1] * c;
    if (cog % 256 == 0 && (xs[3] == 1 || iw == 1) && ts[0] > 0 && ts[1] > 0 && ts[2] > 0 && (ts[0] * 4) % 16 == 0 &&
        (ts[1] * 4) % 16 == 0 && (ts[2] * 4) % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
        n * oh * ow < (1LL << 31) && oh * ow < (1LL << 30)) {
        const int64_t hw = oh * ow;
        const int64_t x0 = -((px + 3) / 4) * 4;
        const int64_t xmax = (ow - 1) * sx - px + (kw - 1) * dx;
        const int64_t pitch = (xmax - x0 + 1 + 3) / 4 * 4;
        // patch geometry for halves of hb pixels: rows under the widest half
        auto patch_for = [&](int64_t hb, int64_t &prows, int64_t &patch_bytes, int64_t &patch_stride) {
            int64_t span = 0;
            for (int64_t q0 = 0; q0 < hw; q0 += hb) {
                const int64_t qb = std::min(q0 + hb, hw) - 1;
                span = std::max(span, qb / ow - q0 / ow);
            }
            prows = span * sy + (kh - 1) * dy + 1;
            patch_bytes = (int64_t)PP_CH * prows * pitch * 4;
            patch_stride = (patch_bytes + 1023) / 1024 * 1024;
            return 2 * patch_stride + BAR_BYTES + PP_CH * kh * kw * 4 + 1024;
        };
        // 112-pixel halves: 128 (N = 256 per pair) measured slower on c4
        // (149.0 vs 145.3 TFLOP/s: register spills and taller patches)
        constexpr int hb = PP_HB;
        int64_t prows, patch_bytes, patch_stride;
        const int64_t smem_fixed = patch_for(hb, prows, patch_bytes, patch_stride);
        const int64_t stage_bytes = PatchTile<hb>::STAGE;
        const int64_t tpi = (hw + 2 * hb - 1) / (2 * hb);
        // as many stages as fit (up to PP_NST): the weight tile of k-tile kt is
        // fetched when the MMAs of kt - nst have freed its stage
        int nst = PP_NST;
        while (nst > 3 && smem_fixed + (int64_t)nst * stage_bytes > SMEM_LIMIT) --nst;
        const int64_t smem = smem_fixed + (int64_t)nst * stage_bytes;
        const int64_t pairs = (cog / 256) * n * tpi * groups;
        CUtensorMap mx;
        const uint64_t dims[4] = {(uint64_t)iw, (uint64_t)ih, (uint64_t)c, (uint64_t)n};
        const uint64_t strides[3] = {(uint64_t)ts[0] * 4, (uint64_t)ts[1] * 4, (uint64_t)ts[2] * 4};
        const uint32_t box[4] = {(uint32_t)pitch, (uint32_t)prows, (uint32_t)PP_CH, 1};
        if (pitch <= 256 && prows <= 256 && smem <= SMEM_LIMIT && 2 * pairs <= INT32_MAX &&
            (2 * pairs >= h->sm_count || h->f32_variant == KX_F32_3XTF32) && make_map4(&mx, x, dims, strides, box)) {
            // The weights' lo parts (and the dense hi rows when the caller's
            // layout is not) go to the workspace once per call; the kernel
            // loads both by TMA.
            const int64_t wp = repack ? (kk + 3) / 4 * 4 : ws[0];
            const uint64_t part = (uint64_t)co * wp * sizeof(float);
            void *buf = nullptr;
            int rc = h->workspace((repack ? 2 : 1) * part, &buf);
            if (rc) return rc;
            float *hi = repack ? static_cast<float *>(buf) : nullptr;
            float *lo = static_cast<float *>(buf) + (repack ? co * wp : 0);
            const float *whi = repack ? hi : w;
            int64_t blocks = (co * wp + 255) / 256;
            if (blocks > 4LL * h->sm_count) blocks = 4LL * h->sm_count;
            split_weights_kernel<<<(unsigned)blocks, 256, 0, h->stream>>>(w, ws[0], ws[1], ws[2], ws[3], co, (int)kh,
                                                                           (int)kw, (int)kk, (int)wp, hi, lo);
            ++h->launches;
            cudaError_t ce = cudaGetLastError();
            if (ce != cudaSuccess) return h->cuda_fail(ce);
            CUtensorMap mw, mwlo;
            if (!make_map(&mw, whi, (uint64_t)kk, (uint64_t)cog, (uint64_t)groups, (uint64_t)wp * 4,
                          (uint64_t)(wp * cog) * 4, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B) ||
                !make_map(&mwlo, lo, (uint64_t)kk, (uint64_t)cog, (uint64_t)groups, (uint64_t)wp * 4,
                          (uint64_t)(wp * cog) * 4, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B))
                return KX_DECLINED;
            fill(whi, wp);
            PatchGeom g;
            g.x0 = (int)x0;
            g.pitch = (int)pitch;
            g.prows = (int)prows;
            g.tpi = (int)tpi;
            g.nimg = (int)n;
            g.patch_bytes = (uint32_t)patch_bytes;
            g.patch_stride = (uint32_t)patch_stride;
            auto k = nst == 6 ? conv_3xtf32_patch_kernel<6, hb>
                     : nst == 5 ? conv_3xtf32_patch_kernel<5, hb>
                     : nst == 4 ? conv_3xtf32_patch_kernel<4, hb>
                                : conv_3xtf32_patch_kernel<3, hb>;
            ce = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (ce == cudaSuccess) {
                cudaLaunchConfig_t cfg = {};
                // persistent: one pair per two SMs in all, each group's pairs walking its tiles
                const int64_t per_group = pairs / groups;
                const int64_t launch = std::min(per_group, std::max<int64_t>(1, h->sm_count / 2 / groups));
                cfg.gridDim = dim3((unsigned)(2 * launch), (unsigned)groups, 1);
                cfg.blockDim = dim3(NTHREADS, 1, 1);
                cfg.dynamicSmemBytes = (size_t)smem;
                cfg.stream = h->stream;
                cudaLaunchAttribute attr[1];
                attr[0].id = cudaLaunchAttributeClusterDimension;
                attr[0].val.clusterDim.x = 2;
                attr[0].val.clusterDim.y = 1;
                attr[0].val.clusterDim.z = 1;
                cfg.attrs = attr;
                cfg.numAttrs = 1;
                ce = cudaLaunchKernelEx(&cfg, k, mw, mwlo, mx, p, g);
                if (ce == cudaSuccess) ce = cudaGetLastError();
            }
            *kernel_name = "conv_tc_3xtf32_patch_256x224";
            ++h->launches;
            return ce == cudaSuccess ? KX_OK : h->cuda_fail(ce);
        }
    }
    // the gathered kernels keep a (ci, ky, kx) table of all taps in shared memory
    if (kh * kw > PAD_TAP || (kk + BK) * (int64_t)sizeof(Tap) + Tile<128>::FIXED_SMEM > SMEM_LIMIT)
        return KX_DECLINED;
    int64_t w_pitch = ws[0];
    if (repack) {
        // repack into dense, 16-byte aligned tap rows in the handle's workspace
        const int pitch = (int)((kk + 3) / 4 * 4);
        void *buf = nullptr;
        int rc = h->workspace((uint64_t)co * pitch * sizeof(float), &buf);
        if (rc) return rc;
        int64_t blocks = (co * pitch + 255) / 256;
        if (blocks > 4LL * h->sm_count) blocks = 4LL * h->sm_count;
        pack_weights_kernel<<<(unsigned)blocks, 256, 0, h->stream>>>(w, ws[0], ws[1], ws[2], ws[3], co, (int)kh,
                                                                      (int)kw, (int)kk, pitch,
                                                                      static_cast<float *>(buf));
        ++h->launches;
        cudaError_t ce = cudaGetLastError();
        if (ce != cudaSuccess) return h->cuda_fail(ce);
        w = static_cast<const float *>(buf);
        w_pitch = pitch;
    }
    if (((cog + BM - 1) / BM) * ((ncols + 127) / 128) > INT32_MAX) return KX_DECLINED;
    CUtensorMap mw;
    if (!make_map(&mw, w, (uint64_t)kk, (uint64_t)cog, (uint64_t)groups, (uint64_t)w_pitch * 4,
                  (uint64_t)(w_pitch * cog) * 4, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B))
        return KX_DECLINED;
    fill(w, w_pitch);
    const int table_pair = (int)((kk + BK - 1) / BK * BK) * (int)sizeof(Tap);
    // CTA pairs (256 channels x 256 pixels) when the group has 256+ output
    // channels and the pairs fill the SMs (a 256-wide one-SM conv tile
    // gathers every input element once per 128 channels; a pair once per 256)
    {
        const int64_t pm = cog / 256;   // whole channel pairs only
        const int64_t pair_ctas = 2 * pm * ((ncols + 255) / 256) * groups;
        if (pm >= 1 && cog % 256 == 0 && (pair_ctas >= 4LL * h->sm_count || h->f32_variant == KX_F32_3XTF32) &&
            PAIR_FIXED_SMEM + table_pair <= SMEM_LIMIT) {
            const int smem = PAIR_FIXED_SMEM + table_pair;
            auto k = conv_3xtf32_pair_kernel;
            cudaError_t ce = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (ce == cudaSuccess) {
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3((unsigned)pair_ctas / (unsigned)groups, (unsigned)groups, 1);
                cfg.blockDim = dim3(NTHREADS, 1, 1);
                cfg.dynamicSmemBytes = smem;
                cfg.stream = h->stream;
                cudaLaunchAttribute attr[1];
                attr[0].id = cudaLaunchAttributeClusterDimension;
                attr[0].val.clusterDim.x = 2;
                attr[0].val.clusterDim.y = 1;
                attr[0].val.clusterDim.z = 1;
                cfg.attrs = attr;
                cfg.numAttrs = 1;
                ce = cudaLaunchKernelEx(&cfg, k, mw, p);
                if (ce == cudaSuccess) ce = cudaGetLastError();
            }
            *kernel_name = "conv_tc_3xtf32_pair_256x256";
            ++h->launches;
            return ce == cudaSuccess ? KX_OK : h->cuda_fail(ce);
        }
    }
    // tile width from the wave model (as the GEMM's), within shared memory
    const int64_t tm = (cog + BM - 1) / BM;
    auto cost = [&](int bn) {
        const int64_t t = tm * ((ncols + bn - 1) / bn) * groups;
        return ((t + h->sm_count - 1) / h->sm_count) * (int64_t)(bn + 32);
    };
    const int table = (int)((kk + BK - 1) / BK * BK) * (int)sizeof(Tap);
    int bn = (cost(256) <= cost(128) && Tile<256>::FIXED_SMEM + table <= SMEM_LIMIT) ? 256 : 128;
    if (Tile<128>::FIXED_SMEM + table > SMEM_LIMIT) return KX_DECLINED;
    const int smem = (bn == 256 ? Tile<256>::FIXED_SMEM : Tile<128>::FIXED_SMEM) + table;
    auto k = bn == 256 ? conv_3xtf32_kernel<256> : conv_3xtf32_kernel<128>;
    cudaError_t ce = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (ce == cudaSuccess) {
        const int64_t tiles_bn = tm * ((ncols + bn - 1) / bn);
        dim3 grid((unsigned)tiles_bn, (unsigned)groups, 1);
        k<<<grid, NTHREADS, smem, h->stream>>>(mw, p);
        ce = cudaGetLastError();
    }
    *kernel_name = bn == 256 ? "conv_tc_3xtf32_128x256" : "conv_tc_3xtf32_128x128";
    ++h->launches;
    return ce == cudaSuccess ? KX_OK : h->cuda_fail(ce);
}

}  // namespace kx
