// Fused attention products: out = softmax_temperature(q . kt, -1, T) . v in one
// persistent tcgen05 kernel, without writing the scores or the probabilities.
//
// Kernix composes attention from three calls -- matmul (ops/linalg.rs:68-214),
// softmax_temperature (ops/math_extra.rs:394-401,425-500,544-557) and matmul
// again -- and materialises S = q kt and P = softmax(S) in full.  On the GPU
// that costs two round trips of the [.., sq, sk] scores through HBM (8.6 GB
// each for 16 x 32 heads of 2048 x 2048).  Here each CTA keeps a 128-row block
// of q on chip and walks the keys in blocks of 64:
//
//   S_j  = q . kt_j                 split-TF32 on the tensor cores (TMEM)
//   m    = max(m, rowmax S_j)       online maximum (Milakov & Gimelshein 2018)
//   P_j  = exp((S_j - m) / T)       written back into TMEM as the A operand
//   O_j  = P_j . v_j                split-TF32, A from TMEM, fresh accumulator
//   O    = O * exp((m_old - m)/T) + O_j    in registers (round-to-nearest)
//   l    = l * exp((m_old - m)/T) + sum P_j
// and stores out = O / l once per row block.  The result equals the composed
// path's up to rounding: exp((x - max)/T) / sum with the final maximum, summed
// against v (the tests bound the difference against the compensated oracle).
// Anything the composition would treat specially -- an inf/NaN score (the
// reference's NonFiniteInput with its first index), an overflowing x - max
// (its divide-first branch), an inf/NaN in v (IEEE propagation through the
// product) -- sets a flag; the host then runs the composed path, which
// reproduces the reference's result or error exactly.
//
// Split-TF32: x = hi + lo with hi = tf32(x) (the raw f32 tile, which the tensor
// core reads truncated) and lo = x - hi; a.b = hi.hi + hi.lo + lo.hi.  The
// score accumulators keep hi.hi and the cross terms apart (K = head dim <= 128
// per block); each key block's O_j holds all three products over 64 keys and
// is folded into f32 registers right away, so the tensor core's truncating
// accumulation never runs over more than 64 keys.
//
// Roles (384 threads, one CTA per SM, persistent over (batch, row block) units):
//   warp 0       TMA producer: q block, then per key block 4 kt slots and
//                4 v slots through a ring of 16 KB slots
//   warp 1       TMEM owner (512 columns) and MMA issuer
//   warps 2..9   rows: two threads per row (TMEM lane), each with half of the
//                scores (S_j -> P_j, m, l) and half of O in registers (the
//                fold of block j - 1 right after the softmax of block j);
//                epilogue stores
//   warps 10,11  split: lo parts of q, kt and v (v checked for inf/NaN)
// Two threads per row and two row warps per SM sub-partition keep the
// softmax (one exponential per score) off the critical path: with one warp
// per sub-partition doing whole rows it paced the tensor cores.
// TMEM: S buffer b (b = key block % 2) at columns [128 b, 128 b + 128): hi.hi
// scores in the first 64, cross terms in the next 64, overwritten in place by
// P_hi and P_lo; O buffer b at [256 + 128 b, 256 + 128 b + 128).
// Every mbarrier wait is bounded (2 s); on expiry the kernel stops its loops,
// waits for its own TMA copies, frees TMEM and sets the handle's status bit.
// With at least 74 units of 256 query rows the same kernel runs on CTA pairs
// (template PAIR, described at the kernel): the leader issues cta_group::2
// MMAs for both CTAs' rows and each CTA stages half of every key and value
// block; otherwise one CTA per SM as above.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "tc_common.cuh"

extern "C" int kx_matmul_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out,
                             kx_error *err);
extern "C" int kx_softmax_temperature_f32(kx_handle *h, const kx_tensor *src, int64_t axis, float temperature,
                                          const kx_tensor *out, kx_error *err);

namespace kx {

namespace tc {
namespace attn {

constexpr int BQ = 128;            // query rows per unit
constexpr int BKEY = 64;           // keys per block
constexpr int DH = 128;            // head dimension (q, kt rows, v columns)
constexpr int NSLOT = 5;           // ring slots
constexpr int SLOT = 16384;        // hi (8 KB) + lo (8 KB)
constexpr int Q_BYTES = BQ * DH * 4;          // 64 KB (hi); lo follows
constexpr int RING_OFF = 2 * Q_BYTES;         // 128 KB
constexpr int MISC_OFF = RING_OFF + NSLOT * SLOT;   // 208 KB
// misc: mbarriers (512 B), the row-maximum exchange [2][2][128] f32 (2 KB)
// and the row-sum exchange [2][128] f32 (1 KB)
constexpr int MISC_BYTES = 512 + 3 * 2 * BQ * 4;
constexpr int SMEM_BYTES = MISC_OFF + MISC_BYTES + 1024;
constexpr int ROW_WARP0 = 2, SPLIT_WARP0 = 10, SPLIT_WARPS = 2;
constexpr int NT = (SPLIT_WARP0 + SPLIT_WARPS) * 32;   // 384
constexpr int SPLIT_THREADS = SPLIT_WARPS * 32;
static_assert(SMEM_BYTES <= 232448, "shared memory");

struct Params {
    float *out;
    int64_t o_rs, o_bs;          // out row and batch strides (elements)
    int sq, sk, nbatch;
    int nq;                      // row blocks per batch entry
    int64_t units;               // nbatch * nq
    int nkb;                     // key blocks
    float c, c_lo;               // log2(e)/T rounded to f32, and its rounding error
    uint32_t *status;            // bit 0: a bounded wait expired
    uint32_t *flag;              // nonzero: run the composed path
};

// exp(x / T) for x = s - max <= 0 as 2^t with t = x * log2(e) / T: c =
// log2(e)/T rounded to f32 and c_lo its rounding error (both from the host in
// double precision), t = x c rounded, tl = the exact residual of x c (one FMA)
// plus x c_lo, then 2^t by the special-function unit (ex2.approx, a few ulp)
// and the first-order correction 2^(t + tl) = 2^t (1 + tl ln 2).  About 3 ulp
// from exp(x / T) in all, the order of the reference's own rounding of
// (x - max) / T before its exp; below 2^-126 the result is flushed to zero.
__device__ __forceinline__ float exp_scaled(float x, float c, float c_lo) {
    const float t = x * c;
    const float tl = fmaf(x, c_lo, fmaf(x, c, -t));
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t));
    return fmaf(e * tl, 0.693147182f, e);
}

// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D (TMEM) += A (TMEM, 128 lanes x 8 tf32 columns) x B (shared memory).
__device__ __forceinline__ void mma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Bounded wait for waits off the critical path (the producer's, the fold's,
// the split's wait for a q block): a short sleep between polls leaves the
// issue slots of the SM sub-partition to the row warps that share it.  Same
// 2 s deadline as mbar_wait.
__device__ __forceinline__ bool mbar_wait_idle(uint64_t *bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    uint64_t deadline = 0;
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        const uint64_t now = globaltimer();
        if (deadline == 0) deadline = now + WAIT_NS;
        else if (now > deadline) return false;
        __nanosleep(200);
    }
}

// Split one buffer of `chunks` 16-byte chunks in place: lo (x - tf32(x)) at
// `lo_off` bytes past each raw chunk.
__device__ __forceinline__ void split_buf(uint32_t base, int chunks, uint32_t lo_off, int wt) {
#pragma unroll 4
    for (int c = wt; c < chunks; c += SPLIT_THREADS * 4) {
        float4 v[4];
        uint32_t at[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int cc = c + u * SPLIT_THREADS;
            at[u] = base + (uint32_t)cc * 16;
            if (cc < chunks) v[u] = lds_v4_f32(at[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int cc = c + u * SPLIT_THREADS;
            if (cc < chunks)
                sts_v4_f32(at[u] + lo_off, v[u].x - tf32_trunc(v[u].x), v[u].y - tf32_trunc(v[u].y),
                           v[u].z - tf32_trunc(v[u].z), v[u].w - tf32_trunc(v[u].w));
        }
    }
}

// lo parts of a [nb, rows, 128] operand (row stride rs, batch stride bs;
// 16-byte rows) into a dense [nb, rows, 128] array, before the fused kernel:
// its TMA then brings hi (the operand itself) and lo into each slot, and no
// warp of the fused kernel splits k or v.  With CHECK, an inf or NaN sets
// bit 1 of `flag` (v: the composed path propagates it through P v).
template <bool CHECK>
__global__ void __launch_bounds__(256) split_lo_kernel(const float *__restrict__ x, int64_t rs, int64_t bs,
                                                       float *__restrict__ lo, int64_t rows, int64_t nb,
                                                       uint32_t *flag) {
    const int64_t n4 = nb * rows * (DH / 4);
    uint32_t mag = 0;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n4; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t d4 = e % (DH / 4), rr = (e / (DH / 4)) % rows, b = e / (DH / 4) / rows;
        const float4 v = *reinterpret_cast<const float4 *>(x + b * bs + rr * rs + d4 * 4);
        if (CHECK)
            mag = max(mag, max(max(__float_as_uint(v.x) & 0x7fffffffu, __float_as_uint(v.y) & 0x7fffffffu),
                               max(__float_as_uint(v.z) & 0x7fffffffu, __float_as_uint(v.w) & 0x7fffffffu)));
        reinterpret_cast<float4 *>(lo)[e] =
            make_float4(v.x - tf32_trunc(v.x), v.y - tf32_trunc(v.y), v.z - tf32_trunc(v.z), v.w - tf32_trunc(v.w));
    }
    if (CHECK && __any_sync(0xffffffffu, mag >= 0x7f800000u) && (threadIdx.x & 31) == 0) atomicOr(flag, 2u);
}

// Slot stream of one unit, in the order the MMA thread consumes it:
// kt_0, kt_1, v_0, kt_2, v_1, ..., kt_{n-1}, v_{n-2}, v_{n-1}; each kt_j and
// v_j is SPB slots (4 on one SM; 2 in each CTA of a pair, which stages half
// of every block).  Slot item e (0-based) of a unit -> (is_v, block, part).
template <int SPB>
__device__ __forceinline__ void slot_item(int e, int nkb, bool &is_v, int &blk, int &part) {
    part = e % SPB;
    const int grp = e / SPB;  // 0: kt_0; then pairs (kt_j, v_{j-1}); last: v_{n-1}
    if (grp == 0) {
        is_v = false;
        blk = 0;
    } else if (grp >= 2 * nkb - 1) {
        is_v = true;
        blk = nkb - 1;
    } else {
        const int j = (grp + 1) >> 1;
        is_v = (grp & 1) == 0;
        blk = is_v ? j - 1 : j;
    }
}

// D (TMEM of both CTAs) += A (TMEM of both CTAs, 128 lanes x 8 tf32 columns
// each) x B (shared memory: each CTA's half of the columns), for a pair.
__device__ __forceinline__ void mma_pair_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Registers are split evenly over the SM's four sub-partitions (16,384
// each); twelve warps put three on each, so a thread may use up to 168.
//
// PAIR: a cluster of two CTAs takes 256 query rows, 128 in each CTA, and the
// leader (cluster rank 0) issues tcgen05.mma.cta_group::2 for both: scores
// with M = 256, N = 64 (each CTA stages 32 of the block's keys) and P.v with
// M = 256, N = 128 (each CTA stages 64 of v's columns, P comes from each CTA's
// own TMEM).  Per SM that halves the key and value bytes loaded and the
// operand bytes the tensor core reads per MMA falls from 6 KB to 5 KB.  Each
// CTA's TMA completes on its own slot barrier; in the second CTA the otherwise
// idle warp 1 relays every filled slot to the leader with a remote arrive; the
// row warps' and split warps' arrivals go to the leader's barriers, and the
// leader commits every MMA completion to the barriers of both CTAs.  The
// softmax, the fold and the epilogue are each CTA's own, as on one SM.
template <bool PAIR>
__global__ void __launch_bounds__(NT, 1)
attn_3xtf32_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKl,
                   const __grid_constant__ CUtensorMap tmVl, const __grid_constant__ Params p) {
    constexpr int SPB = PAIR ? 2 : 4;           // slots per key block and operand
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem + RING_OFF;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + MISC_OFF);
    uint64_t *slot_full = bars;                 // [NSLOT]
    uint64_t *slot_empty = slot_full + NSLOT;   // [NSLOT]
    uint64_t *q_full = slot_empty + NSLOT;
    uint64_t *q_conv = q_full + 1;
    uint64_t *q_empty = q_conv + 1;
    uint64_t *s_full = q_empty + 1;             // [2]
    uint64_t *p_ready = s_full + 2;             // [2]
    uint64_t *o_full = p_ready + 2;             // [2]
    uint64_t *o_empty = o_full + 2;             // [2]
    uint64_t *xbar = o_empty + 2;               // [4] row-maximum exchange per lane quarter
    uint64_t *lbar = xbar + 4;                  // [4] row-sum exchange per lane quarter
    uint64_t *peer_full = lbar + 4;             // [NSLOT] pair leader: the second CTA's slot is full
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(peer_full + NSLOT);
    float *xmax = reinterpret_cast<float *>(smem + MISC_OFF + 512);   // [2][2][BQ]
    float *lsum = xmax + 4 * BQ;                                      // [2][BQ]
    __shared__ int s_fail_storage;
    volatile int &s_fail = s_fail_storage;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_rank() : 0u;
    const bool leader = rank == 0;
    const int64_t unit0 = PAIR ? blockIdx.x / 2 : blockIdx.x;        // this CTA's (pair's) first unit
    const int64_t ustride = PAIR ? gridDim.x / 2 : gridDim.x;
    const int64_t my_units = p.units > unit0 ? (p.units - unit0 + ustride - 1) / ustride : 0;
    const int nkb = p.nkb;
    const int items = 2 * SPB * nkb;  // slot items per unit
    // arrivals that the leader's MMA thread waits for
    auto arrive_leader = [&](uint64_t *bar) {
        if constexpr (PAIR) mbar_arrive_cluster(map_to(smem_u32(bar), 0));
        else mbar_arrive(bar);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < NSLOT; ++s) {
            mbar_init(&slot_full[s], 1);
            mbar_init(&slot_empty[s], 1);
            mbar_init(&peer_full[s], 1);
        }
        mbar_init(q_full, 1);
        mbar_init(q_conv, PAIR ? 2 * SPLIT_WARPS : SPLIT_WARPS);
        mbar_init(q_empty, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_ready[b], PAIR ? 16 : 8);
            mbar_init(&o_full[b], 1);
            mbar_init(&o_empty[b], PAIR ? 16 : 8);
        }
        for (int r = 0; r < 4; ++r) {
            mbar_init(&xbar[r], 2);
            mbar_init(&lbar[r], 2);
        }
        s_fail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                         ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                         ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync_any();    // both CTAs' barriers initialised, TMEM allocated
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA producer ------------------------------------------------
        if (lane == 0) {
            int64_t g = 0;        // slot loads issued so far
            int64_t i = 0;
            for (; i < my_units && !s_fail; ++i) {
                const int64_t u = unit0 + i * ustride;
                const int bh = (int)(u / p.nq), q0 = (int)(u % p.nq) * (PAIR ? 2 * BQ : BQ) + (int)rank * BQ;
                if (i > 0 && !mbar_wait_idle(q_empty, (uint32_t)((i - 1) & 1))) {
                    s_fail = 1;
                    break;
                }
                mbar_expect_tx(q_full, Q_BYTES);
#pragma unroll 1
                for (int t = 0; t < DH / 16; ++t) tma_load_3d(smem + t * 8192, &tmQ, t * 16, q0, bh, q_full);
                for (int e = 0; e < items; ++e, ++g) {
                    const int s = (int)(g % NSLOT);
                    if (g >= NSLOT && !mbar_wait_idle(&slot_empty[s], (uint32_t)(((g / NSLOT) - 1) & 1))) {
                        s_fail = 1;
                        break;
                    }
                    bool is_v;
                    int blk, part;
                    slot_item<SPB>(e, nkb, is_v, blk, part);
                    uint8_t *dst = ring + s * SLOT;
                    mbar_expect_tx(&slot_full[s], SLOT);
                    if (PAIR && !is_v) {
                        // this CTA's 32 keys of kt_j x 64 head columns [64 part, +64): four
                        // 16-column boxes, hi then lo
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            tma_load_3d(dst + c * 2048, &tmK, part * 64 + c * 16, blk * BKEY + (int)rank * 32, bh,
                                        &slot_full[s]);
                            tma_load_3d(dst + SLOT / 2 + c * 2048, &tmKl, part * 64 + c * 16,
                                        blk * BKEY + (int)rank * 32, bh, &slot_full[s]);
                        }
                    } else if (PAIR) {
                        // keys [32 part, +32) of v_j x this CTA's 64 columns [64 rank, +64):
                        // per 16 keys two 32-column boxes, hi then lo
#pragma unroll
                        for (int kh = 0; kh < 2; ++kh)
#pragma unroll
                            for (int c = 0; c < 2; ++c) {
                                const int col = (int)rank * 64 + c * 32, key = blk * BKEY + part * 32 + kh * 16;
                                tma_load_3d(dst + kh * 4096 + c * 2048, &tmV, col, key, bh, &slot_full[s]);
                                tma_load_3d(dst + SLOT / 2 + kh * 4096 + c * 2048, &tmVl, col, key, bh,
                                            &slot_full[s]);
                            }
                    } else if (!is_v) {
                        // kt_j: 64 keys x 32 head columns as two 16-column boxes, hi then lo
                        tma_load_3d(dst, &tmK, part * 32, blk * BKEY, bh, &slot_full[s]);
                        tma_load_3d(dst + 4096, &tmK, part * 32 + 16, blk * BKEY, bh, &slot_full[s]);
                        tma_load_3d(dst + SLOT / 2, &tmKl, part * 32, blk * BKEY, bh, &slot_full[s]);
                        tma_load_3d(dst + SLOT / 2 + 4096, &tmKl, part * 32 + 16, blk * BKEY, bh, &slot_full[s]);
                    } else {
                        // v_j: 16 keys x 128 columns as four 32-column boxes, hi then lo
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            tma_load_3d(dst + c * 2048, &tmV, c * 32, blk * BKEY + part * 16, bh, &slot_full[s]);
                            tma_load_3d(dst + SLOT / 2 + c * 2048, &tmVl, c * 32, blk * BKEY + part * 16, bh,
                                        &slot_full[s]);
                        }
                    }
                }
            }
            // drain: the last copy issued into each slot, and the last q block, have landed
            for (int s = 0; s < NSLOT && s < g; ++s) {
                const int64_t last = s + NSLOT * ((g - 1 - s) / NSLOT);
                mbar_wait(&slot_full[s], (uint32_t)((last / NSLOT) & 1));
            }
            if (i > 0) mbar_wait(q_full, (uint32_t)((i - 1) & 1));
        }
    } else if (warp == 1 && PAIR && !leader) {
        // ---- relay (second CTA of a pair): each filled slot -> the leader --
        if (lane == 0) {
            const uint32_t pf0 = map_to(smem_u32(&peer_full[0]), 0);
            int64_t g = 0;
            for (int64_t i = 0; i < my_units && !s_fail; ++i) {
                for (int e = 0; e < items; ++e, ++g) {
                    const int s = (int)(g % NSLOT);
                    if (!mbar_wait(&slot_full[s], (uint32_t)((g / NSLOT) & 1))) {   // no sleep: on the MMA path
                        s_fail = 1;
                        break;
                    }
                    mbar_arrive_cluster(pf0 + (uint32_t)(s * 8));
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer (one SM, or the leader of a pair) -----------------
        if (lane == 0) {
            constexpr uint32_t idesc_s = PAIR ? idesc_pair(false, BKEY) : idesc_tf32<BKEY>(false);
            constexpr uint32_t idesc_o = PAIR ? idesc_pair(true, DH) : idesc_tf32<DH>(true);
            const uint64_t dq_hi = desc_k_sw64(smem_u32(smem)), dq_lo = desc_k_sw64(smem_u32(smem) + Q_BYTES);
            // the slot's data in this CTA and, for a pair, in the second CTA
            auto slot_ready = [&](int s, int64_t g) -> bool {
                if (!mbar_wait(&slot_full[s], (uint32_t)((g / NSLOT) & 1))) return false;
                if constexpr (PAIR)
                    if (!mbar_wait_cluster(&peer_full[s], (uint32_t)((g / NSLOT) & 1))) return false;
                return true;
            };
            // completion of the MMAs issued so far -> the barrier in every CTA that has it
            auto commit = [&](uint64_t *bar) {
                if constexpr (PAIR) {
                    commit_pair(smem_u32(bar));
                    commit_pair(map_to(smem_u32(bar), 1));
                } else {
                    mma_commit(bar);
                }
            };
            auto mma_s = [&](uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
                if constexpr (PAIR) mma_pair(d, a, b, idesc_s, acc);
                else mma_tf32(d, a, b, idesc_s, acc);
            };
            auto mma_o = [&](uint32_t d, uint32_t a, uint64_t b, uint32_t acc) {
                if constexpr (PAIR) mma_pair_ts(d, a, b, idesc_o, acc);
                else mma_tf32_ts(d, a, b, idesc_o, acc);
            };
            int64_t g = 0;        // slot items consumed
            int64_t kb = 0;       // key blocks started (global, for the TMEM buffers)
            for (int64_t i = 0; i < my_units && !s_fail; ++i) {
                const bool q_ready = PAIR ? mbar_wait_cluster(q_conv, (uint32_t)(i & 1))
                                          : mbar_wait(q_conv, (uint32_t)(i & 1));
                if (!q_ready) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                const int64_t kb0 = kb;
                // S_j for j = 0..nkb-1, PV_{j-1} after S_j, PV_{nkb-1} last
                for (int j = 0; j <= nkb && !s_fail; ++j) {
                    if (j < nkb) {
                        const int64_t gb = kb0 + j;
                        const uint32_t sm = tmem + (uint32_t)((gb & 1) * 128), sx = sm + 64;
#pragma unroll 1
                        for (int t = 0; t < SPB; ++t) {
                            const int s = (int)(g % NSLOT);
                            if (!slot_ready(s, g)) {
                                s_fail = 1;
                                break;
                            }
                            tc_fence_after();
                            // descriptors: base + (byte offset >> 4) in the address field.
                            // One SM: the slot holds head columns [32 t, +32) of all 64
                            // keys as two 16-column boxes of 4 KB; a pair CTA: columns
                            // [64 t, +64) of its 32 keys as four boxes of 2 KB.
                            const uint64_t dk = desc_k_sw64(smem_u32(ring + s * SLOT));
                            constexpr int BOXES = PAIR ? 4 : 2, BOX = PAIR ? 2048 : 4096;
#pragma unroll
                            for (int sub = 0; sub < BOXES; ++sub) {
#pragma unroll
                                for (int ks = 0; ks < 2; ++ks) {
                                    const uint32_t qo = (uint32_t)(((BOXES * t + sub) * 8192 + ks * 32) >> 4);
                                    const uint32_t ko = (uint32_t)((sub * BOX + ks * 32) >> 4);
                                    const uint32_t acc = (t > 0 || sub > 0 || ks > 0) ? 1u : 0u;
                                    mma_s(sm, dq_hi + qo, dk + ko, acc);
                                    mma_s(sx, dq_hi + qo, dk + ko + (SLOT / 2 >> 4), acc);
                                    mma_s(sx, dq_lo + qo, dk + ko, 1u);
                                }
                            }
                            commit(&slot_empty[s]);
                            ++g;
                        }
                        if (s_fail) break;
                        commit(&s_full[gb & 1]);
                        if (j == nkb - 1) commit(q_empty);   // q is read by no later MMA of this unit
                    }
                    if (j >= 1) {
                        const int64_t gb = kb0 + j - 1;
                        const int b = (int)(gb & 1);
                        // P_{j-1} written by the softmax warps; O buffer b read by the fold warps
                        const bool ready =
                            PAIR ? (mbar_wait_cluster(&p_ready[b], (uint32_t)((gb >> 1) & 1)) &&
                                    (gb < 2 || mbar_wait_cluster(&o_empty[b], (uint32_t)(((gb >> 1) - 1) & 1))))
                                 : (mbar_wait(&p_ready[b], (uint32_t)((gb >> 1) & 1)) &&
                                    (gb < 2 || mbar_wait(&o_empty[b], (uint32_t)(((gb >> 1) - 1) & 1))));
                        if (!ready) {
                            s_fail = 1;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t ph = tmem + (uint32_t)(b * 128), pl = ph + 64;
                        const uint32_t od = tmem + 256u + (uint32_t)(b * 128);
#pragma unroll 1
                        for (int t = 0; t < SPB; ++t) {
                            const int s = (int)(g % NSLOT);
                            if (!slot_ready(s, g)) {
                                s_fail = 1;
                                break;
                            }
                            tc_fence_after();
                            // One SM: the slot holds keys [16 t, +16) x all 128 columns as
                            // four 32-column boxes; a pair CTA: keys [32 t, +32) x its 64
                            // columns, per 16 keys two 32-column boxes (4 KB apart).
                            constexpr int KSTEPS = PAIR ? 4 : 2;
#pragma unroll
                            for (int ks = 0; ks < KSTEPS; ++ks) {
                                const uint32_t vbyte = PAIR ? (uint32_t)((ks >> 1) * 4096 + (ks & 1) * 1024)
                                                            : (uint32_t)(ks * 1024);
                                const uint64_t dv = desc_mn_sw128(smem_u32(ring + s * SLOT), 2048, 512) + (vbyte >> 4);
                                const uint32_t col = (uint32_t)(t * 8 * KSTEPS + ks * 8);
                                const uint32_t acc = (t > 0 || ks > 0) ? 1u : 0u;
                                mma_o(od, ph + col, dv, acc);
                                mma_o(od, ph + col, dv + (SLOT / 2 >> 4), 1u);
                                mma_o(od, pl + col, dv, 1u);
                            }
                            commit(&slot_empty[s]);
                            ++g;
                        }
                        if (s_fail) break;
                        commit(&o_full[b]);
                    }
                }
                kb = kb0 + nkb;
            }
            if (s_fail) {   // release every role that may wait on the MMA thread
                for (int b = 0; b < 2; ++b) {
                    commit(&s_full[b]);
                    commit(&o_full[b]);
                }
            }
        }
    } else if (warp >= ROW_WARP0 && warp < SPLIT_WARP0) {
        // ---- row warps: softmax of block j, then the fold of block j-1 ------
        // Two threads per row: warp w and w + 4 share the TMEM lane quarter
        // w % 4; `half` picks score columns [32 half, 32 half + 32) and output
        // columns [64 half, 64 half + 64).  The pair agrees on the row maximum
        // through shared memory and a two-arrival mbarrier per quarter.
        const int quarter = warp & 3;
        const int half = (warp - ROW_WARP0) >> 2;
        const int r = quarter * 32 + lane;                       // row in the block
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        const float ct = p.c, ct_lo = p.c_lo;   // log2(e) / T and its rounding error
        int64_t kb = 0;
        uint32_t bad = 0;
        for (int64_t i = 0; i < my_units && !s_fail; ++i) {
            const int64_t u = unit0 + i * ustride;
            const int bh = (int)(u / p.nq), row = (int)(u % p.nq) * (PAIR ? 2 * BQ : BQ) + (int)rank * BQ + r;
            float m = -INFINITY, l = 0.0f, alpha_prev = 0.0f;
            float o[64];
#pragma unroll
            for (int c = 0; c < 64; ++c) o[c] = 0.0f;
            // O_kb = O * alpha + O_j from TMEM buffer kb % 2, then release it
            auto fold = [&](int64_t fkb, float alpha) -> bool {
                const int fb = (int)(fkb & 1);
                if (!mbar_wait_idle(&o_full[fb], (uint32_t)((fkb >> 1) & 1))) return false;
                tc_fence_after();
                const uint32_t obase = lane_base + 256u + (uint32_t)(fb * 128 + half * 64);
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    uint32_t x[16];
                    tmem_ld16(obase + (uint32_t)(h * 16), x);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 16; ++c) o[h * 16 + c] = fmaf(o[h * 16 + c], alpha, __uint_as_float(x[c]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) arrive_leader(&o_empty[fb]);
                return true;
            };
            for (int j = 0; j < nkb && !s_fail; ++j, ++kb) {
                const int b = (int)(kb & 1);
                if (!mbar_wait_idle(&s_full[b], (uint32_t)((kb >> 1) & 1))) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                if (s_fail) break;
                const int c0 = half * 32;
                const int valid = p.sk - j * BKEY - c0;     // valid columns of this half (may be <= 0 or > 32)
                const uint32_t sbase = lane_base + (uint32_t)(b * 128 + c0);
                // pass 1: this half's row maximum over the valid keys
                float bmax = -INFINITY;
#pragma unroll 1
                for (int h = 0; h < 2; ++h) {
                    uint32_t a0[16], x0[16];
                    tmem_ld16(sbase + (uint32_t)(h * 16), a0);
                    tmem_ld16(sbase + 64u + (uint32_t)(h * 16), x0);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const float sc = __uint_as_float(a0[c]) + __uint_as_float(x0[c]);
                        const bool in = h * 16 + c < valid;
                        bad |= in ? nonfinite_bits(sc) : 0u;
                        bmax = fmaxf(bmax, in ? sc : -INFINITY);
                    }
                }
                xmax[((kb & 1) * 2 + half) * BQ + r] = bmax;
                __syncwarp();
                if (lane == 0) mbar_arrive(&xbar[quarter]);
                if (!mbar_wait(&xbar[quarter], (uint32_t)(kb & 1))) {
                    s_fail = 1;
                    break;
                }
                bmax = fmaxf(bmax, xmax[((kb & 1) * 2 + (half ^ 1)) * BQ + r]);
                const float m_new = fmaxf(m, bmax);
                const float alpha = m != -INFINITY ? exp_scaled(m - m_new, ct, ct_lo) : 0.0f;
                // pass 2: P = exp((S - m) / T) split into hi and lo, written over S
                float bsum = 0.0f;
#pragma unroll 1
                for (int h = 0; h < 2; ++h) {
                    uint32_t a0[16], x0[16];
                    tmem_ld16(sbase + (uint32_t)(h * 16), a0);
                    tmem_ld16(sbase + 64u + (uint32_t)(h * 16), x0);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const bool in = h * 16 + c < valid;
                        const float diff = (__uint_as_float(a0[c]) + __uint_as_float(x0[c])) - m_new;
                        bad |= in ? nonfinite_bits(diff) : 0u;
                        const float pv = in ? exp_scaled(diff, ct, ct_lo) : 0.0f;
                        bsum += pv;
                        const float hi = tf32_trunc(pv);
                        a0[c] = __float_as_uint(hi);
                        x0[c] = __float_as_uint(pv - hi);
                    }
                    tmem_st16(sbase + (uint32_t)(h * 16), a0);
                    tmem_st16(sbase + 64u + (uint32_t)(h * 16), x0);
                }
                l = l * alpha + bsum;
                m = m_new;
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) arrive_leader(&p_ready[b]);
                // fold the previous block's O while the tensor cores run this one
                if (j > 0 && !fold(kb - 1, alpha_prev)) {
                    s_fail = 1;
                    break;
                }
                alpha_prev = alpha;
            }
            if (s_fail || !fold(kb - 1, alpha_prev)) {
                s_fail = 1;
                break;
            }
            // row sum: the two halves' partial sums, added in one order by both
            lsum[half * BQ + r] = l;
            __syncwarp();
            if (lane == 0) mbar_arrive(&lbar[quarter]);
            if (!mbar_wait(&lbar[quarter], (uint32_t)(i & 1))) {
                s_fail = 1;
                break;
            }
            // the partner reads this unit's sums before it joins the next
            // unit's first maximum exchange, which this warp's next write follows
            const float lfin = lsum[r] + lsum[BQ + r];
            if (row < p.sq) {
                float *dst = p.out + (int64_t)bh * p.o_bs + (int64_t)row * p.o_rs + half * 64;
#pragma unroll
                for (int c = 0; c < 64; c += 4)
                    *reinterpret_cast<float4 *>(dst + c) =
                        make_float4(o[c] / lfin, o[c + 1] / lfin, o[c + 2] / lfin, o[c + 3] / lfin);
            }
        }
        if (bad) atomicOr(p.flag, 1u);
    } else if (warp >= SPLIT_WARP0) {
        // ---- split warps: lo part of each q block ---------------------------
        const int wt = threadIdx.x - SPLIT_WARP0 * 32;
        for (int64_t i = 0; i < my_units && !s_fail; ++i) {
            if (!mbar_wait_idle(q_full, (uint32_t)(i & 1))) {
                s_fail = 1;
                break;
            }
            split_buf(smem_u32(smem), Q_BYTES / 16, Q_BYTES, wt);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) arrive_leader(q_conv);
        }
    }

    tc_fence_before();
    if constexpr (PAIR) {
        cluster_sync_any();   // no CTA leaves while the pair's MMAs or the other CTA's arrivals may touch it
    } else {
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                         : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                         : "memory");
    }
    if (threadIdx.x == 0 && s_fail) atomicOr(p.status, KX_TIMEOUT_FLAG);
}

}  // namespace attn
}  // namespace tc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// Launch the fused kernel for q [nb, sq, 128], kt given as k [nb, sk, 128]
// (row stride k_rs, unit stride along the head dimension), v [nb, sk, 128]
// and a C-contiguous out [nb, sq, 128].  KX_DECLINED when the tensor maps
// cannot describe the operands.
int run_attention_fused(Handle *h, const float *q, int64_t q_rs, int64_t q_bs, const float *k, int64_t k_rs,
                        int64_t k_bs, const float *v, int64_t v_rs, int64_t v_bs, float *out, int64_t nb, int64_t sq,
                        int64_t sk, float temperature, const char **kernel_name) {
    using namespace tc;
    using namespace tc::attn;
    auto al16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    if (!al16(q) || !al16(k) || !al16(v) || !al16(out)) return KX_DECLINED;
    for (int64_t s : {q_rs, k_rs, v_rs})
        if (s <= 0 || (s * 4) % 16 != 0) return KX_DECLINED;
    if (nb > 1)
        for (int64_t s : {q_bs, k_bs, v_bs})
            if (s <= 0 || (s * 4) % 16 != 0) return KX_DECLINED;
    if (nb > INT32_MAX || sq > INT32_MAX || sk > INT32_MAX) return KX_DECLINED;
    auto s2 = [&](int64_t bs, int64_t rs, int64_t rows) {
        return nb > 1 ? (uint64_t)bs * 4 : (uint64_t)((rs * 4 * rows + 15) / 16 * 16);
    };
    // lo parts of k and v, dense [nb, sk, 128] each, in the handle's buffer
    const uint64_t lo_elems = (uint64_t)nb * (uint64_t)sk * DH;
    int rc = h->grow(&h->attn, &h->attn_bytes, 2 * lo_elems * sizeof(float));
    if (rc) return rc;
    float *k_lo = static_cast<float *>(h->attn), *v_lo = k_lo + lo_elems;
    const uint64_t lo_bs = (uint64_t)sk * DH * 4;
    // CTA pairs when there are enough 256-row units to keep the pairs busy:
    // each CTA then stages 32 of a block's keys (a 32-row box of kt)
    const int64_t pair_units = (sq + 2 * BQ - 1) / (2 * BQ) * nb;
    const bool pair = pair_units >= h->sm_count / 2;
    const uint32_t krows = pair ? BKEY / 2 : BKEY;
    CUtensorMap mq, mk, mv, mkl, mvl;
    if (!make_map(&mq, q, DH, (uint64_t)sq, (uint64_t)nb, (uint64_t)q_rs * 4, s2(q_bs, q_rs, sq), 16, BQ,
                  CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map(&mk, k, DH, (uint64_t)sk, (uint64_t)nb, (uint64_t)k_rs * 4, s2(k_bs, k_rs, sk), 16, krows,
                  CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map(&mv, v, DH, (uint64_t)sk, (uint64_t)nb, (uint64_t)v_rs * 4, s2(v_bs, v_rs, sk), 32, 16,
                  CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) ||
        !make_map(&mkl, k_lo, DH, (uint64_t)sk, (uint64_t)nb, DH * 4, lo_bs, 16, krows, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map(&mvl, v_lo, DH, (uint64_t)sk, (uint64_t)nb, DH * 4, lo_bs, 32, 16,
                  CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
        return KX_DECLINED;
    Params pp;
    std::memset(&pp, 0, sizeof(pp));
    pp.out = out;
    pp.o_rs = DH;
    pp.o_bs = sq * DH;
    pp.sq = (int)sq;
    pp.sk = (int)sk;
    pp.nbatch = (int)nb;
    pp.nq = (int)(pair ? (sq + 2 * BQ - 1) / (2 * BQ) : (sq + BQ - 1) / BQ);
    pp.units = (int64_t)pp.nq * nb;
    pp.nkb = (int)((sk + BKEY - 1) / BKEY);
    const double cd = 1.4426950408889634 / (double)temperature;
    pp.c = (float)cd;
    pp.c_lo = (float)(cd - (double)pp.c);
    if (!std::isnormal(pp.c) || !std::isfinite(pp.c_lo)) return KX_DECLINED;
    pp.status = h->flags + kStatusWord;
    pp.flag = h->flags + kAttnFlagWord;
    const int64_t slots = pair ? h->sm_count / 2 : h->sm_count;      // pairs, or CTAs
    const int64_t grid = (pp.units < slots ? pp.units : slots) * (pair ? 2 : 1);
    const int64_t n4 = (int64_t)lo_elems / 4;
    const unsigned lo_grid = (unsigned)std::min<int64_t>((n4 + 255) / 256, 8LL * h->sm_count);
    split_lo_kernel<false><<<lo_grid, 256, 0, h->stream>>>(k, k_rs, k_bs, k_lo, sk, nb, pp.flag);
    split_lo_kernel<true><<<lo_grid, 256, 0, h->stream>>>(v, v_rs, v_bs, v_lo, sk, nb, pp.flag);
    h->launches += 2;
    cudaError_t ce = cudaGetLastError();
    if (pair) {
        if (ce == cudaSuccess)
            ce = cudaFuncSetAttribute(attn_3xtf32_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      SMEM_BYTES);
        if (ce == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)grid, 1, 1);
            cfg.blockDim = dim3(NT, 1, 1);
            cfg.dynamicSmemBytes = SMEM_BYTES;
            cfg.stream = h->stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = 2;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            ce = cudaLaunchKernelEx(&cfg, attn_3xtf32_kernel<true>, mq, mk, mv, mkl, mvl, pp);
            if (ce == cudaSuccess) ce = cudaGetLastError();
        }
        *kernel_name = "attn_3xtf32_pair_256x64";
    } else {
        if (ce == cudaSuccess)
            ce = cudaFuncSetAttribute(attn_3xtf32_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      SMEM_BYTES);
        if (ce == cudaSuccess) {
            attn_3xtf32_kernel<false><<<(unsigned)grid, NT, SMEM_BYTES, h->stream>>>(mq, mk, mv, mkl, mvl, pp);
            ce = cudaGetLastError();
        }
        *kernel_name = "attn_3xtf32_128x64";
    }
    ++h->launches;
    return ce == cudaSuccess ? KX_OK : h->cuda_fail(ce);
}


namespace {

// One batch stride for the leading dims of t (all but the last two), when
// they nest in C order (singleton dims ignored); false otherwise.
bool collapse_batch(const kx_tensor *t, int64_t *stride) {
    const int nb = (int)t->rank - 2;
    int64_t st = 0, expect = 0;
    bool have = false;
    for (int d = nb - 1; d >= 0; --d) {
        if (t->dims[d] == 1) continue;
        if (!have) {
            st = t->strides[d];
            expect = st * (int64_t)t->dims[d];
            have = true;
        } else {
            if (t->strides[d] != expect) return false;
            expect *= (int64_t)t->dims[d];
        }
    }
    *stride = have ? st : 0;
    return true;
}

// A C-contiguous descriptor over `data` with the given dims.
kx_tensor dense_desc(void *data, const uint64_t *dims, uint32_t rank) {
    kx_tensor t;
    std::memset(&t, 0, sizeof(t));
    t.data = data;
    t.rank = rank;
    int64_t st = 1;
    for (int d = (int)rank - 1; d >= 0; --d) {
        t.dims[d] = dims[d];
        t.strides[d] = st;
        st *= (int64_t)dims[d];
    }
    t.storage_len = (uint64_t)st;
    return t;
}

}  // namespace

// The composition the fused kernel stands for, run call by call on the
// handle's stream: S = matmul(q, kt), P = softmax_temperature(S, -1, T),
// out = matmul(P, v), with S and P in a grow-only buffer of the handle.
static int attention_composed(kx_handle *hh, const kx_tensor *q, const kx_tensor *kt, const kx_tensor *v,
                              float temperature, const kx_tensor *out, const MatmulPlan &ps, kx_error *err) {
    Handle *h = &hh->impl;
    const uint64_t ns = numel(ps.out_dims, ps.out_rank);
    int rc = h->grow(&h->attn, &h->attn_bytes, 2 * ns * sizeof(float) + 256);
    if (rc) return cuda_err(err, h, "attention");
    float *sbuf = static_cast<float *>(h->attn);
    float *pbuf = sbuf + (ns + 63) / 64 * 64;
    kx_tensor sd = dense_desc(sbuf, ps.out_dims, ps.out_rank);
    kx_tensor pd = dense_desc(pbuf, ps.out_dims, ps.out_rank);
    rc = kx_matmul_f32(hh, q, kt, &sd, err);
    if (rc) return rc;
    rc = kx_softmax_temperature_f32(hh, &sd, -1, temperature, &pd, err);
    if (rc) return rc;
    return kx_matmul_f32(hh, &pd, v, out, err);
}

extern "C" int kx_attention_f32(kx_handle *hh, const kx_tensor *q, const kx_tensor *kt, const kx_tensor *v,
                                float temperature, const kx_tensor *out, kx_error *err) {
    static const char *kOp = "attention";
    if (!hh) return set_err(err, KX_E_PARAM, kOp, "null handle");
    Handle *h = &hh->impl;
    Span sq_, sk_, sv_, so_;
    int rc = validate_tensor(q, 4, &sq_, err);
    if (rc) return rc;
    rc = validate_tensor(kt, 4, &sk_, err);
    if (rc) return rc;
    // the reference order: matmul(q, kt) validates first ...
    MatmulPlan ps, po;
    rc = matmul_shape(q->dims, q->rank, kt->dims, kt->rank, &ps, err);
    if (rc) return rc;
    // ... then softmax_temperature (temperature, then the axis -1 of S) ...
    if (!std::isfinite(temperature) || !(temperature > 0.0f))
        return set_err(err, KX_E_PARAM, "softmax_temperature", "temperature (must be finite and > 0)");
    if (ps.out_rank == 0) return set_err(err, KX_E_AXIS, "softmax_temperature", "axis", (uint64_t)-1, 0);
    // ... then matmul(P, v)
    rc = validate_tensor(v, 4, &sv_, err);
    if (rc) return rc;
    rc = matmul_shape(ps.out_dims, ps.out_rank, v->dims, v->rank, &po, err);
    if (rc) return rc;
    rc = validate_tensor(out, 4, &so_, err);
    if (rc) return rc;
    if (out->rank != po.out_rank)
        return set_err(err, KX_E_LAYOUT, kOp, "output shape mismatch", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
    for (uint32_t i = 0; i < po.out_rank; ++i)
        if (out->dims[i] != po.out_dims[i])
            return set_err(err, KX_E_LAYOUT, kOp, "output shape mismatch", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
    if (!is_c_contiguous(out))
        return set_err(err, KX_E_LAYOUT, kOp, "output must be C-contiguous", KX_LAYOUT_OUTPUT_NOT_C_CONTIGUOUS);
    if (spans_overlap(out->data, so_, q->data, sq_, 4) || spans_overlap(out->data, so_, kt->data, sk_, 4) ||
        spans_overlap(out->data, so_, v->data, sv_, 4))
        return set_err(err, KX_E_ALIAS, kOp, "output overlaps an input");
    if (numel(po.out_dims, po.out_rank) == 0) return KX_OK;
    DeviceGuard g(h->device);
    if (!g.ok) return set_err(err, KX_E_NO_DEVICE, kOp, "cannot select device");

    // Fused path: q [B.., sq, 128], kt [B.., 128, sk] (a transposed view of a
    // row-major k), v [B.., sk, 128], equal batch dims that nest into one
    // stride each, unit strides along the head dimension.
    bool fused = !h->ordered && h->f32_variant != KX_F32_FFMA && q->rank >= 2 && kt->rank == q->rank &&
                 v->rank == q->rank && ps.k == 128 && po.n == 128 && ps.m > 0 && ps.n > 0;
    int64_t qb = 0, kb_ = 0, vb = 0, nb = 1;
    if (fused) {
        const uint32_t br = q->rank - 2;
        for (uint32_t d = 0; d < br; ++d) {
            fused &= q->dims[d] == kt->dims[d] && q->dims[d] == v->dims[d];
            nb *= (int64_t)q->dims[d];
        }
        fused &= q->strides[q->rank - 1] == 1 && kt->strides[kt->rank - 2] == 1 && v->strides[v->rank - 1] == 1;
        fused &= collapse_batch(q, &qb) && collapse_batch(kt, &kb_) && collapse_batch(v, &vb);
    }
    if (fused) {
        cudaError_t ce = cudaMemsetAsync(h->flags + kAttnFlagWord, 0, sizeof(uint32_t), h->stream);
        if (ce != cudaSuccess) {
            h->cuda_fail(ce);
            return cuda_err(err, h, kOp);
        }
        const char *name = "none";
        rc = run_attention_fused(h, static_cast<const float *>(q->data) + q->origin, q->strides[q->rank - 2], qb,
                                 static_cast<const float *>(kt->data) + kt->origin, kt->strides[kt->rank - 1], kb_,
                                 static_cast<const float *>(v->data) + v->origin, v->strides[v->rank - 2], vb,
                                 static_cast<float *>(out->data) + out->origin, nb, (int64_t)ps.m, (int64_t)ps.n,
                                 temperature, &name);
        if (rc == KX_E_CUDA) return cuda_err(err, h, kOp);
        if (rc == KX_OK) {
            h->last_kernel = name;
            uint32_t words[8];
            ce = cudaMemcpyAsync(words, h->flags, sizeof(words), cudaMemcpyDeviceToHost, h->stream);
            if (ce == cudaSuccess) ce = cudaStreamSynchronize(h->stream);
            if (ce != cudaSuccess) {
                h->cuda_fail(ce);
                return cuda_err(err, h, kOp);
            }
            if (words[kStatusWord] & tc::KX_TIMEOUT_FLAG)
                return set_err(err, KX_E_TIMEOUT, kOp, "a bounded device wait expired");
            if (words[kAttnFlagWord] == 0) return KX_OK;
            // an inf/NaN score, an overflowing x - max or an inf/NaN in v: the
            // composed path gives the reference's result or error
        }
    }
    return attention_composed(hh, q, kt, v, temperature, out, ps, err);
}

}  // namespace kx
