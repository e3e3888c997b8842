// Shared pieces of the split-TF32 tcgen05 kernels (GEMM and conv2d): tile
// constants, bounded mbarrier waits, TMA and tcgen05 wrappers, shared-memory
// matrix descriptors, TMEM loads and the hi/lo split of an f32 value.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "kx_internal.hpp"

namespace kx {
namespace tc {

constexpr int BM = 128, BK = 16, STAGES = 4;
constexpr int A_TILE = BM * BK * 4;                   // 8 KB
constexpr int BAR_BYTES = 256;   // 3 x STAGES + 2 mbarriers and the TMEM address
constexpr int NTHREADS = 384;                        // 12 warps
constexpr int WORK_WARP0 = 4, WORK_WARPS = 8, WORK_THREADS = WORK_WARPS * 32;
constexpr int KC = 64;                                // k-tiles (1024 k) per hi*hi chunk
constexpr uint32_t TMEM_COLS = 512;   // main (hi*hi) + cross (hi*lo + lo*hi) accumulators
constexpr uint32_t XCOL = 256;        // first TMEM column of the cross-term accumulator

// Tile width N: 256; 224 when it packs the tiles into fewer full waves of SMs
// (e.g. 512 x 8192 outputs: 148 tiles of 128 x 224 = one wave, against 128
// tiles of 128 x 256 leaving 20 SMs idle); 128 for narrow products (N = 128:
// the attention value product) that would leave most of a wider tile empty.
template <int BN> struct TileN {
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "tile width");
    static constexpr int B_TILE = BN * BK * 4;                   // 16 KB at 256
    static constexpr int STAGE_BYTES = 2 * A_TILE + 2 * B_TILE;  // 48 KB at 256
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
    static constexpr int HALF_COLS = BN / 2;                     // accumulator columns per worker thread
    static constexpr int CONV_CHUNKS = (A_TILE + B_TILE) / 16;   // 16-byte chunks per stage
    static constexpr int CONV_ITERS = (CONV_CHUNKS + WORK_THREADS - 1) / WORK_THREADS;
};
constexpr uint64_t WAIT_NS = 2000000000ull;           // 2 s per wait
constexpr uint32_t KX_TIMEOUT_FLAG = 1u;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Bounded wait for the phase with the given parity; false once `wait_ns`
// nanoseconds have passed without it.
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t parity, uint64_t wait_ns) {
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
        if (deadline == 0) deadline = now + wait_ns;
        else if (now > deadline) return false;
    }
}
// Bounded wait for the phase with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    return mbar_wait_for(bar, parity, WAIT_NS);
}
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}
// Explicit shared-memory accesses by 32-bit shared address (pointers aligned
// through integer arithmetic otherwise become generic accesses).
__device__ __forceinline__ float lds_f32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ int4 lds_v4_s32(uint32_t a) {
    int4 v;
    asm volatile("ld.shared.v4.s32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a)
                 : "memory");
    return v;
}
__device__ __forceinline__ void sts_v4_f32(uint32_t a, float x, float y, float z, float w) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w) : "memory");
}
__device__ __forceinline__ float4 lds_v4_f32(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a)
                 : "memory");
    return v;
}
// TMA tensor store of a shared-memory box (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// at most N bulk groups of this thread still read their shared-memory source
template <int N> __device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// all of this thread's bulk groups have completed
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptors (tcgen05 canonical layouts, version 1).
//   K-major, 64-byte swizzle: 8-row groups 512 B apart (SBO), LBO unused (1).
//   MN-major 32-bit data uses the 128-byte swizzle on 32-byte atoms
//   (layout type 1, TMA CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B): atoms of 4 k-rows
//   x 128 B, 32-element MN blocks LBO apart, 4-row k groups SBO apart.
__device__ __forceinline__ uint64_t desc_k_sw64(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(512 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
}
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46) | ((uint64_t)1 << 61);
}
// Instruction descriptor: f32 accumulate, tf32 A and B, M = 128, N = BN.
template <int BN>
__host__ __device__ constexpr uint32_t idesc_tf32(bool b_mn_major) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (0u << 15) | ((b_mn_major ? 1u : 0u) << 16) |
           ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// Split x = hi + lo with hi = x truncated to tf32 (its low 13 mantissa bits
// cleared) and lo = x - hi, exact in f32.  The tensor core itself reads f32
// operands of a kind::tf32 MMA truncated to tf32, so the raw tile serves as hi
// unchanged and only lo is written.  lo has at most 13 significant bits and the
// MMA keeps 11 of them; with the dropped lo*lo term the error per product stays
// below ~1.7e-6 |a b| even for adversarial mantissas.
__device__ __forceinline__ float tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }
// Stores through an NVLink multicast address: one store reaches the same
// offset of C on every GPU bound to the multicast object.
__device__ __forceinline__ void mc_st4(float *addr, float a, float b, float c, float d) {
    asm volatile("multimem.st.weak.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}
__device__ __forceinline__ void mc_st1(float *addr, float v) {
    asm volatile("multimem.st.weak.global.b32 [%0], %1;" ::"l"(addr), "r"(__float_as_uint(v)) : "memory");
}

// Exponent of all ones: an inf or NaN input.
__device__ __forceinline__ uint32_t nonfinite_bits(float x) {
    return (__float_as_uint(x) & 0x7F800000u) == 0x7F800000u ? 1u : 0u;
}

// Split one stage's raw TMA tiles in place: each of this thread's 16-byte
// chunks c = wt, wt + NT, ... below `chunks` (A's first `a_chunks`, B's from
// byte `b_off`) gets its lo part x - tf32(x) `a_lo` (A) or `b_lo` (B) bytes
// further; the raw chunk stays as hi.  All loads are issued before the
// stores, with explicit shared-memory instructions.  Returns the nonfinite
// bits of the chunks read.
template <int ITERS, int NT>
__device__ __forceinline__ uint32_t split_stage(uint32_t base, int wt, int chunks, int a_chunks, uint32_t b_off,
                                                uint32_t a_lo, uint32_t b_lo) {
    float4 v[ITERS];
    uint32_t at[ITERS];
#pragma unroll
    for (int j = 0; j < ITERS; ++j) {
        const int c = wt + j * NT;
        at[j] = c < a_chunks ? base + (uint32_t)c * 16 : base + b_off + (uint32_t)(c - a_chunks) * 16;
        if (c < chunks) v[j] = lds_v4_f32(at[j]);
    }
    uint32_t bad = 0;
#pragma unroll
    for (int j = 0; j < ITERS; ++j) {
        const int c = wt + j * NT;
        if (c < chunks) {
            bad |= nonfinite_bits(v[j].x) | nonfinite_bits(v[j].y) | nonfinite_bits(v[j].z) | nonfinite_bits(v[j].w);
            sts_v4_f32(at[j] + (c < a_chunks ? a_lo : b_lo), v[j].x - tf32_trunc(v[j].x), v[j].y - tf32_trunc(v[j].y),
                       v[j].z - tf32_trunc(v[j].z), v[j].w - tf32_trunc(v[j].w));
        }
    }
    return bad;
}

// 16 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Add this thread's half row (HALF columns starting at col0) of the hi*hi
// TMEM accumulator into the register running sum.
template <int HALF>
__device__ __forceinline__ void tmem_accumulate(uint32_t tmem, int quarter, int col0, float (&sum)[HALF]) {
    static_assert(HALF % 16 == 0, "16-column groups");
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col0;
#pragma unroll
    for (int c = 0; c < HALF / 32; ++c) {
        uint32_t r0[16], r1[16];   // two loads in flight per wait
        tmem_ld16(lane_base + (uint32_t)(c * 32), r0);
        tmem_ld16(lane_base + (uint32_t)(c * 32 + 16), r1);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            sum[c * 32 + j] += __uint_as_float(r0[j]);
            sum[c * 32 + 16 + j] += __uint_as_float(r1[j]);
        }
    }
    if constexpr (HALF % 32 != 0) {
        constexpr int c0 = HALF / 32 * 32;
        uint32_t r0[16];
        tmem_ld16(lane_base + (uint32_t)c0, r0);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) sum[c0 + j] += __uint_as_float(r0[j]);
    }
}

// K-major, no swizzle (canonical interleaved layout): 8-row x 16-byte core
// matrices, `lbo` bytes between core matrices adjacent along k, `sbo` bytes
// between those adjacent along m/n.  Used for tiles written by threads.
__device__ __forceinline__ uint64_t desc_k_none(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
}

// ---- CTA pairs (tcgen05 cta_group::2) -------------------------------------
// f32 accumulate, tf32 A and B, M = 256 (the pair), N = the pair's width.
__host__ __device__ constexpr uint32_t idesc_pair(bool b_mn_major, int bnp) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(bnp >> 3) << 17) |
           ((uint32_t)(256 >> 4) << 24);
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
// Every thread of both CTAs arrives once per phase; threads may reach it
// from divergent paths (no .aligned).
__device__ __forceinline__ void cluster_sync_any() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Arrive on a barrier of either CTA of the pair (default semantics; the
// shared-memory writes it publishes were made visible to the tensor core's
// proxy by the writer's fence.proxy.async).  An explicit .release.cluster
// here cost a cluster-scope memory barrier per warp and k-tile.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z),
          "r"(z), "r"(z), "r"(z)
        : "memory");
}
// Completion of the leader's MMAs issued so far -> one arrive on the barrier
// at `cluster_addr` (in either CTA of the pair).
__device__ __forceinline__ void commit_pair(uint32_t cluster_addr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
                 : "memory");
}
// Bounded wait with cluster-scope acquire: the arrivals come from both CTAs
// (remote arrives carry release.cluster).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    uint64_t deadline = 0;
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        const uint64_t now = globaltimer();
        if (deadline == 0) deadline = now + WAIT_NS;
        else if (now > deadline) return false;
    }
}
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t cluster_addr) {
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
    return v;
}


// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// 3-d f32 tensor map: dims innermost first, strides (bytes) of dims 1 and 2.
inline bool make_map(CUtensorMap *map, const float *base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
              uint64_t s2_bytes, uint32_t b0, uint32_t b1, CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1_bytes, s2_bytes};
    cuuint32_t box[3] = {b0, b1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 4-d f32 tensor map without swizzle (dims innermost first, strides in bytes
// of dims 1..3), zero fill outside the tensor.
inline bool make_map4(CUtensorMap *map, const float *base, const uint64_t (&dims)[4], const uint64_t (&strides)[3],
                      const uint32_t (&box)[4]) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
    cuuint64_t st[3] = {strides[0], strides[1], strides[2]};
    cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(base), d, st, bx, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace tc
}  // namespace kx
