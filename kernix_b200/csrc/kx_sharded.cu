// Work split across the GPUs of one node, one process (and one handle) per GPU.
//
// Kernix splits a product over host threads inside one process:
// CpuExecutor::matmul_into (crates/kernix-ops/src/execution.rs:188-233) gives
// each worker a chunk of output rows.  Across GPUs each process owns its
// device, so the split is a plan every rank computes the same way, and the one
// exchange the row split needs -- every rank ending with the whole output --
// is done by this library over NVLink:
//
//   * kx_shard_window: a contiguous window of a batch axis (independent
//     units: attention heads, conv2d images); no exchange.
//   * kx_row_piece: the block-cyclic row plan of a row-sharded product:
//     global row block i * world + rank of `piece` rows is rank's piece i, so
//     each rank's pieces interleave and piece i of all ranks fills one
//     contiguous band of the output.
//   * kx_gemm_sharded_f32: the same row split driven from ONE process over
//     several handles (one per GPU): each handle multiplies its window of
//     rows, then the copy engines copy every window into every other
//     handle's output (peer access enabled between the devices).
//   * kx_matmul_rows_sharded_f32: one rank's share of the row-sharded product,
//     each piece pushed into every peer's output as soon as it is computed:
//     copy engines (one stream per peer) while the next piece multiplies, and
//     for the last piece, with nothing left to overlap, either one store
//     through an NVLink multicast address (the NVSwitch fans it out) or a
//     kernel on all SMs writing to every peer.
#include <algorithm>
#include <atomic>
#include <cstring>

#include "kx_internal.hpp"

extern "C" int kx_matmul_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out,
                             kx_error *err);
extern "C" int kx_peer_broadcast(kx_handle *h, const void *src, void *const *dsts, int ndst, uint64_t bytes,
                                 kx_error *err);

namespace kx {
namespace {

constexpr int kMaxWorld = Handle::kMaxWorld;

// The handle's peer streams and events, created on first use.
bool push_streams(Handle *h) {
    if (h->peer_ready) return true;
    for (int r = 0; r < kMaxWorld; ++r) {
        if (cudaStreamCreateWithFlags(&h->peer_stream[r], cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&h->peer_done[r], cudaEventDisableTiming) != cudaSuccess)
            return false;
    }
    return cudaEventCreateWithFlags(&h->peer_ready, cudaEventDisableTiming) == cudaSuccess;
}

// c[i] = p0[i] + p1[i] for n floats (C-contiguous row blocks): the two K
// halves of the split last piece, summed into the output rows.
__global__ void tail_sum_kernel(float *__restrict__ c, const float *__restrict__ p0, const float *__restrict__ p1,
                                uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t i0 = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    uint64_t done = 0;
    if (((reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(p0) | reinterpret_cast<uintptr_t>(p1)) & 15) ==
        0) {
        float4 *c4 = reinterpret_cast<float4 *>(c);
        const float4 *a4 = reinterpret_cast<const float4 *>(p0);
        const float4 *b4 = reinterpret_cast<const float4 *>(p1);
        const uint64_t n4 = n / 4;
        for (uint64_t j = i0; j < n4; j += stride) {
            const float4 x = a4[j], y = b4[j];
            c4[j] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
        }
        done = n4 * 4;
    }
    for (uint64_t j = done + i0; j < n; j += stride) c[j] = p0[j] + p1[j];
}

// The last piece's fan-out below this many bytes (all peers together) costs
// too little exposed time for the split to pay: about 40 us at the measured
// 770 GB/s of one GPU's NVLink, against the split's two sums.
constexpr uint64_t kTailSplitBytes = 32ull << 20;

// Peer access from `dev` to `peer` for this process, enabled once per pair
// (copies between the devices then go over NVLink directly; without it the
// runtime stages them, still correct).
void enable_peer(int dev, int peer) {
    static std::atomic<uint64_t> done[kMaxWorld * 8] = {};
    if (dev == peer || dev < 0 || peer < 0) return;
    const int word = dev % (kMaxWorld * 8);
    const uint64_t bit = 1ull << (peer % 64);
    if (done[word].load() & bit) return;
    int can = 0;
    if (cudaDeviceCanAccessPeer(&can, dev, peer) == cudaSuccess && can) {
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(dev);
        // already enabled is no error for the caller, and a refusal leaves the
        // copies staged: either way nothing is left for a later error check
        if (cudaDeviceEnablePeerAccess(peer, 0) != cudaSuccess) cudaGetLastError();
        if (prev >= 0) cudaSetDevice(prev);
    }
    done[word].fetch_or(bit);
}

}  // namespace
}  // namespace kx

using namespace kx;

extern "C" {

int kx_shard_window(uint64_t total, uint32_t rank, uint32_t world, uint64_t *start, uint64_t *count) {
    if (!start || !count || world == 0 || rank >= world) return KX_E_PARAM;
    // the first total % world ranks take one unit more
    const uint64_t base = total / world, extra = total % world;
    *start = rank * base + std::min<uint64_t>(rank, extra);
    *count = base + (rank < extra ? 1 : 0);
    return KX_OK;
}

int kx_row_piece(uint64_t m, uint32_t world, uint64_t target_piece, uint64_t *piece, uint64_t *pieces) {
    if (!piece || !pieces || world == 0 || m % world != 0 || target_piece == 0) return KX_E_PARAM;
    // the largest piece <= target_piece that tiles M evenly across the ranks
    const uint64_t per_rank = m / world;
    uint64_t p = std::min<uint64_t>(target_piece, per_rank);
    while (p > 1 && per_rank % p) --p;
    if (p == 0) return KX_E_PARAM;
    *piece = p;
    *pieces = per_rank / p;
    return KX_OK;
}

int kx_matmul_rows_sharded_f32(kx_handle *hh, const kx_tensor *a_local, const kx_tensor *b, const kx_tensor *out,
                               uint32_t rank, uint32_t world, uint64_t piece, void *const *peer_out, void *out_mc,
                               kx_error *err) {
    static const char *kOp = "matmul_rows_sharded";
    if (!hh) return set_err(err, KX_E_PARAM, kOp, "null handle");
    Handle *h = &hh->impl;
    if (world == 0 || world > kMaxWorld || rank >= world)
        return set_err(err, KX_E_PARAM, kOp, "rank and world (1..8 GPUs)", rank, world);
    if (!a_local || !out || a_local->rank != 2 || out->rank != 2)
        return set_err(err, KX_E_PARAM, kOp, "rank-two local A and output");
    const uint64_t m = out->dims[0], n = out->dims[1];
    if (piece == 0 || m % ((uint64_t)world * piece) != 0)
        return set_err(err, KX_E_PARAM, kOp, "piece rows must tile M over the ranks", m, piece);
    const uint64_t pieces = m / ((uint64_t)world * piece);
    if (a_local->dims[0] != pieces * piece)
        return set_err(err, KX_E_PARAM, kOp, "local A must hold this rank's rows", a_local->dims[0], pieces * piece);
    if (!is_c_contiguous(out))
        return set_err(err, KX_E_LAYOUT, kOp, "output must be C-contiguous", KX_LAYOUT_OUTPUT_NOT_C_CONTIGUOUS);
    DeviceGuard g(h->device);
    if (!g.ok) return set_err(err, KX_E_NO_DEVICE, kOp, "cannot select device");
    const bool push = peer_out != nullptr && world > 1;
    if (push && !push_streams(h)) return set_err(err, KX_E_CUDA, kOp, "cannot create the push streams");
    float *c = static_cast<float *>(out->data) + out->origin;
    const uint64_t row_bytes = n * sizeof(float);
    // rows [off, off + bytes) of C into every peer's C: by the copy engines
    // (one stream per peer) after what the handle's stream has queued so far
    auto push_ce = [&](uint64_t off, uint64_t bytes) -> int {
        const char *src = reinterpret_cast<const char *>(c) + off;
        cudaError_t ce = cudaEventRecord(h->peer_ready, h->stream);
        for (uint32_t r = 0; r < world && ce == cudaSuccess; ++r) {
            if (r == rank) continue;
            ce = cudaStreamWaitEvent(h->peer_stream[r], h->peer_ready, 0);
            if (ce == cudaSuccess)
                ce = cudaMemcpyAsync(static_cast<char *>(peer_out[r]) + out->origin * sizeof(float) + off, src, bytes,
                                     cudaMemcpyDeviceToDevice, h->peer_stream[r]);
        }
        if (ce != cudaSuccess) {
            h->cuda_fail(ce);
            return cuda_err(err, h, kOp);
        }
        return KX_OK;
    };
    // the same for the last rows, with nothing left to overlap: one store
    // through the multicast address, or a kernel on all SMs
    auto push_last = [&](uint64_t off, uint64_t bytes) -> int {
        const char *src = reinterpret_cast<const char *>(c) + off;
        if (out_mc) {
            if (mc_copy(h, src, static_cast<char *>(out_mc) + out->origin * sizeof(float) + off, bytes))
                return cuda_err(err, h, kOp);
            return KX_OK;
        }
        void *dsts[kMaxWorld];
        int nd = 0;
        for (uint32_t r = 0; r < world; ++r)
            if (r != rank) dsts[nd++] = static_cast<char *>(peer_out[r]) + out->origin * sizeof(float) + off;
        return kx_peer_broadcast(hh, src, dsts, nd, bytes, err);
    };
    // The last piece's push has no GEMM left to hide behind.  When its fan-out
    // is large, the piece runs as two row halves, each ONE batched GEMM whose
    // batch is its two K halves (the same number of CTAs as the whole piece:
    // one wave, half as long), the halves' partial products summed into the
    // output rows by a small kernel; the first half's rows then go out on the
    // copy engines while the second half multiplies, and only the second
    // half's push is exposed.  Measured on the 8192^3 product: 4 GPUs 781.7 ->
    // 794.2 TFLOP/s; 8 GPUs 1012.1 -> 985.8, where the first half's push
    // meets the previous piece's push still arriving from seven peers on the
    // same inbound links -- so up to 4 GPUs only.
    const uint64_t k = a_local->dims[1];
    const bool tail_split = push && world <= 4 && !h->ordered && h->f32_variant == KX_F32_AUTO &&
                            piece % 256 == 0 && k % 8 == 0 && k >= 2048 &&
                            (uint64_t)(world - 1) * piece * row_bytes >= kTailSplitBytes;
    if (tail_split && h->grow(&h->tail, &h->tail_bytes, piece * row_bytes)) return cuda_err(err, h, kOp);
    for (uint64_t i = 0; i < pieces; ++i) {
        const uint64_t g0 = (i * world + rank) * piece;       // global rows of this piece
        if (i + 1 == pieces && tail_split) {
            const uint64_t hr = piece / 2, kh = k / 2;
            float *part = static_cast<float *>(h->tail);      // [2][hr][n]: the two K halves
            for (uint64_t half = 0; half < 2; ++half) {
                const uint64_t lr = i * piece + half * hr, gr = g0 + half * hr;
                kx_tensor a3 = *a_local;                      // [2, hr, kh]: K halves as a batch
                a3.rank = 3;
                a3.dims[0] = 2;
                a3.dims[1] = hr;
                a3.dims[2] = kh;
                a3.strides[0] = (int64_t)kh * a_local->strides[1];
                a3.strides[1] = a_local->strides[0];
                a3.strides[2] = a_local->strides[1];
                a3.origin = a_local->origin + (uint64_t)((int64_t)lr * a_local->strides[0]);
                kx_tensor b3 = *b;                            // [2, kh, n]
                b3.rank = 3;
                b3.dims[0] = 2;
                b3.dims[1] = kh;
                b3.dims[2] = n;
                b3.strides[0] = (int64_t)kh * b->strides[0];
                b3.strides[1] = b->strides[0];
                b3.strides[2] = b->strides[1];
                kx_tensor p3;
                std::memset(&p3, 0, sizeof(p3));
                p3.data = part;
                p3.storage_len = 2 * hr * n;
                p3.rank = 3;
                p3.dims[0] = 2;
                p3.dims[1] = hr;
                p3.dims[2] = n;
                p3.strides[0] = (int64_t)(hr * n);
                p3.strides[1] = (int64_t)n;
                p3.strides[2] = 1;
                int rc = kx_matmul_f32(hh, &a3, &b3, &p3, err);
                if (rc) return rc;
                const uint64_t total = hr * n;
                uint64_t blocks = (total / 4 + 255) / 256;
                blocks = std::max<uint64_t>(1, std::min<uint64_t>(blocks, 4ull * h->sm_count));
                tail_sum_kernel<<<(unsigned)blocks, 256, 0, h->stream>>>(c + gr * n, part, part + total, total);
                ++h->launches;
                const cudaError_t ce = cudaGetLastError();
                if (ce != cudaSuccess) {
                    h->cuda_fail(ce);
                    return cuda_err(err, h, kOp);
                }
                rc = half == 0 ? push_ce(gr * row_bytes, hr * row_bytes) : push_last(gr * row_bytes, hr * row_bytes);
                if (rc) return rc;
            }
            continue;
        }
        kx_tensor ap = *a_local;                               // local rows [i * piece, (i + 1) * piece)
        ap.dims[0] = piece;
        ap.origin = a_local->origin + (uint64_t)((int64_t)(i * piece) * a_local->strides[0]);
        kx_tensor cp = *out;
        cp.dims[0] = piece;
        cp.origin = out->origin + g0 * n;
        int rc = kx_matmul_f32(hh, &ap, b, &cp, err);
        if (rc) return rc;
        if (!push) continue;
        rc = i + 1 == pieces ? push_last(g0 * row_bytes, piece * row_bytes) : push_ce(g0 * row_bytes, piece * row_bytes);
        if (rc) return rc;
    }
    if (push) {
        // the handle's stream completes only after every push has
        for (uint32_t r = 0; r < world; ++r) {
            if (r == rank) continue;
            cudaError_t ce = cudaEventRecord(h->peer_done[r], h->peer_stream[r]);
            if (ce == cudaSuccess) ce = cudaStreamWaitEvent(h->stream, h->peer_done[r], 0);
            if (ce != cudaSuccess) {
                h->cuda_fail(ce);
                return cuda_err(err, h, kOp);
            }
        }
    }
    return KX_OK;
}

int kx_gemm_sharded_f32(kx_handle *const *handles, uint32_t ngpu, const kx_tensor *a, const kx_tensor *b,
                        const kx_tensor *out, int gather_out, kx_error *err) {
    static const char *kOp = "gemm_sharded";
    if (!handles || !a || !b || !out) return set_err(err, KX_E_PARAM, kOp, "null argument");
    if (ngpu == 0 || ngpu > (uint32_t)kMaxWorld) return set_err(err, KX_E_PARAM, kOp, "ngpu (1..8)", ngpu);
    for (uint32_t r = 0; r < ngpu; ++r)
        if (!handles[r]) return set_err(err, KX_E_PARAM, kOp, "null handle", r);
    // Every argument is checked before any work is enqueued.
    if (out[0].rank != 2) return set_err(err, KX_E_PARAM, kOp, "rank-two outputs");
    const uint64_t m = out[0].dims[0], n = out[0].dims[1];
    if (a[0].rank != 2) return set_err(err, KX_E_PARAM, kOp, "rank-two blocks of A");
    const uint64_t k = a[0].dims[1];
    Span so[kMaxWorld];
    for (uint32_t r = 0; r < ngpu; ++r) {
        Span sa, sb;
        int rc = validate_tensor(a + r, 4, &sa, err);
        if (!rc) rc = validate_tensor(b + r, 4, &sb, err);
        if (!rc) rc = validate_tensor(out + r, 4, &so[r], err);
        if (rc) return rc;
        uint64_t start = 0, count = 0;
        kx_shard_window(m, r, ngpu, &start, &count);
        if (a[r].rank != 2 || a[r].dims[0] != count || a[r].dims[1] != k)
            return set_err(err, KX_E_PARAM, kOp, "a[r] must be [rows of window r, K]", r, count);
        if (b[r].rank != 2 || b[r].dims[0] != k || b[r].dims[1] != n)
            return set_err(err, KX_E_PARAM, kOp, "b[r] must be [K, N]", r);
        if (out[r].rank != 2 || out[r].dims[0] != m || out[r].dims[1] != n)
            return set_err(err, KX_E_LAYOUT, kOp, "every output [M, N]", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
        if (!is_c_contiguous(out + r))
            return set_err(err, KX_E_LAYOUT, kOp, "output must be C-contiguous", KX_LAYOUT_OUTPUT_NOT_C_CONTIGUOUS);
        if (spans_overlap(out[r].data, so[r], a[r].data, sa, 4) || spans_overlap(out[r].data, so[r], b[r].data, sb, 4))
            return set_err(err, KX_E_ALIAS, kOp, "output overlaps an input");
    }
    if (gather_out)
        for (uint32_t r = 0; r < ngpu; ++r)
            for (uint32_t q = r + 1; q < ngpu; ++q)
                if (spans_overlap(out[r].data, so[r], out[q].data, so[q], 4))
                    return set_err(err, KX_E_ALIAS, kOp, "gathered outputs overlap", r, q);
    if (m == 0 || n == 0) return KX_OK;
    // Rows of window r in output q: one contiguous byte range.
    auto rows_at = [&](uint32_t q, uint64_t start) {
        return static_cast<char *>(out[q].data) + (out[q].origin + start * n) * sizeof(float);
    };
    const bool gather = gather_out && ngpu > 1;
    if (gather) {
        for (uint32_t r = 0; r < ngpu; ++r) {
            Handle *h = &handles[r]->impl;
            DeviceGuard g(h->device);
            if (!g.ok) return set_err(err, KX_E_NO_DEVICE, kOp, "cannot select device", r);
            if (!push_streams(h)) return set_err(err, KX_E_CUDA, kOp, "cannot create the gather events");
            for (uint32_t q = 0; q < ngpu; ++q) enable_peer(h->device, handles[q]->impl.device);
            // the point after which output r may be written by the other handles
            const cudaError_t ce = cudaEventRecord(h->peer_done[0], h->stream);
            if (ce != cudaSuccess) {
                h->cuda_fail(ce);
                return cuda_err(err, h, kOp);
            }
        }
    }
    for (uint32_t r = 0; r < ngpu; ++r) {
        Handle *h = &handles[r]->impl;
        uint64_t start = 0, count = 0;
        kx_shard_window(m, r, ngpu, &start, &count);
        if (count == 0) continue;
        kx_tensor cp = out[r];
        cp.dims[0] = count;
        cp.origin = out[r].origin + start * n;
        int rc = kx_matmul_f32(handles[r], a + r, b + r, &cp, err);
        if (rc) return rc;
        if (!gather) continue;
        DeviceGuard g(h->device);
        cudaError_t ce = cudaSuccess;
        for (uint32_t q = 0; q < ngpu && ce == cudaSuccess; ++q) {
            if (q == r) continue;
            const Handle *hq = &handles[q]->impl;
            ce = cudaStreamWaitEvent(h->stream, hq->peer_done[0], 0);
            if (ce != cudaSuccess) break;
            const uint64_t bytes = count * n * sizeof(float);
            ce = hq->device == h->device
                     ? cudaMemcpyAsync(rows_at(q, start), rows_at(r, start), bytes, cudaMemcpyDeviceToDevice, h->stream)
                     : cudaMemcpyPeerAsync(rows_at(q, start), hq->device, rows_at(r, start), h->device, bytes,
                                           h->stream);
        }
        if (ce == cudaSuccess) ce = cudaEventRecord(h->peer_ready, h->stream);
        if (ce != cudaSuccess) {
            h->cuda_fail(ce);
            return cuda_err(err, h, kOp);
        }
    }
    if (gather) {
        // each handle's stream completes only after every window has reached its output
        for (uint32_t q = 0; q < ngpu; ++q) {
            Handle *h = &handles[q]->impl;
            DeviceGuard g(h->device);
            for (uint32_t r = 0; r < ngpu; ++r) {
                uint64_t start = 0, count = 0;
                kx_shard_window(m, r, ngpu, &start, &count);
                if (r == q || count == 0) continue;
                const cudaError_t ce = cudaStreamWaitEvent(h->stream, handles[r]->impl.peer_ready, 0);
                if (ce != cudaSuccess) {
                    h->cuda_fail(ce);
                    return cuda_err(err, h, kOp);
                }
            }
        }
    }
    return KX_OK;
}

}  // extern "C"
