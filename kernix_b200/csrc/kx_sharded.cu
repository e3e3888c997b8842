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
//   * kx_matmul_rows_sharded_f32: one rank's share of the row-sharded product,
//     each piece pushed into every peer's output as soon as it is computed:
//     copy engines (one stream per peer) while the next piece multiplies, and
//     for the last piece, with nothing left to overlap, either one store
//     through an NVLink multicast address (the NVSwitch fans it out) or a
//     kernel on all SMs writing to every peer.
#include <algorithm>
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

// The second stream and the events of the split last piece, created on first use.
bool tail_streams(Handle *h) {
    if (h->aux) return true;
    for (auto &e : h->aux_ev)
        if (!e && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return false;
    return cudaStreamCreateWithFlags(&h->aux, cudaStreamNonBlocking) == cudaSuccess;
}

// c[i] += p[i] for n floats of two C-contiguous row blocks.
__global__ void tail_add_kernel(float *__restrict__ c, const float *__restrict__ p, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t i0 = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    uint64_t done = 0;
    if (((reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(p)) & 15) == 0) {
        float4 *c4 = reinterpret_cast<float4 *>(c);
        const float4 *p4 = reinterpret_cast<const float4 *>(p);
        const uint64_t n4 = n / 4;
        for (uint64_t j = i0; j < n4; j += stride) {
            float4 x = c4[j];
            const float4 y = p4[j];
            x.x += y.x;
            x.y += y.y;
            x.z += y.z;
            x.w += y.w;
            c4[j] = x;
        }
        done = n4 * 4;
    }
    for (uint64_t j = done + i0; j < n; j += stride) c[j] += p[j];
}

// The last piece's fan-out below this many bytes (all peers together) costs
// too little exposed time for the split to pay: about 40 us at the measured
// 770 GB/s of one GPU's NVLink, against the split's two sums.
constexpr uint64_t kTailSplitBytes = 32ull << 20;

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
        return set_err(err, KX_E_LAYOUT, kOp, "local A must hold this rank's rows", a_local->dims[0], pieces * piece);
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
    // is large, the piece runs as two row halves, each as its two K halves at
    // once (the handle's stream and a second one, each planned for half the
    // SMs: one wave between them), summed by a small kernel; the first half's
    // rows then go out on the copy engines while the second half multiplies,
    // and only the second half's push is exposed.
    const uint64_t k = a_local->dims[1];
    const bool tail_split = push && !h->ordered && h->f32_variant == KX_F32_AUTO && piece % 256 == 0 &&
                            k % 8 == 0 && k >= 2048 && (uint64_t)(world - 1) * piece * row_bytes >= kTailSplitBytes;
    if (tail_split) {
        if (!tail_streams(h)) return set_err(err, KX_E_CUDA, kOp, "cannot create the second stream");
        if (h->grow(&h->tail, &h->tail_bytes, piece * row_bytes)) return cuda_err(err, h, kOp);
    }
    for (uint64_t i = 0; i < pieces; ++i) {
        const uint64_t g0 = (i * world + rank) * piece;       // global rows of this piece
        if (i + 1 == pieces && tail_split) {
            const uint64_t hr = piece / 2, kh = k / 2;
            float *part = static_cast<float *>(h->tail);
            // the second stream starts after everything the handle's stream holds so far
            cudaError_t ce = cudaEventRecord(h->aux_ev[0], h->stream);
            if (ce == cudaSuccess) ce = cudaStreamWaitEvent(h->aux, h->aux_ev[0], 0);
            if (ce != cudaSuccess) {
                h->cuda_fail(ce);
                return cuda_err(err, h, kOp);
            }
            for (uint64_t half = 0; half < 2; ++half) {
                const uint64_t lr = i * piece + half * hr, gr = g0 + half * hr;
                kx_tensor a1 = *a_local;                      // rows, first K half
                a1.dims[0] = hr;
                a1.dims[1] = kh;
                a1.origin = a_local->origin + (uint64_t)((int64_t)lr * a_local->strides[0]);
                kx_tensor a2 = a1;                            // second K half
                a2.origin = a1.origin + (uint64_t)((int64_t)kh * a_local->strides[1]);
                kx_tensor b1 = *b;
                b1.dims[0] = kh;
                kx_tensor b2 = b1;
                b2.origin = b->origin + (uint64_t)((int64_t)kh * b->strides[0]);
                kx_tensor c1 = *out;
                c1.dims[0] = hr;
                c1.origin = out->origin + gr * n;
                kx_tensor p2;
                std::memset(&p2, 0, sizeof(p2));
                p2.data = part + half * hr * n;
                p2.storage_len = hr * n;
                p2.rank = 2;
                p2.dims[0] = hr;
                p2.dims[1] = n;
                p2.strides[0] = (int64_t)n;
                p2.strides[1] = 1;
                const int budget = h->sm_budget;
                h->sm_budget = h->sm_count / 2;
                int rc = kx_matmul_f32(hh, &a1, &b1, &c1, err);
                if (rc == KX_OK) {
                    cudaStream_t main_stream = h->stream;
                    h->stream = h->aux;
                    rc = kx_matmul_f32(hh, &a2, &b2, &p2, err);
                    h->stream = main_stream;
                }
                h->sm_budget = budget;
                if (rc) return rc;
                ce = cudaEventRecord(h->aux_ev[1 + half], h->aux);
                if (ce == cudaSuccess) ce = cudaStreamWaitEvent(h->stream, h->aux_ev[1 + half], 0);
                if (ce == cudaSuccess) {
                    const uint64_t total = hr * n;
                    uint64_t blocks = (total / 4 + 255) / 256;
                    blocks = std::max<uint64_t>(1, std::min<uint64_t>(blocks, 4ull * h->sm_count));
                    tail_add_kernel<<<(unsigned)blocks, 256, 0, h->stream>>>(c + gr * n, part + half * hr * n, total);
                    ++h->launches;
                    ce = cudaGetLastError();
                }
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

}  // extern "C"
