// Internal handle state shared by the C-ABI translation units.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "kx_host.hpp"

namespace kx {

template <typename T> struct GemmParams;

// One handle per (device, caller thread).  Owns a growable device workspace
// (split-K partials, host-hook staging) and a small flag area for device-side
// status words.  Not thread-safe: use one handle per thread/stream.
struct Handle {
    int device = 0;
    int sm_count = 148;
    cudaStream_t stream = nullptr;
    int f32_variant = KX_F32_AUTO;
    int f64_variant = KX_F64_AUTO;
    bool ordered = false;        // CpuExecutor::with_ordered_matmul equivalent
    uint64_t launches = 0;
    const char *last_kernel = "none";
    int last_cuda_error = 0;
    // Diagnostic (kx_diag_expire_next_gemm): nonzero makes the next one-SM
    // split-TF32 GEMM launch issue no copies and bound its waits by this many
    // nanoseconds, so that they expire.
    uint64_t diag_wait_ns = 0;

    void *ws = nullptr;          // split-K partials
    uint64_t ws_bytes = 0;
    void *stage[3] = {nullptr, nullptr, nullptr};   // host-hook device staging (a, b, out)
    uint64_t stage_bytes[3] = {0, 0, 0};
    void *attn = nullptr;        // scores and probabilities of the composed attention path
    uint64_t attn_bytes = 0;
    void *bwd = nullptr;         // full-batch gradients before their broadcast sum (kx_backward.cu)
    uint64_t bwd_bytes = 0;
    void *perm = nullptr;        // tensordot operands gathered into GEMM order (kx_tensordot.cu)
    uint64_t perm_bytes = 0;
    uint32_t *flags = nullptr;   // device status words (nonfinite index, timeouts)
    static constexpr int kFlagWords = 64;
    // Host-hook pipeline: copy streams and per-piece events, created on first use.
    cudaStream_t h2d = nullptr, d2h = nullptr;
    static constexpr int kMaxPieces = 16;
    // Row-sharded products (kx_sharded.cu): one copy stream per peer GPU and
    // events to order them after a piece and before the end of the call.
    static constexpr int kMaxWorld = 8;
    cudaStream_t peer_stream[kMaxWorld] = {};
    cudaEvent_t peer_ready = nullptr;
    cudaEvent_t peer_done[kMaxWorld] = {};
    // The K-half partial products of a row-sharded product's split last piece
    // (kx_sharded.cu).
    void *tail = nullptr;
    uint64_t tail_bytes = 0;
    cudaEvent_t ev[3 * kMaxPieces + 2] = {};

    int cuda_fail(cudaError_t ce) {
        last_cuda_error = (int)ce;
        return KX_E_CUDA;
    }
    // Grow-only device buffer.  Growing synchronises the stream first so that
    // no queued kernel still reads the old allocation.
    int grow(void **buf, uint64_t *cap, uint64_t need) {
        if (need <= *cap) return KX_OK;
        if (*buf) {
            cudaError_t ce = cudaStreamSynchronize(stream);
            if (ce != cudaSuccess) return cuda_fail(ce);
            cudaFree(*buf);
            *buf = nullptr;
            *cap = 0;
        }
        uint64_t bytes = need < (1u << 20) ? (1u << 20) : need;
        cudaError_t ce = cudaMalloc(buf, bytes);
        if (ce != cudaSuccess) {
            *buf = nullptr;
            return cuda_fail(ce);
        }
        *cap = bytes;
        return KX_OK;
    }
    int workspace(uint64_t need, void **out) {
        int rc = grow(&ws, &ws_bytes, need);
        if (rc == KX_OK) *out = ws;
        return rc;
    }
};

// Make the handle's device current for the duration of a call and restore the
// caller's device afterwards.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// Error record for a failed CUDA call.
inline int cuda_err(kx_error *e, Handle *h, const char *op) {
    set_err(e, KX_E_CUDA, op, cudaGetErrorString((cudaError_t)h->last_cuda_error));
    if (e) e->cuda_error = h->last_cuda_error;
    return KX_E_CUDA;
}

template <typename T> int run_gemm(Handle *h, GemmParams<T> p, const char **kernel_name);
// Split-TF32 tensor-core GEMM (kx_gemm_tc.cu).  KX_DECLINED when a tensor map
// cannot describe the operands (the caller then uses the SIMT kernel).
bool tc_eligible(const GemmParams<float> &p);
int run_gemm_tc(Handle *h, const GemmParams<float> &p, const char **kernel_name);
// The same arithmetic on CTA pairs (tcgen05 cta_group::2, 256 x 256 tiles;
// kx_gemm_tc2.cu).  KX_DECLINED when a tensor map cannot describe the operands.
int run_gemm_tc_pair(Handle *h, const GemmParams<float> &p, const char **kernel_name);
// Persistent split-TF32 kernel for K <= 1024 with the epilogue overlapping the
// next tile (kx_gemm_tc_short.cu).  KX_DECLINED for longer K or unmappable operands.
int run_gemm_tc_short(Handle *h, const GemmParams<float> &p, const char **kernel_name);
// conv2d as a split-TF32 implicit GEMM on the tensor cores (kx_conv_tc.cu);
// strides of x and w in elements (singleton dims zero).  KX_DECLINED when the
// weights are not dense tap rows or the tap count is outside its table.
int run_conv_tc(Handle *h, const float *x, const int64_t *xs, const float *w, const int64_t *ws, float *y,
                int64_t n, int64_t c, int64_t ih, int64_t iw, int64_t co, int64_t cg, int64_t kh, int64_t kw,
                int64_t oh, int64_t ow, int64_t groups, int64_t sy, int64_t sx, int64_t py, int64_t px, int64_t dy,
                int64_t dx, const char **kernel_name);
// f64 on the FP64 tensor pipe (kx_gemm_f64.cu).  KX_DECLINED for layouts
// without a unit stride along k or m/n (the SIMT DFMA kernel takes those).
int run_gemm_dmma(Handle *h, const GemmParams<double> &p, const char **kernel_name);
// Store `bytes` (a multiple of 4) from this GPU's `src` through the NVLink
// multicast address `mc_dst`: the bytes land at the same offset in the buffer
// of every GPU bound to the multicast object (kx_nvls.cu).
int mc_copy(Handle *h, const void *src, void *mc_dst, uint64_t bytes);
// Layout of the handle's device flag area (32-bit words), one owner per word:
//   [1]     status written by device code: bit 0 = a bounded wait expired
//   [2..3]  softmax: 64-bit key of the first nonfinite element (8-byte aligned)
//   [4]     conv2d: some weight is NaN or infinite
//   [5]     fused attention: the composed path must run (bit 0: a score or
//           x - max is inf/NaN; bit 1: v holds an inf/NaN)
constexpr int kStatusWord = 1;
constexpr int kSoftmaxWord = 2;
constexpr int kConvFlagWord = 4;
constexpr int kAttnFlagWord = 5;

}  // namespace kx

struct kx_handle {
    kx::Handle impl;
};
