// Gathered output of a row-sharded GEMM across the GPUs of one node: export a
// device buffer to the node's other processes, map theirs, and push rows into
// them with the copy engines.
//
// Kernix's CpuExecutor::matmul_into (crates/kernix-ops/src/execution.rs:188-233)
// splits the rows of one output over threads that share it.  One process per
// GPU cannot share a buffer that way, so each rank computes its rows into its
// own copy of C and pushes them into every peer's copy: CUDA IPC maps the
// peers' allocations into this process (peer access over NVLink), and
// cudaMemcpyAsync between mapped device pointers runs on the copy engines, so
// the exchange overlaps the next GEMM without taking its SMs.
#include <cstring>

#include "kx_internal.hpp"

using namespace kx;

static_assert(sizeof(cudaIpcMemHandle_t) == KX_IPC_HANDLE_BYTES, "IPC handle size");

namespace {

constexpr int kMaxPeers = 8;
struct PeerDsts {
    float4 *d[kMaxPeers];
    int n;
};

// src -> every destination, 16 bytes at a time, all SMs: used for the last
// piece of a sharded GEMM, when no GEMM is left to overlap and the copy
// engines' fan-out rate would set the step time.  Stores to mapped peer
// memory travel over NVLink; the closing fence orders them before whatever
// tells the peers that this rank is done.
__global__ void __launch_bounds__(256) peer_broadcast_kernel(const float4 *__restrict__ src, const PeerDsts dst,
                                                             uint64_t n16) {
    const uint64_t nth = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += nth) {
        const float4 v = __ldg(src + i);
#pragma unroll
        for (int j = 0; j < kMaxPeers; ++j)
            if (j < dst.n) dst.d[j][i] = v;
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

}  // namespace

extern "C" {

int kx_ipc_export(kx_handle *hh, void *device_ptr, unsigned char *handle_out, kx_error *err) {
    static const char *kOp = "ipc_export";
    if (!hh || !device_ptr || !handle_out) return set_err(err, KX_E_PARAM, kOp, "null argument");
    Handle *h = &hh->impl;
    DeviceGuard g(h->device);
    cudaIpcMemHandle_t ipc;
    cudaError_t ce = cudaIpcGetMemHandle(&ipc, device_ptr);
    if (ce != cudaSuccess) {
        h->cuda_fail(ce);
        return cuda_err(err, h, kOp);
    }
    std::memcpy(handle_out, &ipc, sizeof(ipc));
    return KX_OK;
}

int kx_ipc_import(kx_handle *hh, const unsigned char *handle, void **device_ptr, kx_error *err) {
    static const char *kOp = "ipc_import";
    if (!hh || !handle || !device_ptr) return set_err(err, KX_E_PARAM, kOp, "null argument");
    Handle *h = &hh->impl;
    DeviceGuard g(h->device);
    cudaIpcMemHandle_t ipc;
    std::memcpy(&ipc, handle, sizeof(ipc));
    *device_ptr = nullptr;
    cudaError_t ce = cudaIpcOpenMemHandle(device_ptr, ipc, cudaIpcMemLazyEnablePeerAccess);
    if (ce != cudaSuccess) {
        *device_ptr = nullptr;
        h->cuda_fail(ce);
        return cuda_err(err, h, kOp);
    }
    return KX_OK;
}

int kx_ipc_close(kx_handle *hh, void *device_ptr) {
    if (!hh || !device_ptr) return KX_E_PARAM;
    DeviceGuard g(hh->impl.device);
    return cudaIpcCloseMemHandle(device_ptr) == cudaSuccess ? KX_OK : KX_E_CUDA;
}

int kx_peer_broadcast(kx_handle *hh, const void *src, void *const *dsts, int ndst, uint64_t bytes, kx_error *err) {
    static const char *kOp = "peer_broadcast";
    if (!hh) return set_err(err, KX_E_PARAM, kOp, "null handle");
    if (ndst < 0 || ndst > kMaxPeers) return set_err(err, KX_E_PARAM, kOp, "ndst (0..8)");
    if (bytes == 0 || ndst == 0) return KX_OK;
    if (!src || !dsts || bytes % 16 || (reinterpret_cast<uintptr_t>(src) & 15))
        return set_err(err, KX_E_PARAM, kOp, "16-byte aligned source and size");
    PeerDsts d;
    std::memset(&d, 0, sizeof(d));
    d.n = ndst;
    for (int j = 0; j < ndst; ++j) {
        if (!dsts[j] || (reinterpret_cast<uintptr_t>(dsts[j]) & 15))
            return set_err(err, KX_E_PARAM, kOp, "16-byte aligned destinations");
        d.d[j] = static_cast<float4 *>(dsts[j]);
    }
    Handle *h = &hh->impl;
    DeviceGuard g(h->device);
    const uint64_t n16 = bytes / 16;
    int64_t blocks = (int64_t)((n16 + 255) / 256);
    if (blocks > 4LL * h->sm_count) blocks = 4LL * h->sm_count;
    peer_broadcast_kernel<<<(unsigned)blocks, 256, 0, h->stream>>>(static_cast<const float4 *>(src), d, n16);
    ++h->launches;
    cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) {
        h->cuda_fail(ce);
        return cuda_err(err, h, kOp);
    }
    return KX_OK;
}

int kx_copy_async(kx_handle *hh, void *dst, const void *src, uint64_t bytes, void *stream, kx_error *err) {
    static const char *kOp = "copy_async";
    if (!hh) return set_err(err, KX_E_PARAM, kOp, "null handle");
    if (bytes == 0) return KX_OK;
    if (!dst || !src) return set_err(err, KX_E_PARAM, kOp, "null pointer");
    Handle *h = &hh->impl;
    DeviceGuard g(h->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->stream;
    cudaError_t ce = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s);
    if (ce != cudaSuccess) {
        h->cuda_fail(ce);
        return cuda_err(err, h, kOp);
    }
    return KX_OK;
}

}  // extern "C"
