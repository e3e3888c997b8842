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
