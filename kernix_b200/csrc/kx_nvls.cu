// Stores through an NVLink multicast address (NVLS): one multimem.st from
// this GPU reaches the same offset in the buffer of every GPU bound to the
// multicast object, the NVSwitch doing the fan-out.  Used to gather the
// output of a row-sharded GEMM: each rank stores its rows once and every
// rank's copy of C receives them.  The split-TF32 GEMM stores its epilogue
// this way directly; other kernels write locally and this copy follows.
#include "kx_internal.hpp"

using namespace kx;

namespace {

__device__ __forceinline__ void mc_st4(float *addr, float4 v) {
    asm volatile("multimem.st.weak.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ void mc_st1(float *addr, float v) {
    asm volatile("multimem.st.weak.global.b32 [%0], %1;" ::"l"(addr), "r"(__float_as_uint(v)) : "memory");
}

// n4 four-byte words from src to the multicast address; `vec` when both
// addresses are 16-byte aligned.  A system-scope fence orders the stores
// before whatever signals completion to the other GPUs.
__global__ void __launch_bounds__(256) mc_copy_kernel(const float *__restrict__ src, float *mc, uint64_t n4, int vec) {
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nth = (uint64_t)gridDim.x * blockDim.x;
    if (vec) {
        const uint64_t n16 = n4 / 4;
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        for (uint64_t i = tid; i < n16; i += nth) mc_st4(mc + 4 * i, __ldg(s4 + i));
        for (uint64_t i = n16 * 4 + tid; i < n4; i += nth) mc_st1(mc + i, __ldg(src + i));
    } else {
        for (uint64_t i = tid; i < n4; i += nth) mc_st1(mc + i, __ldg(src + i));
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

}  // namespace

namespace kx {

int mc_copy(Handle *h, const void *src, void *mc_dst, uint64_t bytes) {
    if (bytes == 0) return KX_OK;
    const uint64_t n4 = bytes / 4;
    const int vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(mc_dst)) & 15) == 0;
    int64_t blocks = (int64_t)((n4 / (vec ? 4 : 1) + 255) / 256);
    if (blocks > 4LL * h->sm_count) blocks = 4LL * h->sm_count;
    if (blocks < 1) blocks = 1;
    mc_copy_kernel<<<(unsigned)blocks, 256, 0, h->stream>>>(static_cast<const float *>(src), static_cast<float *>(mc_dst),
                                                           n4, vec);
    ++h->launches;
    cudaError_t ce = cudaGetLastError();
    return ce == cudaSuccess ? KX_OK : h->cuda_fail(ce);
}

}  // namespace kx

extern "C" int kx_multicast_store(kx_handle *hh, const void *src, void *mc_dst, uint64_t bytes, kx_error *err) {
    static const char *kOp = "multicast_store";
    if (!hh) return set_err(err, KX_E_PARAM, kOp, "null handle");
    if (bytes % 4 || (reinterpret_cast<uintptr_t>(src) & 3) || (reinterpret_cast<uintptr_t>(mc_dst) & 3))
        return set_err(err, KX_E_PARAM, kOp, "bytes and addresses must be multiples of 4");
    if (bytes && (!src || !mc_dst)) return set_err(err, KX_E_PARAM, kOp, "null pointer");
    Handle *h = &hh->impl;
    DeviceGuard g(h->device);
    int rc = mc_copy(h, src, mc_dst, bytes);
    return rc == KX_E_CUDA ? cuda_err(err, h, kOp) : rc;
}
