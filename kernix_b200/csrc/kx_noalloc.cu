// kx_matmul_splitk_f32_static: a split-K f32 GEMM that allocates nothing.
//
// Who needs it: callers that are not allowed to call cudaMalloc while they run.
// Two common cases are a host process whose device memory is owned up front by
// its own pool (serving stacks that reserve the GPU at start-up, so any further
// cudaMalloc fails or fragments the pool) and latency-critical loops, where
// cudaMalloc/cudaFree can synchronise the device and stall every other stream.
// The regular entry point (kx_matmul_f32) grows a per-handle workspace with
// cudaMalloc the first time a split-K product needs more partial-sum space, and
// creating a handle allocates too; this entry point takes no handle and keeps
// its partial sums in a fixed array that the CUDA module reserves when it is
// loaded.
//
// Limits and sharing:
//   * the array holds kStaticScratchBytes (16 MiB) = 4,194,304 f32 partial sums;
//     a product is accepted when two splits fit, i.e. M*N <= 2,097,152, and the
//     split count is lowered until splits*M*N fits;
//   * every GPU that loads this library keeps the array until the process exits;
//   * every call on a device shares the one array and it keeps the last call's
//     contents; calls whose kernels overlap on the GPU (different streams, or
//     different host threads) race on it -- serialise them on one stream;
//   * nothing in the array has to start at zero: each split writes its full
//     M x N partial before the reduction reads it, and a product with one
//     split (K under 128) stores C directly without reading the array.
// Set-up: the first call on a device, with that device current, resolves the
// array's device address once (cudaGetSymbolAddress, which also loads the
// module on that device); make that first call before any stream capture.
#include <atomic>
#include <cstring>
#include <mutex>

#include "gemm_simt.cuh"
#include "kx_host.hpp"

namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

// The scratch.  In host code this name is only a stand-in for the symbol; the
// device address comes from cudaGetSymbolAddress (see scratch_on_current_device).
static __device__ __align__(256) unsigned char g_splitk_scratch[kStaticScratchBytes];

std::atomic<void *> g_scratch_addr[kMaxDevices];
std::mutex g_setup_mutex;

// Device address of the array on the current device (set up once per device).
int scratch_on_current_device(float **out, kx_error *err) {
    int dev = -1;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess || dev < 0)
        return kx::set_err(err, KX_E_NO_DEVICE, "matmul_splitk_static", "no current CUDA device");
    if (dev >= kMaxDevices)
        return kx::set_err(err, KX_E_UNSUPPORTED, "matmul_splitk_static", "device ordinal above 63", dev);
    void *p = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        p = g_scratch_addr[dev].load(std::memory_order_relaxed);
        if (!p) {
            ce = cudaGetSymbolAddress(&p, g_splitk_scratch);
            if (ce != cudaSuccess || !p) {
                kx::set_err(err, KX_E_CUDA, "matmul_splitk_static", cudaGetErrorString(ce));
                if (err) err->cuda_error = (int)ce;
                return KX_E_CUDA;
            }
            g_scratch_addr[dev].store(p, std::memory_order_release);
        }
    }
    *out = static_cast<float *>(p);
    return KX_OK;
}

// Same 64x64x16 tile family as the regular split-K path.
struct StaticCfg : kx::TileCfg<float, 64, 64, 16, 4, 4, 2> {};

template <int AM, int BM>
cudaError_t launch(const kx::GemmParams<float> &p, cudaStream_t s) {
    const int64_t tiles = (int64_t)((p.M + StaticCfg::BM - 1) / StaticCfg::BM) * ((p.N + StaticCfg::BN - 1) / StaticCfg::BN);
    dim3 grid((unsigned)tiles, (unsigned)p.splits, 1);
    kx::gemm_simt_kernel<float, StaticCfg, AM, BM, false><<<grid, StaticCfg::NT, 0, s>>>(p);
    return cudaGetLastError();
}

template <int AM>
cudaError_t launch_b(const kx::GemmParams<float> &p, int bm, cudaStream_t s) {
    switch (bm) {
        case kx::kVecK: return launch<AM, kx::kVecK>(p, s);
        case kx::kVecMN: return launch<AM, kx::kVecMN>(p, s);
        case kx::kGatherMN: return launch<AM, kx::kGatherMN>(p, s);
        default: return launch<AM, kx::kGatherK>(p, s);
    }
}

int pick(const float *base, int64_t s_r, int64_t s_k, int64_t R, int64_t K) {
    const bool aligned = reinterpret_cast<uintptr_t>(base) % 16 == 0;
    if (aligned && s_k == 1 && K % 4 == 0 && s_r % 4 == 0) return kx::kVecK;
    if (aligned && s_r == 1 && R % 4 == 0 && s_k % 4 == 0) return kx::kVecMN;
    return (s_r < 0 ? -s_r : s_r) <= (s_k < 0 ? -s_k : s_k) ? kx::kGatherMN : kx::kGatherK;
}

}  // namespace

extern "C" int kx_matmul_splitk_f32_static(const kx_tensor *a, const kx_tensor *b, const kx_tensor *out,
                                           void *stream, kx_error *err) {
    static const char *kOp = "matmul_splitk_static";
    kx::Span sa, sb, so;
    int rc = kx::validate_tensor(a, 4, &sa, err);
    if (rc) return rc;
    rc = kx::validate_tensor(b, 4, &sb, err);
    if (rc) return rc;
    if (a->rank != 2 || b->rank != 2)
        return kx::set_err(err, KX_E_UNSUPPORTED, kOp, "rank-two operands only", a->rank, b->rank);
    kx::MatmulPlan pl;
    rc = kx::matmul_shape(a->dims, 2, b->dims, 2, &pl, err);
    if (rc) return rc;
    rc = kx::validate_tensor(out, 4, &so, err);
    if (rc) return rc;
    if (out->rank != 2 || out->dims[0] != pl.m || out->dims[1] != pl.n)
        return kx::set_err(err, KX_E_LAYOUT, kOp, "output shape mismatch", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
    if (!kx::is_c_contiguous(out))
        return kx::set_err(err, KX_E_LAYOUT, kOp, "output must be C-contiguous", KX_LAYOUT_OUTPUT_NOT_C_CONTIGUOUS);
    if (kx::spans_overlap(out->data, so, a->data, sa, 4) || kx::spans_overlap(out->data, so, b->data, sb, 4))
        return kx::set_err(err, KX_E_ALIAS, kOp, "output overlaps an input");
    const uint64_t m = pl.m, n = pl.n, k = pl.k;
    const uint64_t cap = kStaticScratchBytes / sizeof(float);
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX || m * n > cap / 2)
        return kx::set_err(err, KX_E_UNSUPPORTED, kOp,
                           "M*N above the static split-K scratch (2,097,152 outputs for two splits)", m * n, cap / 2);
    if (m == 0 || n == 0) return KX_OK;
    float *scratch = nullptr;
    rc = scratch_on_current_device(&scratch, err);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float *c = static_cast<float *>(out->data) + out->origin;
    if (k == 0) {
        cudaError_t ce = cudaMemsetAsync(c, 0, m * n * sizeof(float), s);
        if (ce != cudaSuccess) {
            kx::set_err(err, KX_E_CUDA, kOp, cudaGetErrorString(ce));
            if (err) err->cuda_error = (int)ce;
            return KX_E_CUDA;
        }
        return KX_OK;
    }

    kx::GemmParams<float> p;
    std::memset(&p, 0, sizeof(p));
    p.A = static_cast<const float *>(a->data) + a->origin;
    p.B = static_cast<const float *>(b->data) + b->origin;
    p.C = c;
    p.a_rs = m == 1 ? 0 : a->strides[0];
    p.a_cs = k == 1 ? 0 : a->strides[1];
    p.b_rs = k == 1 ? 0 : b->strides[0];
    p.b_cs = n == 1 ? 0 : b->strides[1];
    p.c_rs = (int64_t)n;
    p.c_cs = 1;
    p.M = (int)m;
    p.N = (int)n;
    p.K = (int)k;
    p.nbatch = 1;
    // Splits: enough CTAs for a full machine (~2 per SM on 148 SMs), at least
    // four k-tiles per split, and splits * M * N within the array.  A short K
    // (under 128) ends with one split: the GEMM kernel then stores C itself
    // and neither the array nor the reduction is used.
    const int64_t tiles = (int64_t)((m + 63) / 64) * ((n + 63) / 64);
    int64_t splits = (296 + tiles - 1) / tiles;
    const int64_t by_k = (int64_t)k / (4 * StaticCfg::BK);
    if (splits > by_k) splits = by_k;
    const int64_t by_cap = (int64_t)(cap / (m * n));
    if (splits > by_cap) splits = by_cap;
    if (splits < 1) splits = 1;
    int64_t kps = ((int64_t)k + splits - 1) / splits;
    kps = (kps + StaticCfg::BK - 1) / StaticCfg::BK * StaticCfg::BK;
    splits = ((int64_t)k + kps - 1) / kps;   // rounding kps up can only lower it
    if (splits < 1) splits = 1;
    p.splits = (int)splits;
    p.k_per_split = (int)kps;
    p.ws = scratch;
    const int am = pick(p.A, p.a_rs, p.a_cs, p.M, p.K);
    const int bm = pick(p.B, p.b_cs, p.b_rs, p.N, p.K);
    cudaError_t ce;
    switch (am) {
        case kx::kVecK: ce = launch_b<kx::kVecK>(p, bm, s); break;
        case kx::kVecMN: ce = launch_b<kx::kVecMN>(p, bm, s); break;
        case kx::kGatherMN: ce = launch_b<kx::kGatherMN>(p, bm, s); break;
        default: ce = launch_b<kx::kGatherK>(p, bm, s); break;
    }
    if (ce == cudaSuccess && p.splits > 1) {
        const int64_t total = (int64_t)m * n;
        int64_t blocks = (total + 255) / 256;
        if (blocks > 1184) blocks = 1184;
        kx::splitk_reduce_kernel<float><<<(unsigned)blocks, 256, 0, s>>>(p);
        ce = cudaGetLastError();
    }
    if (ce != cudaSuccess) {
        kx::set_err(err, KX_E_CUDA, kOp, cudaGetErrorString(ce));
        if (err) err->cuda_error = (int)ce;
        return KX_E_CUDA;
    }
    return KX_OK;
}
