// C-ABI entry points: handles, device buffers, shape planning, matmul and the
// MatmulElement-style host-buffer hooks.  All validation happens on the host
// before any device work, so a rejected call writes nothing.
#include <algorithm>
#include <cstring>
#include <new>

#include "gemm_simt.cuh"
#include "kx_internal.hpp"
#include "tc_common.cuh"

using namespace kx;

namespace {


template <typename T> constexpr uint32_t ES = (uint32_t)sizeof(T);

// Fill the batch geometry and matrix strides of a GEMM from validated
// descriptors and the matmul plan (linalg.rs:94-116 shape roles; batch_index
// linalg.rs:219-232 broadcast mapping expressed as zero strides).
template <typename T>
int build_params(const MatmulPlan &pl, const kx_tensor *a, const T *a_ptr, const kx_tensor *b, const T *b_ptr,
                 const int64_t *c_strides, T *c_ptr, GemmParams<T> *p, kx_error *err) {
    if (pl.m > INT32_MAX || pl.n > INT32_MAX || pl.k > INT32_MAX)
        return set_err(err, KX_E_UNSUPPORTED, "matmul", "matrix extent above 2^31-1");
    std::memset(p, 0, sizeof(*p));
    p->A = a_ptr;
    p->B = b_ptr;
    p->C = c_ptr;
    p->M = (int)pl.m;
    p->N = (int)pl.n;
    p->K = (int)pl.k;
    const uint32_t ar = a->rank, br = b->rank;
    if (pl.a_vector) {
        p->a_rs = 0;
        p->a_cs = a->strides[0];
    } else {
        p->a_rs = a->dims[ar - 2] == 1 ? 0 : a->strides[ar - 2];
        p->a_cs = a->dims[ar - 1] == 1 ? 0 : a->strides[ar - 1];
    }
    if (pl.b_vector) {
        p->b_rs = b->strides[0];
        p->b_cs = 0;
    } else {
        p->b_rs = b->dims[br - 2] == 1 ? 0 : b->strides[br - 2];
        p->b_cs = b->dims[br - 1] == 1 ? 0 : b->strides[br - 1];
    }
    const uint32_t orank = pl.out_rank;
    if (!pl.a_vector && !pl.b_vector) {
        p->c_rs = c_strides[orank - 2];
        p->c_cs = c_strides[orank - 1];
    } else if (pl.a_vector && !pl.b_vector) {
        p->c_rs = 0;
        p->c_cs = c_strides[orank - 1];
    } else if (!pl.a_vector && pl.b_vector) {
        p->c_rs = c_strides[orank - 1];
        p->c_cs = 0;
    }
    if (p->M == 1) p->c_rs = 0;
    if (p->N == 1) p->c_cs = 0;
    // Batch: keep only non-singleton output batch axes.
    int nd = 0;
    int64_t nbatch = 1;
    for (uint32_t d = 0; d < pl.batch_rank; ++d) {
        const uint64_t dim = pl.batch[d];
        if (dim == 1) continue;
        if (nd == kMaxBatchDims) return set_err(err, KX_E_UNSUPPORTED, "matmul", "too many batch axes");
        const int ad = (int)d - (int)(pl.batch_rank - pl.a_batch_rank);
        const int bd = (int)d - (int)(pl.batch_rank - pl.b_batch_rank);
        p->batch.dims[nd] = (int64_t)dim;
        p->batch.a_str[nd] = (ad >= 0 && a->dims[ad] != 1) ? a->strides[ad] : 0;
        p->batch.b_str[nd] = (bd >= 0 && b->dims[bd] != 1) ? b->strides[bd] : 0;
        p->batch.c_str[nd] = c_strides[d];
        nbatch *= (int64_t)dim;
        ++nd;
    }
    // Merge adjacent batch axes that every operand walks as one (stride of the
    // outer axis = stride x extent of the inner one): [16, 32] heads become a
    // single axis of 512 with the same element offsets.
    int w = 0;
    for (int d = 0; d < nd; ++d) {
        if (w > 0) {
            BatchGeom &g = p->batch;
            const int64_t e = g.dims[d];
            if (g.a_str[w - 1] == g.a_str[d] * e && g.b_str[w - 1] == g.b_str[d] * e &&
                g.c_str[w - 1] == g.c_str[d] * e) {
                g.dims[w - 1] *= e;
                g.a_str[w - 1] = g.a_str[d];
                g.b_str[w - 1] = g.b_str[d];
                g.c_str[w - 1] = g.c_str[d];
                continue;
            }
        }
        p->batch.dims[w] = p->batch.dims[d];
        p->batch.a_str[w] = p->batch.a_str[d];
        p->batch.b_str[w] = p->batch.b_str[d];
        p->batch.c_str[w] = p->batch.c_str[d];
        ++w;
    }
    p->batch.ndims = w;
    p->nbatch = nbatch;
    p->splits = 1;
    p->k_per_split = p->K;
    return KX_OK;
}

template <typename T>
int matmul_device(kx_handle *hh, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out, kx_error *err,
                  void *out_mc = nullptr) {
    if (!hh) return set_err(err, KX_E_PARAM, "matmul", "null handle");
    Handle *h = &hh->impl;
    Span sa, sb, so;
    int rc = validate_tensor(a, ES<T>, &sa, err);
    if (rc) return rc;
    rc = validate_tensor(b, ES<T>, &sb, err);
    if (rc) return rc;
    MatmulPlan pl;
    rc = matmul_shape(a->dims, a->rank, b->dims, b->rank, &pl, err);
    if (rc) return rc;
    rc = validate_tensor(out, ES<T>, &so, err);
    if (rc) return rc;
    if (out->rank != pl.out_rank)
        return set_err(err, KX_E_LAYOUT, "matmul", "output shape mismatch", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
    for (uint32_t i = 0; i < pl.out_rank; ++i)
        if (out->dims[i] != pl.out_dims[i])
            return set_err(err, KX_E_LAYOUT, "matmul", "output shape mismatch", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
    if (!is_c_contiguous(out))
        return set_err(err, KX_E_LAYOUT, "matmul", "output must be C-contiguous", KX_LAYOUT_OUTPUT_NOT_C_CONTIGUOUS);
    if (spans_overlap(out->data, so, a->data, sa, ES<T>) || spans_overlap(out->data, so, b->data, sb, ES<T>))
        return set_err(err, KX_E_ALIAS, "matmul", "output overlaps an input");
    const uint64_t total = numel(pl.out_dims, pl.out_rank);
    if (total == 0) return KX_OK;
    DeviceGuard g(h->device);
    if (!g.ok) return set_err(err, KX_E_NO_DEVICE, "matmul", "cannot select device");
    T *c_ptr = static_cast<T *>(out->data) + out->origin;
    T *mc_ptr = out_mc ? static_cast<T *>(out_mc) + out->origin : nullptr;
    if (pl.k == 0) {
        cudaError_t ce = cudaMemsetAsync(c_ptr, 0, total * sizeof(T), h->stream);
        if (ce != cudaSuccess) {
            h->cuda_fail(ce);
            return cuda_err(err, h, "matmul");
        }
        h->last_kernel = "memset";
        rc = mc_ptr ? mc_copy(h, c_ptr, mc_ptr, total * sizeof(T)) : KX_OK;
        return rc == KX_E_CUDA ? cuda_err(err, h, "matmul") : rc;
    }
    GemmParams<T> p;
    rc = build_params<T>(pl, a, static_cast<const T *>(a->data) + a->origin, b,
                         static_cast<const T *>(b->data) + b->origin, out->strides, c_ptr, &p, err);
    if (rc) return rc;
    p.C_mc = mc_ptr;
    const char *name = "none";
    rc = run_gemm<T>(h, p, &name);
    h->last_kernel = name;
    if (rc == KX_E_CUDA) return cuda_err(err, h, "matmul");
    if (rc) return set_err(err, rc, "matmul", "launch");
    return KX_OK;
}

// Pipelined host-buffer GEMM for A with disjoint rows (positive row stride
// larger than the row's reach): B goes up first, then A in row pieces on a
// copy stream; piece i multiplies while piece i+1 uploads and piece i-1's rows
// of C download on a third stream, so both PCIe directions and the GEMM
// overlap.  Same staging layout as the one-shot path.
template <typename T>
int hook_gemm_pipelined(Handle *h, const T *a_host, uint64_t a_start, uint64_t a_count, uint64_t a_origin,
                        int64_t a_rs, int64_t a_cs, const T *b_host, uint64_t b_start, uint64_t b_count,
                        uint64_t b_origin, int64_t b_rs, int64_t b_cs, T *out, uint64_t m, uint64_t k, uint64_t n,
                        T *da, T *db, T *dc, int pieces) {
    cudaError_t ce = cudaSuccess;
    if (!h->h2d) ce = cudaStreamCreateWithFlags(&h->h2d, cudaStreamNonBlocking);
    if (ce == cudaSuccess && !h->d2h) ce = cudaStreamCreateWithFlags(&h->d2h, cudaStreamNonBlocking);
    for (int i = 0; ce == cudaSuccess && i < 3 * pieces + 2; ++i)
        if (!h->ev[i]) ce = cudaEventCreateWithFlags(&h->ev[i], cudaEventDisableTiming);
    if (ce != cudaSuccess) return h->cuda_fail(ce);
    cudaEvent_t start = h->ev[0], b_up = h->ev[1];
    cudaEvent_t *a_up = h->ev + 2, *c_done = h->ev + 2 + pieces, *c_down = h->ev + 2 + 2 * pieces;
    const uint64_t rows = (m + pieces - 1) / pieces;
    // staging is free once earlier work on the handle's stream is done
    ce = cudaEventRecord(start, h->stream);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(h->h2d, start, 0);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(h->d2h, start, 0);
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(db, b_host + b_start, b_count * sizeof(T), cudaMemcpyHostToDevice, h->h2d);
    if (ce == cudaSuccess) ce = cudaEventRecord(b_up, h->h2d);
    for (int i = 0; ce == cudaSuccess && i < pieces; ++i) {
        const uint64_t r0 = i * rows, r1 = std::min<uint64_t>(m, r0 + rows);
        if (r0 >= r1) break;
        const uint64_t s0 = a_origin + r0 * (uint64_t)a_rs;
        const uint64_t s1 = a_origin + (r1 - 1) * (uint64_t)a_rs + (k - 1) * (uint64_t)a_cs + 1;
        ce = cudaMemcpyAsync(da + (s0 - a_start), a_host + s0, (s1 - s0) * sizeof(T), cudaMemcpyHostToDevice,
                             h->h2d);
        if (ce == cudaSuccess) ce = cudaEventRecord(a_up[i], h->h2d);
    }
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(h->stream, b_up, 0);
    if (ce != cudaSuccess) return h->cuda_fail(ce);
    int rc = KX_OK;
    const char *name = "none";
    int last = -1;
    for (int i = 0; i < pieces; ++i) {
        const uint64_t r0 = i * rows, r1 = std::min<uint64_t>(m, r0 + rows);
        if (r0 >= r1) break;
        ce = cudaStreamWaitEvent(h->stream, a_up[i], 0);
        if (ce != cudaSuccess) return h->cuda_fail(ce);
        GemmParams<T> p;
        std::memset(&p, 0, sizeof(p));
        p.A = da + (a_origin - a_start) + r0 * (uint64_t)a_rs;
        p.B = db + (b_origin - b_start);
        p.C = dc + r0 * n;
        p.a_rs = (r1 - r0) == 1 ? 0 : a_rs;
        p.a_cs = k == 1 ? 0 : a_cs;
        p.b_rs = k == 1 ? 0 : b_rs;
        p.b_cs = n == 1 ? 0 : b_cs;
        p.c_rs = (int64_t)n;
        p.c_cs = 1;
        p.M = (int)(r1 - r0);
        p.N = (int)n;
        p.K = (int)k;
        p.nbatch = 1;
        p.splits = 1;
        p.k_per_split = (int)k;
        rc = run_gemm<T>(h, p, &name);
        if (rc) break;
        ce = cudaEventRecord(c_done[i], h->stream);
        if (ce == cudaSuccess) ce = cudaStreamWaitEvent(h->d2h, c_done[i], 0);
        if (ce == cudaSuccess)
            ce = cudaMemcpyAsync(out + r0 * n, dc + r0 * n, (r1 - r0) * n * sizeof(T), cudaMemcpyDeviceToHost,
                                 h->d2h);
        if (ce == cudaSuccess) ce = cudaEventRecord(c_down[i], h->d2h);
        if (ce != cudaSuccess) return h->cuda_fail(ce);
        last = i;
    }
    h->last_kernel = name;
    // the call returns once the last rows are on the host; later work on the
    // handle's stream is ordered after the downloads
    if (last >= 0) {
        ce = cudaStreamWaitEvent(h->stream, c_down[last], 0);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(h->d2h);
    }
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(h->stream);
    if (ce != cudaSuccess) return h->cuda_fail(ce);
    return rc;
}

// Host-buffer GEMM used by both hooks: copy the reachable spans to device
// staging, run, copy the C-order product back.  a_start/b_start are the first
// reachable elements; the GEMM reads A at a_dev + (origin - start).
template <typename T>
int hook_gemm(Handle *h, const T *a_host, uint64_t a_start, uint64_t a_count, uint64_t a_origin, int64_t a_rs,
              int64_t a_cs, const T *b_host, uint64_t b_start, uint64_t b_count, uint64_t b_origin, int64_t b_rs,
              int64_t b_cs, T *out, uint64_t m, uint64_t k, uint64_t n) {
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return KX_DECLINED;
    DeviceGuard g(h->device);
    if (!g.ok) return KX_E_NO_DEVICE;
    const uint64_t out_bytes = m * n * sizeof(T);
    int rc = h->grow(&h->stage[0], &h->stage_bytes[0], a_count * sizeof(T));
    if (!rc) rc = h->grow(&h->stage[1], &h->stage_bytes[1], b_count * sizeof(T));
    if (!rc) rc = h->grow(&h->stage[2], &h->stage_bytes[2], out_bytes);
    if (rc) return rc;
    T *da = static_cast<T *>(h->stage[0]);
    T *db = static_cast<T *>(h->stage[1]);
    T *dc = static_cast<T *>(h->stage[2]);
    // Large products with disjoint A rows: overlap the transfers with the GEMM.
    const uint64_t flops = 2 * m * n * k;
    const bool disjoint_rows = a_rs > 0 && a_cs >= 0 && (uint64_t)a_cs * (k - 1) < (uint64_t)a_rs;
    if (disjoint_rows && m >= 1024 && flops >= (1ull << 34)) {
        const int pieces = (int)std::min<uint64_t>(8, m / 512);
        return hook_gemm_pipelined<T>(h, a_host, a_start, a_count, a_origin, a_rs, a_cs, b_host, b_start, b_count,
                                      b_origin, b_rs, b_cs, out, m, k, n, da, db, dc, pieces);
    }
    cudaError_t ce = cudaMemcpyAsync(da, a_host + a_start, a_count * sizeof(T), cudaMemcpyHostToDevice, h->stream);
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(db, b_host + b_start, b_count * sizeof(T), cudaMemcpyHostToDevice, h->stream);
    if (ce != cudaSuccess) return h->cuda_fail(ce);
    GemmParams<T> p;
    std::memset(&p, 0, sizeof(p));
    p.A = da + (a_origin - a_start);
    p.B = db + (b_origin - b_start);
    p.C = dc;
    p.a_rs = m == 1 ? 0 : a_rs;
    p.a_cs = k == 1 ? 0 : a_cs;
    p.b_rs = k == 1 ? 0 : b_rs;
    p.b_cs = n == 1 ? 0 : b_cs;
    p.c_rs = (int64_t)n;
    p.c_cs = 1;
    p.M = (int)m;
    p.N = (int)n;
    p.K = (int)k;
    p.nbatch = 1;
    p.splits = 1;
    p.k_per_split = (int)k;
    const char *name = "none";
    rc = run_gemm<T>(h, p, &name);
    h->last_kernel = name;
    if (rc) return rc;
    ce = cudaMemcpyAsync(out, dc, out_bytes, cudaMemcpyDeviceToHost, h->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(h->stream);
    if (ce != cudaSuccess) return h->cuda_fail(ce);
    return KX_OK;
}

inline bool mul_ok(uint64_t a, uint64_t b, uint64_t *r) { return !__builtin_mul_overflow(a, b, r); }

// try_dense_matmul (matmul_element.rs:139-251): exact extents or decline.
template <typename T>
int try_dense(kx_handle *hh, const T *a, uint64_t a_len, const T *b, uint64_t b_len, T *out, uint64_t out_len,
              uint64_t m, uint64_t k, uint64_t n) {
    // Extents first (matmul_element.rs:147-159): a mismatch declines before
    // anything else, and empty or k == 0 products need no device.
    uint64_t mk, kn, mn;
    if (!mul_ok(m, k, &mk) || mk != a_len || !mul_ok(k, n, &kn) || kn != b_len || !mul_ok(m, n, &mn) ||
        mn != out_len)
        return KX_DECLINED;
    if (m == 0 || n == 0) return KX_OK;
    if (k == 0) {
        for (uint64_t i = 0; i < mn; ++i) out[i] = T(0);
        return KX_OK;
    }
    if (k > kIsizeMax || n > kIsizeMax) return KX_DECLINED;
    if (!hh || !a || !b || !out) return KX_DECLINED;
    return hook_gemm<T>(&hh->impl, a, 0, mk, 0, (int64_t)k, 1, b, 0, kn, 0, (int64_t)n, 1, out, m, k, n);
}

int matrix_validate(const kx_matrix *mtx, uint32_t es, Span *s, kx_error *err) {
    if (!mtx) return set_err(err, KX_E_PARAM, "MatrixInput", "null descriptor");
    int rc = validate_dims(mtx->dims, 2, err);
    if (rc) return rc;
    rc = span_of(mtx->dims, mtx->strides, 2, mtx->origin, s, err);
    if (rc) return rc;
    rc = validate_storage(*s, mtx->storage_len, es, err);
    if (rc) return rc;
    if (!s->empty && !mtx->data) return set_err(err, KX_E_PARAM, "MatrixInput", "null data pointer");
    return KX_OK;
}

// try_strided_matmul (matmul_element.rs:53-138).
template <typename T>
int try_strided(kx_handle *hh, const kx_matrix *a, const kx_matrix *b, T *out, uint64_t out_len) {
    if (!a || !b) return KX_DECLINED;
    Span sa, sb;
    int rc = matrix_validate(a, ES<T>, &sa, nullptr);
    if (rc) return rc;
    rc = matrix_validate(b, ES<T>, &sb, nullptr);
    if (rc) return rc;
    const uint64_t m = a->dims[0], k = a->dims[1], n = b->dims[1];
    uint64_t mn;
    if (k != b->dims[0] || !mul_ok(m, n, &mn) || mn != out_len) return KX_DECLINED;
    if (m == 0 || n == 0) return KX_OK;
    if (k == 0) {
        for (uint64_t i = 0; i < mn; ++i) out[i] = T(0);
        return KX_OK;
    }
    if (n > kIsizeMax || !out || !hh) return KX_DECLINED;
    // MatrixInput::new normalises singleton strides to zero.
    const int64_t a_rs = m <= 1 ? 0 : a->strides[0], a_cs = k <= 1 ? 0 : a->strides[1];
    const int64_t b_rs = k <= 1 ? 0 : b->strides[0], b_cs = n <= 1 ? 0 : b->strides[1];
    return hook_gemm<T>(&hh->impl, static_cast<const T *>(a->data), sa.start, sa.end - sa.start, a->origin, a_rs,
                        a_cs, static_cast<const T *>(b->data), sb.start, sb.end - sb.start, b->origin, b_rs, b_cs,
                        out, m, k, n);
}

}  // namespace

extern "C" {

int kx_abi_version(void) { return KX_ABI_VERSION; }

int kx_device_count(int *count) {
    int c = 0;
    if (cudaGetDeviceCount(&c) != cudaSuccess) c = 0;
    if (count) *count = c;
    return KX_OK;
}

int kx_create(int device, kx_handle **out, kx_error *err) {
    if (!out) return set_err(err, KX_E_PARAM, "kx_create", "null output");
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)
        return set_err(err, KX_E_NO_DEVICE, "kx_create", "no CUDA device");
    if (device < 0 || device >= count) return set_err(err, KX_E_NO_DEVICE, "kx_create", "device ordinal out of range");
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
        return set_err(err, KX_E_NO_DEVICE, "kx_create", "cannot query device");
    if (prop.major != 10)
        return set_err(err, KX_E_NO_DEVICE, "kx_create", "device is not sm_100 (B200)", prop.major, prop.minor);
    kx_handle *hh = new (std::nothrow) kx_handle();
    if (!hh) return set_err(err, KX_E_PARAM, "kx_create", "out of host memory");
    hh->impl.device = device;
    hh->impl.sm_count = prop.multiProcessorCount;
    DeviceGuard g(device);
    cudaError_t ce = cudaMalloc(&hh->impl.flags, Handle::kFlagWords * sizeof(uint32_t));
    if (ce == cudaSuccess) ce = cudaMemset(hh->impl.flags, 0, Handle::kFlagWords * sizeof(uint32_t));
    if (ce != cudaSuccess) {
        delete hh;
        return set_err(err, KX_E_CUDA, "kx_create", cudaGetErrorString(ce));
    }
    *out = hh;
    return KX_OK;
}

int kx_destroy(kx_handle *hh) {
    if (!hh) return KX_OK;
    Handle &h = hh->impl;
    {
        DeviceGuard g(h.device);
        if (h.stream) cudaStreamSynchronize(h.stream);
        else cudaDeviceSynchronize();
        if (h.h2d) cudaStreamSynchronize(h.h2d);
        if (h.d2h) cudaStreamSynchronize(h.d2h);
        cudaFree(h.ws);
        for (auto &s : h.stage) cudaFree(s);
        cudaFree(h.attn);
        cudaFree(h.bwd);
        cudaFree(h.perm);
        cudaFree(h.flags);
        for (auto &e : h.ev)
            if (e) cudaEventDestroy(e);
        for (int r = 0; r < Handle::kMaxWorld; ++r) {
            if (h.peer_stream[r]) {
                cudaStreamSynchronize(h.peer_stream[r]);
                cudaStreamDestroy(h.peer_stream[r]);
            }
            if (h.peer_done[r]) cudaEventDestroy(h.peer_done[r]);
        }
        if (h.peer_ready) cudaEventDestroy(h.peer_ready);
        cudaFree(h.tail);
        if (h.h2d) cudaStreamDestroy(h.h2d);
        if (h.d2h) cudaStreamDestroy(h.d2h);
    }
    delete hh;
    return KX_OK;
}

int kx_set_stream(kx_handle *hh, void *stream) {
    if (!hh) return KX_E_PARAM;
    hh->impl.stream = static_cast<cudaStream_t>(stream);
    return KX_OK;
}

int kx_set_f32_variant(kx_handle *hh, int variant) {
    if (!hh || variant < KX_F32_AUTO || variant > KX_F32_3XTF32_1SM) return KX_E_PARAM;
    hh->impl.f32_variant = variant;
    return KX_OK;
}

int kx_set_f64_variant(kx_handle *hh, int variant) {
    if (!hh || variant < KX_F64_AUTO || variant > KX_F64_DMMA) return KX_E_PARAM;
    hh->impl.f64_variant = variant;
    return KX_OK;
}

int kx_set_ordered_matmul(kx_handle *hh, int ordered) {
    if (!hh) return KX_E_PARAM;
    hh->impl.ordered = ordered != 0;
    return KX_OK;
}

int kx_ordered_matmul(const kx_handle *hh) { return hh && hh->impl.ordered ? 1 : 0; }

int kx_diag_expire_next_gemm(kx_handle *hh, uint64_t wait_ns) {
    if (!hh) return KX_E_PARAM;
    if (wait_ns < 1000000ull || wait_ns > tc::WAIT_NS) return KX_E_PARAM;
    hh->impl.diag_wait_ns = wait_ns;
    return KX_OK;
}

void kx_cuda_config_default(kx_cuda_config *cfg) {
    if (!cfg) return;
    std::memset(cfg, 0, sizeof(*cfg));
    cfg->f32_variant = KX_F32_AUTO;
    cfg->f64_variant = KX_F64_AUTO;
}

int kx_context_create(const kx_cuda_config *cfg, kx_handle **out, kx_error *err) {
    static const char *kOp = "Context::new";
    if (!out) return set_err(err, KX_E_PARAM, kOp, "null output");
    *out = nullptr;
    if (!cfg) return set_err(err, KX_E_PARAM, kOp, "null configuration");
    if (cfg->device < 0) return set_err(err, KX_E_PARAM, kOp, "cuda.device must be non-negative");
    if (cfg->f32_variant < KX_F32_AUTO || cfg->f32_variant > KX_F32_3XTF32_1SM)
        return set_err(err, KX_E_PARAM, kOp, "cuda.f32_variant is not a kernel family");
    if (cfg->f64_variant < KX_F64_AUTO || cfg->f64_variant > KX_F64_DMMA)
        return set_err(err, KX_E_PARAM, kOp, "cuda.f64_variant is not a kernel family");
    if (cfg->ordered_matmul != 0 && cfg->ordered_matmul != 1)
        return set_err(err, KX_E_PARAM, kOp, "cuda.ordered_matmul must be 0 or 1");
    kx_handle *hh = nullptr;
    int rc = kx_create(cfg->device, &hh, err);
    if (rc) return rc;
    Handle &h = hh->impl;
    h.f32_variant = cfg->f32_variant;
    h.f64_variant = cfg->f64_variant;
    h.ordered = cfg->ordered_matmul != 0;
    if (cfg->workspace_bytes) {
        DeviceGuard g(h.device);
        if (h.grow(&h.ws, &h.ws_bytes, cfg->workspace_bytes)) {
            rc = cuda_err(err, &h, kOp);
            kx_destroy(hh);
            return rc;
        }
    }
    *out = hh;
    return KX_OK;
}

int kx_handle_config(const kx_handle *hh, kx_cuda_config *out) {
    if (!hh || !out) return KX_E_PARAM;
    const Handle &h = hh->impl;
    std::memset(out, 0, sizeof(*out));
    out->device = h.device;
    out->f32_variant = h.f32_variant;
    out->f64_variant = h.f64_variant;
    out->ordered_matmul = h.ordered ? 1 : 0;
    out->workspace_bytes = h.ws_bytes;
    return KX_OK;
}

int kx_synchronize(kx_handle *hh, kx_error *err) {
    if (!hh) return set_err(err, KX_E_PARAM, "synchronize", "null handle");
    DeviceGuard g(hh->impl.device);
    cudaError_t ce = cudaStreamSynchronize(hh->impl.stream);
    if (ce != cudaSuccess) {
        hh->impl.cuda_fail(ce);
        return cuda_err(err, &hh->impl, "synchronize");
    }
    // Device status word: a kernel whose bounded wait expired leaves a flag
    // here instead of hanging; report it once and clear it.
    uint32_t status = 0;
    ce = cudaMemcpy(&status, hh->impl.flags + kStatusWord, sizeof(status), cudaMemcpyDeviceToHost);
    if (ce != cudaSuccess) {
        hh->impl.cuda_fail(ce);
        return cuda_err(err, &hh->impl, "synchronize");
    }
    if (status) {
        cudaMemset(hh->impl.flags + kStatusWord, 0, sizeof(status));
        return set_err(err, KX_E_TIMEOUT, "synchronize", "a device-side wait expired", status);
    }
    return KX_OK;
}

int kx_alloc(kx_handle *hh, uint64_t bytes, void **out, kx_error *err) {
    if (!hh || !out) return set_err(err, KX_E_PARAM, "alloc", "null argument");
    DeviceGuard g(hh->impl.device);
    cudaError_t ce = cudaMalloc(out, bytes ? bytes : 1);
    if (ce != cudaSuccess) {
        *out = nullptr;
        hh->impl.cuda_fail(ce);
        return cuda_err(err, &hh->impl, "alloc");
    }
    return KX_OK;
}

int kx_free(kx_handle *hh, void *ptr) {
    if (!hh) return KX_E_PARAM;
    DeviceGuard g(hh->impl.device);
    return cudaFree(ptr) == cudaSuccess ? KX_OK : KX_E_CUDA;
}

int kx_upload(kx_handle *hh, void *dst, const void *src, uint64_t bytes, kx_error *err) {
    if (!hh) return set_err(err, KX_E_PARAM, "upload", "null handle");
    DeviceGuard g(hh->impl.device);
    cudaError_t ce = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, hh->impl.stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(hh->impl.stream);
    if (ce != cudaSuccess) {
        hh->impl.cuda_fail(ce);
        return cuda_err(err, &hh->impl, "upload");
    }
    return KX_OK;
}

int kx_download(kx_handle *hh, void *dst, const void *src, uint64_t bytes, kx_error *err) {
    if (!hh) return set_err(err, KX_E_PARAM, "download", "null handle");
    DeviceGuard g(hh->impl.device);
    cudaError_t ce = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, hh->impl.stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(hh->impl.stream);
    if (ce != cudaSuccess) {
        hh->impl.cuda_fail(ce);
        return cuda_err(err, &hh->impl, "download");
    }
    return KX_OK;
}

int kx_matmul_shape(const uint64_t *a_dims, uint32_t a_rank, const uint64_t *b_dims, uint32_t b_rank,
                    uint32_t *out_rank, uint64_t *out_dims, kx_error *err) {
    if ((a_rank && !a_dims) || (b_rank && !b_dims) || !out_rank || !out_dims)
        return set_err(err, KX_E_PARAM, "matmul", "null argument");
    MatmulPlan pl;
    int rc = matmul_shape(a_dims, a_rank, b_dims, b_rank, &pl, err);
    if (rc) return rc;
    *out_rank = pl.out_rank;
    for (uint32_t i = 0; i < pl.out_rank; ++i) out_dims[i] = pl.out_dims[i];
    return KX_OK;
}

int kx_conv2d_shape(const uint64_t *input_dims, uint32_t input_rank, const uint64_t *weight_dims,
                    uint32_t weight_rank, const kx_conv2d_options *options, uint64_t *out_dims, kx_error *err) {
    if ((input_rank && !input_dims) || (weight_rank && !weight_dims) || !out_dims)
        return set_err(err, KX_E_PARAM, "conv2d", "null argument");
    if (input_rank > KX_MAX_RANK || weight_rank > KX_MAX_RANK)
        return set_err(err, KX_E_EXACT_RANK, "conv2d", "rank", 4, input_rank > 4 ? input_rank : weight_rank);
    return conv_shape(input_dims, input_rank, weight_dims, weight_rank, options, out_dims, err);
}

int kx_validate_tensor(const kx_tensor *t, uint32_t elem_bytes, kx_error *err) {
    if (elem_bytes == 0) return set_err(err, KX_E_PARAM, "layout", "zero-sized element type");
    return validate_tensor(t, elem_bytes, nullptr, err);
}

int kx_matrix_validate(const kx_matrix *m, uint32_t elem_bytes, kx_error *err) {
    if (elem_bytes == 0) return set_err(err, KX_E_PARAM, "layout", "zero-sized element type");
    Span s;
    return matrix_validate(m, elem_bytes, &s, err);
}

int kx_matmul_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out, kx_error *err) {
    return matmul_device<float>(h, a, b, out, err);
}
int kx_matmul_f64(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out, kx_error *err) {
    return matmul_device<double>(h, a, b, out, err);
}
int kx_matmul_replicated_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out,
                             void *out_mc, kx_error *err) {
    if (!out_mc) return set_err(err, KX_E_PARAM, "matmul_replicated", "null multicast address");
    return matmul_device<float>(h, a, b, out, err, out_mc);
}
int kx_matmul_replicated_f64(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out,
                             void *out_mc, kx_error *err) {
    if (!out_mc) return set_err(err, KX_E_PARAM, "matmul_replicated", "null multicast address");
    return matmul_device<double>(h, a, b, out, err, out_mc);
}

int kx_try_dense_matmul_f32(kx_handle *h, const float *a, uint64_t a_len, const float *b, uint64_t b_len, float *out,
                            uint64_t out_len, uint64_t m, uint64_t k, uint64_t n) {
    return try_dense<float>(h, a, a_len, b, b_len, out, out_len, m, k, n);
}
int kx_try_dense_matmul_f64(kx_handle *h, const double *a, uint64_t a_len, const double *b, uint64_t b_len,
                            double *out, uint64_t out_len, uint64_t m, uint64_t k, uint64_t n) {
    return try_dense<double>(h, a, a_len, b, b_len, out, out_len, m, k, n);
}
int kx_try_strided_matmul_f32(kx_handle *h, const kx_matrix *a, const kx_matrix *b, float *out, uint64_t out_len) {
    return try_strided<float>(h, a, b, out, out_len);
}
int kx_try_strided_matmul_f64(kx_handle *h, const kx_matrix *a, const kx_matrix *b, double *out, uint64_t out_len) {
    return try_strided<double>(h, a, b, out, out_len);
}

uint64_t kx_launch_count(const kx_handle *h) { return h ? h->impl.launches : 0; }
const char *kx_last_kernel(const kx_handle *h) { return h ? h->impl.last_kernel : "none"; }

const char *kx_status_name(int status) {
    switch (status) {
        case KX_OK: return "KX_OK";
        case KX_DECLINED: return "KX_DECLINED";
        case KX_E_INVALID_RANK: return "KX_E_INVALID_RANK";
        case KX_E_CONTRACT: return "KX_E_CONTRACT";
        case KX_E_BROADCAST: return "KX_E_BROADCAST";
        case KX_E_SHAPE_OVERFLOW: return "KX_E_SHAPE_OVERFLOW";
        case KX_E_DIM_OVERFLOW: return "KX_E_DIM_OVERFLOW";
        case KX_E_LAYOUT: return "KX_E_LAYOUT";
        case KX_E_PARAM: return "KX_E_PARAM";
        case KX_E_EXACT_RANK: return "KX_E_EXACT_RANK";
        case KX_E_NONFINITE: return "KX_E_NONFINITE";
        case KX_E_AXIS: return "KX_E_AXIS";
        case KX_E_ALIAS: return "KX_E_ALIAS";
        case KX_E_CUDA: return "KX_E_CUDA";
        case KX_E_NO_DEVICE: return "KX_E_NO_DEVICE";
        case KX_E_TIMEOUT: return "KX_E_TIMEOUT";
        case KX_E_UNSUPPORTED: return "KX_E_UNSUPPORTED";
        case KX_E_AXES_MISMATCH: return "KX_E_AXES_MISMATCH";
        case KX_E_DUPLICATE_AXIS: return "KX_E_DUPLICATE_AXIS";
        default: return "KX_UNKNOWN";
    }
}

}  // extern "C"
