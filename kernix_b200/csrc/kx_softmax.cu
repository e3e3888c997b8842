// Row softmax with temperature on device memory (the softmax step between the
// attention score and value products).
//
// Restates kernix-ops ops/math_extra.rs:425-500 (normalized_exp_advanced with no
// mask) and :394-401 (scaled_difference):
//   * every element of a row must be finite, else NonFiniteInput with the
//     indices of the first nonfinite element in the reference scan order
//     (outer rows in C order, then position along the axis);
//   * max over the row; delta = (x - max) / T, or x/T - max/T when the
//     difference overflows;
//   * out = exp(delta) / sum(exp(delta)).
// The row sum is a warp/block tree reduction rather than the reference's
// sequential sum, so the last bits can differ (tolerance-checked).
#include <cfloat>
#include <cmath>
#include <cstring>
#include <type_traits>

#include "kx_internal.hpp"

using namespace kx;

namespace {

constexpr int kMaxOuter = KX_MAX_RANK;

struct RowGeom {
    int64_t len;          // elements along the axis
    int64_t rows;         // number of rows (product of the other dims)
    int64_t s_axis;       // source stride along the axis
    int64_t o_axis;       // output stride along the axis
    int nouter;
    int64_t odims[kMaxOuter];   // outer dims (axis removed), C order
    int64_t sstr[kMaxOuter];    // source strides of the outer dims
    int64_t ostr[kMaxOuter];    // output strides of the outer dims
};

__device__ __forceinline__ void row_bases(const RowGeom &g, int64_t row, int64_t &sb, int64_t &ob) {
    sb = ob = 0;
    for (int d = g.nouter - 1; d >= 0; --d) {
        int64_t c = row % g.odims[d];
        row /= g.odims[d];
        sb += c * g.sstr[d];
        ob += c * g.ostr[d];
    }
}

template <typename T> __device__ __forceinline__ T kexp(T x);
template <> __device__ __forceinline__ float kexp<float>(float x) { return expf(x); }
template <> __device__ __forceinline__ double kexp<double>(double x) { return exp(x); }

template <typename T>
__device__ __forceinline__ T scaled_difference(T v, T m, T t) {
    T d = v - m;
    return isfinite(d) ? d / t : v / t - m / t;
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int64_t warp_min_i64(int64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        int64_t w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w < v ? w : v;
    }
    return v;
}

// One warp per row; the row lives in registers (len <= 32 * ITEMS).
template <typename T, int ITEMS>
__global__ void __launch_bounds__(256) softmax_rows_warp(const T *__restrict__ src, T *__restrict__ out,
                                                         const __grid_constant__ RowGeom g, T temperature,
                                                         unsigned long long *first_bad) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < g.rows; row += warps) {
        int64_t sb, ob;
        row_bases(g, row, sb, ob);
        T v[ITEMS];
        T mx = -INFINITY;
        int64_t bad = INT64_MAX;
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            const int64_t j = lane + 32 * i;
            if (j < g.len) {
                v[i] = __ldg(src + sb + j * g.s_axis);
                if (!isfinite(v[i])) bad = bad < j ? bad : j;
                mx = fmax(mx, v[i]);
            } else {
                v[i] = T(0);
            }
        }
        bad = warp_min_i64(bad);
        if (bad != INT64_MAX) {
            if (lane == 0) atomicMin(first_bad, (unsigned long long)(row * g.len + bad));
            continue;
        }
        mx = warp_max(mx);
        T s = T(0);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            const int64_t j = lane + 32 * i;
            if (j < g.len) {
                v[i] = kexp(scaled_difference(v[i], mx, temperature));
                s += v[i];
            }
        }
        s = warp_sum(s);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            const int64_t j = lane + 32 * i;
            if (j < g.len) out[ob + j * g.o_axis] = v[i] / s;
        }
    }
}

// Contiguous rows (unit strides, 16-byte aligned, len % 4 == 0): float4 traffic.
template <int ITEMS4>
__global__ void __launch_bounds__(256) softmax_rows_warp_vec(const float *__restrict__ src, float *__restrict__ out,
                                                             const __grid_constant__ RowGeom g, float temperature,
                                                             unsigned long long *first_bad) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t len4 = g.len >> 2;
    for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < g.rows; row += warps) {
        int64_t sb, ob;
        row_bases(g, row, sb, ob);
        float4 v[ITEMS4];
        float mx = -INFINITY;
        int64_t bad = INT64_MAX;
#pragma unroll
        for (int i = 0; i < ITEMS4; ++i) {
            const int64_t q = lane + 32 * i;
            if (q < len4) {
                v[i] = __ldg(reinterpret_cast<const float4 *>(src + sb) + q);
                const float *e = reinterpret_cast<const float *>(&v[i]);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (!isfinite(e[c])) bad = bad < 4 * q + c ? bad : 4 * q + c;
                    mx = fmaxf(mx, e[c]);
                }
            } else {
                v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        bad = warp_min_i64(bad);
        if (bad != INT64_MAX) {
            if (lane == 0) atomicMin(first_bad, (unsigned long long)(row * g.len + bad));
            continue;
        }
        mx = warp_max(mx);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < ITEMS4; ++i) {
            const int64_t q = lane + 32 * i;
            if (q < len4) {
                float *e = reinterpret_cast<float *>(&v[i]);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    e[c] = expf(scaled_difference(e[c], mx, temperature));
                    s += e[c];
                }
            }
        }
        s = warp_sum(s);
#pragma unroll
        for (int i = 0; i < ITEMS4; ++i) {
            const int64_t q = lane + 32 * i;
            if (q < len4) {
                float4 r = v[i];
                r.x = r.x / s;
                r.y = r.y / s;
                r.z = r.z / s;
                r.w = r.w / s;
                reinterpret_cast<float4 *>(out + ob)[q] = r;
            }
        }
    }
}

// Long rows: one block per row, three passes over global memory.
template <typename T>
__global__ void __launch_bounds__(256) softmax_rows_block(const T *__restrict__ src, T *__restrict__ out,
                                                          const __grid_constant__ RowGeom g, T temperature,
                                                          unsigned long long *first_bad) {
    __shared__ T red[32];
    __shared__ int64_t redi[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
        int64_t sb, ob;
        row_bases(g, row, sb, ob);
        T mx = -INFINITY;
        int64_t bad = INT64_MAX;
        for (int64_t j = threadIdx.x; j < g.len; j += blockDim.x) {
            T x = src[sb + j * g.s_axis];
            if (!isfinite(x) && j < bad) bad = j;
            mx = fmax(mx, x);
        }
        mx = warp_max(mx);
        bad = warp_min_i64(bad);
        if (lane == 0) {
            red[warp] = mx;
            redi[warp] = bad;
        }
        __syncthreads();
        if (warp == 0) {
            T m2 = lane < nw ? red[lane] : -INFINITY;
            int64_t b2 = lane < nw ? redi[lane] : INT64_MAX;
            m2 = warp_max(m2);
            b2 = warp_min_i64(b2);
            if (lane == 0) {
                red[0] = m2;
                redi[0] = b2;
            }
        }
        __syncthreads();
        mx = red[0];
        bad = redi[0];
        __syncthreads();
        if (bad != INT64_MAX) {
            if (threadIdx.x == 0) atomicMin(first_bad, (unsigned long long)(row * g.len + bad));
            continue;
        }
        T s = T(0);
        for (int64_t j = threadIdx.x; j < g.len; j += blockDim.x)
            s += kexp(scaled_difference(src[sb + j * g.s_axis], mx, temperature));
        s = warp_sum(s);
        if (lane == 0) red[warp] = s;
        __syncthreads();
        if (warp == 0) {
            T s2 = lane < nw ? red[lane] : T(0);
            s2 = warp_sum(s2);
            if (lane == 0) red[0] = s2;
        }
        __syncthreads();
        s = red[0];
        __syncthreads();
        for (int64_t j = threadIdx.x; j < g.len; j += blockDim.x)
            out[ob + j * g.o_axis] = kexp(scaled_difference(src[sb + j * g.s_axis], mx, temperature)) / s;
    }
}

template <typename T>
int softmax_impl(kx_handle *hh, const kx_tensor *src, int64_t axis, T temperature, const kx_tensor *out,
                 kx_error *err) {
    static const char *kOp = "softmax_temperature";
    if (!hh) return set_err(err, KX_E_PARAM, kOp, "null handle");
    Handle *h = &hh->impl;
    // normalized_exp_advanced: temperature first, then axis, then shape.
    if (!std::isfinite((double)temperature) || !(temperature > T(0)))
        return set_err(err, KX_E_PARAM, kOp, "temperature (must be finite and > 0)");
    Span ss, so;
    int rc = validate_tensor(src, sizeof(T), &ss, err);
    if (rc) return rc;
    const uint32_t rank = src->rank;
    int64_t ax;
    {
        bool ok;
        if (axis < 0) {
            ax = (int64_t)rank + axis;
            ok = ax >= 0;
        } else {
            ax = axis;
            ok = true;
        }
        if (!ok || ax >= (int64_t)rank) {
            set_err(err, KX_E_AXIS, kOp, "axis", (uint64_t)axis, rank);
            return KX_E_AXIS;
        }
    }
    rc = validate_tensor(out, sizeof(T), &so, err);
    if (rc) return rc;
    if (out->rank != rank)
        return set_err(err, KX_E_LAYOUT, kOp, "output shape mismatch", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
    for (uint32_t i = 0; i < rank; ++i)
        if (out->dims[i] != src->dims[i])
            return set_err(err, KX_E_LAYOUT, kOp, "output shape mismatch", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
    if (!is_c_contiguous(out))
        return set_err(err, KX_E_LAYOUT, kOp, "output must be C-contiguous", KX_LAYOUT_OUTPUT_NOT_C_CONTIGUOUS);
    if (spans_overlap(out->data, so, src->data, ss, sizeof(T)))
        return set_err(err, KX_E_ALIAS, kOp, "output overlaps the input");
    const uint64_t total = numel(src->dims, rank);
    if (total == 0) return KX_OK;

    RowGeom g;
    std::memset(&g, 0, sizeof(g));
    g.len = (int64_t)src->dims[ax];
    g.rows = (int64_t)(total / src->dims[ax]);
    g.s_axis = src->strides[ax];
    g.o_axis = out->strides[ax];
    int nd = 0;
    for (uint32_t d = 0; d < rank; ++d) {
        if ((int64_t)d == ax) continue;
        g.odims[nd] = (int64_t)src->dims[d];
        g.sstr[nd] = src->strides[d];
        g.ostr[nd] = out->strides[d];
        ++nd;
    }
    g.nouter = nd;
    if (g.rows > (INT64_MAX / (g.len > 0 ? g.len : 1)))
        return set_err(err, KX_E_UNSUPPORTED, kOp, "too many elements");

    int dev_prev = -1;
    cudaGetDevice(&dev_prev);
    if (dev_prev != h->device) cudaSetDevice(h->device);
    const T *sp = static_cast<const T *>(src->data) + src->origin;
    T *op = static_cast<T *>(out->data) + out->origin;
    unsigned long long *flag = reinterpret_cast<unsigned long long *>(h->flags + kSoftmaxWord);
    cudaError_t ce = cudaMemsetAsync(flag, 0xff, sizeof(unsigned long long), h->stream);
    if (ce == cudaSuccess) {
        const int64_t blocks_cap = 16LL * h->sm_count;
        const int64_t wblocks = (g.rows + 7) / 8;
        const unsigned grid_w = (unsigned)(wblocks < blocks_cap ? wblocks : blocks_cap);
        const bool contig = std::is_same<T, float>::value && g.s_axis == 1 && g.o_axis == 1 && g.len % 4 == 0 &&
                            (reinterpret_cast<uintptr_t>(sp) % 16 == 0) && (reinterpret_cast<uintptr_t>(op) % 16 == 0);
        bool rows_aligned = true;
        for (int d = 0; d < nd; ++d) rows_aligned &= (g.sstr[d] % 4 == 0) && (g.ostr[d] % 4 == 0);
        if (contig && rows_aligned && g.len <= 32 * 4 * 16) {
            if constexpr (std::is_same<T, float>::value) {
                if (g.len <= 32 * 4 * 4)
                    softmax_rows_warp_vec<4><<<grid_w, 256, 0, h->stream>>>(sp, op, g, temperature, flag);
                else
                    softmax_rows_warp_vec<16><<<grid_w, 256, 0, h->stream>>>(sp, op, g, temperature, flag);
            }
            h->last_kernel = "softmax_rows_warp_vec";
        } else if (g.len <= 32 * 4) {
            softmax_rows_warp<T, 4><<<grid_w, 256, 0, h->stream>>>(sp, op, g, temperature, flag);
            h->last_kernel = "softmax_rows_warp";
        } else if (g.len <= 32 * 32) {
            softmax_rows_warp<T, 32><<<grid_w, 256, 0, h->stream>>>(sp, op, g, temperature, flag);
            h->last_kernel = "softmax_rows_warp";
        } else {
            const unsigned grid_b = (unsigned)(g.rows < blocks_cap ? g.rows : blocks_cap);
            softmax_rows_block<T><<<grid_b, 256, 0, h->stream>>>(sp, op, g, temperature, flag);
            h->last_kernel = "softmax_rows_block";
        }
        ce = cudaGetLastError();
        ++h->launches;
    }
    unsigned long long first = ~0ull;
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(&first, flag, sizeof(first), cudaMemcpyDeviceToHost, h->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(h->stream);
    if (dev_prev >= 0 && dev_prev != h->device) cudaSetDevice(dev_prev);
    if (ce != cudaSuccess) {
        h->cuda_fail(ce);
        return cuda_err(err, h, kOp);
    }
    if (first != ~0ull) {
        const int64_t row = (int64_t)(first / (uint64_t)g.len);
        const int64_t pos = (int64_t)(first % (uint64_t)g.len);
        set_err(err, KX_E_NONFINITE, kOp, "nonfinite input");
        if (err) {
            int64_t r = row;
            uint64_t idx[KX_MAX_RANK];
            for (int d = nd - 1; d >= 0; --d) {
                idx[d] = (uint64_t)(r % g.odims[d]);
                r /= g.odims[d];
            }
            uint32_t w = 0;
            for (uint32_t d = 0; d < rank; ++d) {
                if ((int64_t)d == ax) err->indices[w++] = (uint64_t)pos;
                else err->indices[w++] = idx[d < (uint32_t)ax ? d : d - 1];
            }
            err->nindices = rank;
        }
        return KX_E_NONFINITE;
    }
    return KX_OK;
}

}  // namespace

extern "C" {
int kx_softmax_temperature_f32(kx_handle *h, const kx_tensor *src, int64_t axis, float temperature,
                               const kx_tensor *out, kx_error *err) {
    return softmax_impl<float>(h, src, axis, temperature, out, err);
}
int kx_softmax_temperature_f64(kx_handle *h, const kx_tensor *src, int64_t axis, double temperature,
                               const kx_tensor *out, kx_error *err) {
    return softmax_impl<double>(h, src, axis, temperature, out, err);
}
}
