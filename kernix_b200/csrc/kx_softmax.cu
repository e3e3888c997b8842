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
#include <limits>
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
    int collapsed;              // row r starts at r * rs_s (source) and r * rs_o (output)
    int64_t rs_s, rs_o;
};

__device__ __forceinline__ void row_bases(const RowGeom &g, int64_t row, int64_t &sb, int64_t &ob) {
    if (g.collapsed) {
        sb = row * g.rs_s;
        ob = row * g.rs_o;
        return;
    }
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

// a / b from y = 1/b (the correctly rounded reciprocal) and one residual
// correction, Markstein's scheme ("IA-64 and Elementary Functions", 2000):
// q0 = a*y, r = a - b*q0 (exact through the fused multiply-add), q = q0 + r*y.
// The result is within one ulp of the IEEE quotient (equal to it for almost
// all operands) and costs three FMA-pipe instructions instead of a division.
// Used only when y is a normal number (checked on the host).
template <typename T>
__device__ __forceinline__ T div_by(T a, T b, T y) {
    const T q = a * y;
    const T r = fma(-b, q, a);
    return fma(r, y, q);
}

template <typename T> struct Vec16;
template <> struct Vec16<float> {
    using type = float4;
    static constexpr int n = 4;
};
template <> struct Vec16<double> {
    using type = double2;
    static constexpr int n = 2;
};
template <typename V, typename T> __device__ __forceinline__ T &lane_of(V &v, int c) {
    return reinterpret_cast<T *>(&v)[c];
}

template <typename T>
__device__ __forceinline__ T warp_min(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmin(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
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

// Contiguous rows that fit in registers (unit stride along the axis, 16-byte
// aligned rows): one 256-thread block per row, NV 16-byte vectors per thread,
// grid-stride over rows.  A block per row keeps ~30 registers per thread, so
// 16 blocks share an SM and their loads overlap each other's exp/normalise
// phases (a warp per row at 2048 elements ran at half the HBM rate).
// Nonfinite inputs are detected from the row's max, min and sum (a NaN or +inf
// makes the sum NaN, a -inf shows as the minimum); such rows are rescanned
// from memory for the first bad index and nothing is written for them.
template <typename T, int NV>
__global__ void __launch_bounds__(256) softmax_rows_block_vec(const T *__restrict__ src, T *__restrict__ out,
                                                              const __grid_constant__ RowGeom g, T temperature,
                                                              T recip, int use_recip,
                                                              unsigned long long *first_bad) {
    using V = typename Vec16<T>::type;
    constexpr int VN = Vec16<T>::n;
    constexpr int NW = 8;
    __shared__ T red[2][2][NW];
    __shared__ int64_t redi[NW];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t lenv = g.len / VN;
    int par = 0;
    for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x, par ^= 1) {
        int64_t sb, ob;
        row_bases(g, row, sb, ob);
        const V *sv = reinterpret_cast<const V *>(src + sb);
        V v[NV];
        T mx = -INFINITY, mn = INFINITY;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int64_t q = threadIdx.x + 256 * i;
            if (q < lenv) {
                v[i] = __ldg(sv + q);
#pragma unroll
                for (int c = 0; c < VN; ++c) {
                    mx = fmax(mx, lane_of<V, T>(v[i], c));
                    mn = fmin(mn, lane_of<V, T>(v[i], c));
                }
            }
        }
        mx = warp_max(mx);
        mn = warp_min(mn);
        if (lane == 0) {
            red[par][0][w] = mx;
            red[par][1][w] = mn;
        }
        __syncthreads();
        mx = red[par][0][0];
        mn = red[par][1][0];
#pragma unroll
        for (int j = 1; j < NW; ++j) {
            mx = fmax(mx, red[par][0][j]);
            mn = fmin(mn, red[par][1][j]);
        }
        T s = T(0);
        if (use_recip && isfinite(mx - mn)) {
            // every difference x - max is finite: (x - max) / T directly
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                if (threadIdx.x + 256 * i < lenv) {
#pragma unroll
                    for (int c = 0; c < VN; ++c) {
                        T &e = lane_of<V, T>(v[i], c);
                        e = kexp(div_by(e - mx, temperature, recip));
                        s += e;
                    }
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                if (threadIdx.x + 256 * i < lenv) {
#pragma unroll
                    for (int c = 0; c < VN; ++c) {
                        T &e = lane_of<V, T>(v[i], c);
                        e = kexp(scaled_difference(e, mx, temperature));
                        s += e;
                    }
                }
            }
        }
        s = warp_sum(s);
        __syncthreads();   // all maxima read before the sums reuse the slot
        if (lane == 0) red[par][0][w] = s;
        __syncthreads();
        s = T(0);
#pragma unroll
        for (int j = 0; j < NW; ++j) s += red[par][0][j];
        if (!isfinite(s) || mn == -INFINITY) {
            // some element is inf or NaN: find the first one in axis order
            int64_t bad = INT64_MAX;
            for (int64_t j = threadIdx.x; j < g.len; j += blockDim.x)
                if (!isfinite(src[sb + j]) && j < bad) bad = j;
            bad = warp_min_i64(bad);
            if (lane == 0) redi[w] = bad;
            __syncthreads();
            if (threadIdx.x == 0) {
                int64_t b = redi[0];
                for (int j = 1; j < NW; ++j) b = redi[j] < b ? redi[j] : b;
                atomicMin(first_bad, (unsigned long long)(row * g.len + b));
            }
            __syncthreads();
            continue;
        }
        const T rs = T(1) / s;   // s >= 1: the maximum contributes exp(0)
        V *ov = reinterpret_cast<V *>(out + ob);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int64_t q = threadIdx.x + 256 * i;
            if (q < lenv) {
                V r = v[i];
#pragma unroll
                for (int c = 0; c < VN; ++c) lane_of<V, T>(r, c) = div_by(lane_of<V, T>(r, c), s, rs);
                ov[q] = r;
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

// True when row r (C order over the outer dims) starts at r * (*rs): the outer
// dims nest like one C-ordered axis.  Size-one dims are ignored.
bool collapse_rows(const int64_t *dims, const int64_t *str, int n, int64_t *rs) {
    int64_t prod = 1, base = 0;
    bool have = false;
    for (int d = n - 1; d >= 0; --d) {
        if (dims[d] == 1) continue;
        if (!have) {
            base = str[d];
            have = true;
        } else if (str[d] != base * prod) {
            return false;
        }
        prod *= dims[d];
    }
    *rs = base;
    return true;
}

// `plain` selects softmax (math.rs:398-465,531-536): exp(x - max) / sum with
// no temperature and "softmax" as the operation of its errors.  Running it as
// temperature 1 gives the same values: (x - max) / 1 and the reciprocal path's
// x * 1 are exact, and the divide-first fallback x/1 - max/1 is x - max again.
template <typename T>
int softmax_impl(kx_handle *hh, const kx_tensor *src, int64_t axis, T temperature, const kx_tensor *out,
                 kx_error *err, bool plain = false) {
    const char *kOp = plain ? "softmax" : "softmax_temperature";
    if (!hh) return set_err(err, KX_E_PARAM, kOp, "null handle");
    Handle *h = &hh->impl;
    // normalized_exp_advanced: temperature first, then axis, then shape;
    // normalized_exp (plain): axis, then shape.
    if (!plain && (!std::isfinite((double)temperature) || !(temperature > T(0))))
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
    g.collapsed = collapse_rows(g.odims, g.sstr, nd, &g.rs_s) && collapse_rows(g.odims, g.ostr, nd, &g.rs_o);
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
        const unsigned grid_r = (unsigned)(g.rows < blocks_cap ? g.rows : blocks_cap);
        constexpr int VN = Vec16<T>::n;
        const bool aligned16 = g.s_axis == 1 && g.o_axis == 1 && g.len % VN == 0 &&
                               (reinterpret_cast<uintptr_t>(sp) % 16 == 0) &&
                               (reinterpret_cast<uintptr_t>(op) % 16 == 0);
        bool rows_aligned = true;
        for (int d = 0; d < nd; ++d) rows_aligned &= (g.sstr[d] % VN == 0) && (g.ostr[d] % VN == 0);
        const int64_t lenv = g.len / VN;
        // (x - max) / T through the reciprocal when 1/T is a normal number
        const T recip = T(1) / temperature;
        const int use_recip = std::isnormal((double)recip) && std::isnormal((double)temperature) &&
                              std::fabs((double)recip) < (double)std::numeric_limits<T>::max() / 4;
        if (aligned16 && rows_aligned && lenv <= 256 * 8 && g.len > 32 * VN * 4) {
            if (lenv <= 256)
                softmax_rows_block_vec<T, 1><<<grid_r, 256, 0, h->stream>>>(sp, op, g, temperature, recip, use_recip, flag);
            else if (lenv <= 512)
                softmax_rows_block_vec<T, 2><<<grid_r, 256, 0, h->stream>>>(sp, op, g, temperature, recip, use_recip, flag);
            else if (lenv <= 1024)
                softmax_rows_block_vec<T, 4><<<grid_r, 256, 0, h->stream>>>(sp, op, g, temperature, recip, use_recip, flag);
            else
                softmax_rows_block_vec<T, 8><<<grid_r, 256, 0, h->stream>>>(sp, op, g, temperature, recip, use_recip, flag);
            h->last_kernel = "softmax_rows_block_vec";
        } else if (std::is_same<T, float>::value && aligned16 && rows_aligned && g.len <= 32 * 4 * 4) {
            if constexpr (std::is_same<T, float>::value)
                softmax_rows_warp_vec<4><<<grid_w, 256, 0, h->stream>>>(sp, op, g, temperature, flag);
            h->last_kernel = "softmax_rows_warp_vec";
        } else if (g.len <= 32 * 4) {
            softmax_rows_warp<T, 4><<<grid_w, 256, 0, h->stream>>>(sp, op, g, temperature, flag);
            h->last_kernel = "softmax_rows_warp";
        } else if (g.len <= 32 * 32) {
            softmax_rows_warp<T, 32><<<grid_w, 256, 0, h->stream>>>(sp, op, g, temperature, flag);
            h->last_kernel = "softmax_rows_warp";
        } else {
            softmax_rows_block<T><<<grid_r, 256, 0, h->stream>>>(sp, op, g, temperature, flag);
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
int kx_softmax_f32(kx_handle *h, const kx_tensor *src, int64_t axis, const kx_tensor *out, kx_error *err) {
    return softmax_impl<float>(h, src, axis, 1.0f, out, err, true);
}
int kx_softmax_f64(kx_handle *h, const kx_tensor *src, int64_t axis, const kx_tensor *out, kx_error *err) {
    return softmax_impl<double>(h, src, axis, 1.0, out, err, true);
}
}
