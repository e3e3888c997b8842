// conv2d as an implicit GEMM with im2col fused into the operand load.
//
// Restates kernix-ops neural.rs:200-302 (conv_impl's native branch): per batch
// and group, columns[(ci,ky,kx)][pixel] gathered from the NCHW input with zero
// padding, then weight[co][(ci,ky,kx)] x columns.  Here no column buffer exists:
// the B-operand loader reads input elements straight from HBM through a
// per-CTA table of (ci,ky,kx) offsets, and every GEMM column is one output
// pixel of one image (the GEMM n extent is batch*oh*ow).  The output is written
// directly in NCHW order.
//
// Nonfinite weights with padding: the reference routes nonfinite data to its
// ordered scalar path (neural.rs:212-216, 341-357), which skips padded taps,
// whereas a padded tap here contributes 0*w.  A weight scan sets a device flag
// and, only when it is set, a direct kernel recomputes the output in the
// scalar path's order, so 0*inf never reaches the result.
#include <cstring>
#include <type_traits>

#include "gemm_simt.cuh"
#include "kx_internal.hpp"

using namespace kx;

namespace {

struct ConvGeom {
    int64_t n, c, h, w;         // input dims
    int64_t co, cg, kh, kw;     // weight dims (cg = input channels per group)
    int64_t oh, ow;
    int64_t groups, cog;        // groups and output channels per group
    int64_t sy, sx, py, px, dy, dx;
    int64_t xs[4];              // input strides (elements)
    int64_t ws[4];              // weight strides
    int64_t os[4];              // output strides (C-contiguous)
    int64_t kk;                 // GEMM k extent = cg*kh*kw
    int64_t ncols;              // GEMM n extent = n*oh*ow
};

struct KEntry {
    int64_t x_off;   // ci*xs1 + ky*dy*xs2 + kx*dx*xs3
    int64_t w_off;   // ci*ws1 + ky*ws2 + kx*ws3
    int32_t ry, rx;  // ky*dy, kx*dx
};

__device__ __forceinline__ KEntry make_entry(const ConvGeom &g, int64_t kk) {
    const int64_t khw = g.kh * g.kw;
    const int64_t ci = kk / khw, r = kk % khw;
    const int64_t ky = r / g.kw, kx = r % g.kw;
    KEntry e;
    e.ry = (int32_t)(ky * g.dy);
    e.rx = (int32_t)(kx * g.dx);
    e.x_off = ci * g.xs[1] + (int64_t)e.ry * g.xs[2] + (int64_t)e.rx * g.xs[3];
    e.w_off = ci * g.ws[1] + ky * g.ws[2] + kx * g.ws[3];
    return e;
}

template <typename T, typename Cfg, bool kTable>
__global__ void __launch_bounds__(Cfg::NT, Cfg::MinBlocks) conv_igemm_kernel(const T *__restrict__ x, const T *__restrict__ wt,
                                                              T *__restrict__ y, const __grid_constant__ ConvGeom g) {
    constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, NT = Cfg::NT;
    constexpr int PA = Cfg::PA, PB = Cfg::PB;
    static_assert(NT % BN == 0 && BK % (NT / BN) == 0, "column mapping");
    static_assert(NT % BK == 0 && BM % (NT / BK) == 0, "weight mapping");
    constexpr int B_PER = BK / (NT / BN);   // k rows per thread for the input gather
    constexpr int A_PER = BM / (NT / BK);   // rows per thread for the weight gather
    __shared__ __align__(16) T sa[2][BK * PA];
    __shared__ __align__(16) T sb[2][BK * PB];
    extern __shared__ __align__(16) unsigned char dyn[];
    KEntry *table = reinterpret_cast<KEntry *>(dyn);

    const int tid = threadIdx.x;
    const int tiles_m = (int)((g.cog + BM - 1) / BM);
    const int tiles_n = (int)((g.ncols + BN - 1) / BN);
    int tm, tn;
    raster(blockIdx.x, tiles_m, tiles_n, 8, tm, tn);
    const int64_t m0 = (int64_t)tm * BM, n0 = (int64_t)tn * BN;
    const int64_t grp = blockIdx.y;

    if constexpr (kTable) {
        for (int64_t k = tid; k < g.kk; k += NT) table[k] = make_entry(g, k);
    }

    // This thread's input column (one output pixel of one image).
    const int col = tid % BN;
    const int krow0 = tid / BN;
    const int64_t gcol = n0 + col;
    const bool col_ok = gcol < g.ncols;
    // Input coordinates fit int32 (the host bounds padding, stride and extents).
    int iy0 = 0, ix0 = 0;
    int64_t xbase = 0;
    const int ih = (int)g.h, iw = (int)g.w;
    if (col_ok) {
        const int64_t hw = g.oh * g.ow;
        const int64_t img = gcol / hw, p = gcol % hw;
        const int64_t oy = p / g.ow, ox = p % g.ow;
        iy0 = (int)(oy * g.sy - g.py);
        ix0 = (int)(ox * g.sx - g.px);
        xbase = img * g.xs[0] + grp * g.cg * g.xs[1] + (int64_t)iy0 * g.xs[2] + (int64_t)ix0 * g.xs[3];
    }
    // Weight rows: thread walks k fastest.
    const int a_k = tid % BK;
    const int a_row0 = tid / BK;
    const T *wgrp = wt + grp * g.cog * g.ws[0];

    T ra[A_PER], rb[B_PER];
    auto load = [&](int64_t k0) {
#pragma unroll
        for (int i = 0; i < B_PER; ++i) {
            const int64_t kk = k0 + krow0 + i * (NT / BN);
            T v = T(0);
            if (col_ok && kk < g.kk) {
                KEntry e;
                if constexpr (kTable) e = table[kk];
                else e = make_entry(g, kk);
                const int iy = iy0 + e.ry, ix = ix0 + e.rx;
                if (iy >= 0 && iy < ih && ix >= 0 && ix < iw) v = __ldg(x + xbase + e.x_off);
            }
            rb[i] = v;
        }
        const int64_t kk = k0 + a_k;
        int64_t woff = 0;
        if (kk < g.kk) {
            if constexpr (kTable) woff = table[kk].w_off;
            else woff = make_entry(g, kk).w_off;
        }
#pragma unroll
        for (int i = 0; i < A_PER; ++i) {
            const int64_t co = m0 + a_row0 + i * (NT / BK);
            ra[i] = (co < g.cog && kk < g.kk) ? __ldg(wgrp + co * g.ws[0] + woff) : T(0);
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int i = 0; i < B_PER; ++i) sb[buf][(krow0 + i * (NT / BN)) * PB + col] = rb[i];
#pragma unroll
        for (int i = 0; i < A_PER; ++i) sa[buf][a_k * PA + a_row0 + i * (NT / BK)] = ra[i];
    };

    if constexpr (kTable) __syncthreads();
    MicroTile<T, BM, BN, Cfg::TM, Cfg::TN> mt;
    mt.init(tid);
    const int ktiles = (int)((g.kk + BK - 1) / BK);
    load(0);
    store(0);
    __syncthreads();
    for (int kt = 0; kt < ktiles; ++kt) {
        const int cur = kt & 1;
        if (kt + 1 < ktiles) load((int64_t)(kt + 1) * BK);
        mt.template mma<BK, PA, PB>(sa[cur], sb[cur]);
        if (kt + 1 < ktiles) store(cur ^ 1);
        __syncthreads();
    }

    // Epilogue: column -> (image, pixel); row -> output channel of this group.
    // The output is C-contiguous, so element (img, co, p) sits at
    // (img*co_total + co)*hw + p.
    constexpr int HN = Cfg::TN / 2;
    const int64_t hw = g.oh * g.ow;
    constexpr bool kVec = sizeof(T) == 4 && HN == 4;
    const bool vec = kVec && (hw % 4 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0);
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
        const int64_t c0 = n0 + mt.col(h2 * HN);
        if (vec && c0 + HN <= g.ncols) {
            // Four columns in one image at consecutive pixels (hw % 4 == 0).
            const int64_t img = c0 / hw, p = c0 % hw;
#pragma unroll
            for (int i = 0; i < Cfg::TM; ++i) {
                const int64_t co = m0 + mt.row(i);
                if (co < g.cog) {
                    float4 v;
                    float *pv = reinterpret_cast<float *>(&v);
#pragma unroll
                    for (int j = 0; j < 4; ++j) pv[j] = (float)mt.acc(i, h2 * HN + j);
                    *reinterpret_cast<float4 *>(y + (img * g.co + grp * g.cog + co) * hw + p) = v;
                }
            }
            continue;
        }
#pragma unroll
        for (int j = 0; j < HN; ++j) {
            const int64_t cc = c0 + j;
            if (cc >= g.ncols) continue;
            const int64_t img = cc / hw, p = cc % hw;
#pragma unroll
            for (int i = 0; i < Cfg::TM; ++i) {
                const int64_t co = m0 + mt.row(i);
                if (co < g.cog) y[(img * g.co + grp * g.cog + co) * hw + p] = mt.acc(i, h2 * HN + j);
            }
        }
    }
}

// Sets *flag when any weight is NaN or infinite.
template <typename T>
__global__ void conv_weight_scan(const T *__restrict__ wt, const __grid_constant__ ConvGeom g, uint32_t *flag) {
    const int64_t total = g.co * g.cg * g.kh * g.kw;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = e;
        const int64_t kx = r % g.kw; r /= g.kw;
        const int64_t ky = r % g.kh; r /= g.kh;
        const int64_t ci = r % g.cg; r /= g.cg;
        const int64_t co = r;
        const T v = wt[co * g.ws[0] + ci * g.ws[1] + ky * g.ws[2] + kx * g.ws[3]];
        if (!isfinite(v)) atomicOr(flag, 1u);
    }
}

// Ordered scalar convolution (neural.rs:341-357 order: ci, ky, kx increasing,
// padded taps skipped, separate multiply and add).  With a flag it runs only
// when *flag is set (nonfinite-weight fixup); without one it always runs (the
// conv2d_reference mode of an ordered handle).
template <typename T>
__global__ void conv_direct_fixup(const T *__restrict__ x, const T *__restrict__ wt, T *__restrict__ y,
                                  const __grid_constant__ ConvGeom g, const uint32_t *flag) {
    if (flag && *flag == 0) return;
    const int64_t total = g.n * g.co * g.oh * g.ow;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = e;
        const int64_t ox = r % g.ow; r /= g.ow;
        const int64_t oy = r % g.oh; r /= g.oh;
        const int64_t co = r % g.co; r /= g.co;
        const int64_t img = r;
        const int64_t grp = co / g.cog;
        T sum = T(0);
        for (int64_t ci = 0; ci < g.cg; ++ci)
            for (int64_t ky = 0; ky < g.kh; ++ky)
                for (int64_t kx = 0; kx < g.kw; ++kx) {
                    const int64_t iy = oy * g.sy + ky * g.dy - g.py;
                    const int64_t ix = ox * g.sx + kx * g.dx - g.px;
                    if (iy < 0 || iy >= g.h || ix < 0 || ix >= g.w) continue;
                    const T a = x[img * g.xs[0] + (grp * g.cg + ci) * g.xs[1] + iy * g.xs[2] + ix * g.xs[3]];
                    const T b = wt[co * g.ws[0] + ci * g.ws[1] + ky * g.ws[2] + kx * g.ws[3]];
                    T prod;
                    if constexpr (sizeof(T) == 4) prod = __fmul_rn(a, b);
                    else prod = __dmul_rn(a, b);
                    if constexpr (sizeof(T) == 4) sum = __fadd_rn(sum, prod);
                    else sum = __dadd_rn(sum, prod);
                }
        y[img * g.os[0] + co * g.os[1] + oy * g.os[2] + ox * g.os[3]] = sum;
    }
}

template <typename T> struct ConvCfg;
template <> struct ConvCfg<float> : TileCfg<float, 128, 128, 8, 8, 8, 2> {};
template <> struct ConvCfg<double> : TileCfg<double, 128, 128, 8, 8, 8> {};
template <typename T> struct ConvSmallCfg;
template <> struct ConvSmallCfg<float> : TileCfg<float, 64, 64, 16, 4, 4, 2> {};
template <> struct ConvSmallCfg<double> : TileCfg<double, 64, 64, 16, 4, 4, 2> {};

template <typename T, typename Cfg>
cudaError_t launch_igemm(Handle *h, const T *x, const T *w, T *y, const ConvGeom &g) {
    const int64_t tiles = ((g.cog + Cfg::BM - 1) / Cfg::BM) * ((g.ncols + Cfg::BN - 1) / Cfg::BN);
    dim3 grid((unsigned)tiles, (unsigned)g.groups, 1);
    const size_t table_bytes = (size_t)g.kk * sizeof(KEntry);
    const size_t static_bytes = 2 * (size_t)Cfg::BK * (Cfg::PA + Cfg::PB) * sizeof(T);
    if (table_bytes + static_bytes <= 160 * 1024) {
        auto kern = conv_igemm_kernel<T, Cfg, true>;
        cudaError_t ce = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)table_bytes);
        if (ce != cudaSuccess) return ce;
        kern<<<grid, Cfg::NT, table_bytes, h->stream>>>(x, w, y, g);
    } else {
        conv_igemm_kernel<T, Cfg, false><<<grid, Cfg::NT, 0, h->stream>>>(x, w, y, g);
    }
    return cudaGetLastError();
}

template <typename T>
int conv_impl(kx_handle *hh, const kx_tensor *in, const kx_tensor *wt, const kx_conv2d_options *o,
              const kx_tensor *out, kx_error *err) {
    static const char *kOp = "conv2d";
    if (!hh) return set_err(err, KX_E_PARAM, kOp, "null handle");
    Handle *h = &hh->impl;
    Span si, sw, so;
    int rc = validate_tensor(in, sizeof(T), &si, err);
    if (rc) return rc;
    rc = validate_tensor(wt, sizeof(T), &sw, err);
    if (rc) return rc;
    uint64_t od[4];
    rc = conv_shape(in->dims, in->rank, wt->dims, wt->rank, o, od, err);
    if (rc) return rc;
    rc = validate_tensor(out, sizeof(T), &so, err);
    if (rc) return rc;
    if (out->rank != 4 || out->dims[0] != od[0] || out->dims[1] != od[1] || out->dims[2] != od[2] ||
        out->dims[3] != od[3])
        return set_err(err, KX_E_LAYOUT, kOp, "output shape mismatch", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
    if (!is_c_contiguous(out))
        return set_err(err, KX_E_LAYOUT, kOp, "output must be C-contiguous", KX_LAYOUT_OUTPUT_NOT_C_CONTIGUOUS);
    if (spans_overlap(out->data, so, in->data, si, sizeof(T)) || spans_overlap(out->data, so, wt->data, sw, sizeof(T)))
        return set_err(err, KX_E_ALIAS, kOp, "output overlaps an input");
    const uint64_t total = numel(od, 4);
    if (total == 0) return KX_OK;

    ConvGeom g;
    std::memset(&g, 0, sizeof(g));
    g.n = (int64_t)in->dims[0];
    g.c = (int64_t)in->dims[1];
    g.h = (int64_t)in->dims[2];
    g.w = (int64_t)in->dims[3];
    g.co = (int64_t)wt->dims[0];
    g.cg = (int64_t)wt->dims[1];
    g.kh = (int64_t)wt->dims[2];
    g.kw = (int64_t)wt->dims[3];
    g.oh = (int64_t)od[2];
    g.ow = (int64_t)od[3];
    g.groups = (int64_t)o->groups;
    g.cog = g.co / g.groups;
    g.sy = (int64_t)o->stride[0];
    g.sx = (int64_t)o->stride[1];
    g.py = (int64_t)o->padding[0];
    g.px = (int64_t)o->padding[1];
    g.dy = (int64_t)o->dilation[0];
    g.dx = (int64_t)o->dilation[1];
    for (int i = 0; i < 4; ++i) {
        g.xs[i] = in->dims[i] <= 1 ? 0 : in->strides[i];
        g.ws[i] = wt->dims[i] <= 1 ? 0 : wt->strides[i];
        g.os[i] = out->dims[i] <= 1 ? 0 : out->strides[i];
    }
    g.kk = g.cg * g.kh * g.kw;
    g.ncols = g.n * g.oh * g.ow;
    // Geometry that reaches int32 limits in the tile loops is outside this
    // kernel's envelope (the validated span keeps every address in range).
    if (g.kh * g.dy > INT32_MAX / 4 || g.kw * g.dx > INT32_MAX / 4 || g.groups > 65535 || g.py > INT32_MAX / 4 ||
        g.px > INT32_MAX / 4 || g.h > INT32_MAX / 4 || g.w > INT32_MAX / 4 || g.oh * g.sy > INT32_MAX / 4 ||
        g.ow * g.sx > INT32_MAX / 4)
        return set_err(err, KX_E_UNSUPPORTED, kOp, "geometry outside kernel limits");

    int dev_prev = -1;
    cudaGetDevice(&dev_prev);
    if (dev_prev != h->device) cudaSetDevice(h->device);
    const T *xp = static_cast<const T *>(in->data) + in->origin;
    const T *wp = static_cast<const T *>(wt->data) + wt->origin;
    T *yp = static_cast<T *>(out->data) + out->origin;
    cudaError_t ce = cudaSuccess;
    if (h->ordered) {
        int64_t blocks = ((int64_t)total + 255) / 256;
        if (blocks > 16LL * h->sm_count) blocks = 16LL * h->sm_count;
        conv_direct_fixup<T><<<(unsigned)blocks, 256, 0, h->stream>>>(xp, wp, yp, g, nullptr);
        ce = cudaGetLastError();
        ++h->launches;
        h->last_kernel = "conv_direct_ordered";
        if (dev_prev >= 0 && dev_prev != h->device) cudaSetDevice(dev_prev);
        if (ce != cudaSuccess) {
            h->cuda_fail(ce);
            return cuda_err(err, h, kOp);
        }
        return KX_OK;
    }
    const bool padded = g.py != 0 || g.px != 0;
    if (padded) {
        ce = cudaMemsetAsync(h->flags + kConvFlagWord, 0, sizeof(uint32_t), h->stream);
        if (ce == cudaSuccess) {
            const int64_t wtotal = g.co * g.kk;
            int64_t blocks = (wtotal + 255) / 256;
            if (blocks > 4LL * h->sm_count) blocks = 4LL * h->sm_count;
            conv_weight_scan<T><<<(unsigned)blocks, 256, 0, h->stream>>>(wp, g, h->flags + kConvFlagWord);
            ce = cudaGetLastError();
            ++h->launches;
        }
    }
    bool done = false;
    if constexpr (std::is_same<T, float>::value) {
        // Tensor cores for the split-TF32 implicit GEMM when the tiles cover
        // the SMs (or the handle asks for it); the SIMT kernel otherwise.
        const int64_t tc_tiles = ((g.cog + 127) / 128) * ((g.ncols + 127) / 128) * g.groups;
        if (ce == cudaSuccess && h->f32_variant != KX_F32_FFMA &&
            (h->f32_variant == KX_F32_3XTF32 || tc_tiles >= h->sm_count / 2)) {
            int64_t ws[4] = {g.ws[0], g.ws[1], g.ws[2], g.ws[3]};
            if (g.co == 1) ws[0] = (g.kk + 3) / 4 * 4;   // a single row: any aligned pitch
            const char *name = "none";
            const int rc = run_conv_tc(h, xp, g.xs, wp, ws, yp, g.n, g.c, g.h, g.w, g.co, g.cg, g.kh, g.kw, g.oh,
                                       g.ow, g.groups, g.sy, g.sx, g.py, g.px, g.dy, g.dx, &name);
            if (rc == KX_OK) {
                h->last_kernel = name;
                done = true;
            } else if (rc != KX_DECLINED) {
                ce = (cudaError_t)h->last_cuda_error;
            }
        }
    }
    if (ce == cudaSuccess && !done) {
        const int64_t big = ((g.cog + 127) / 128) * ((g.ncols + 127) / 128) * g.groups;
        if (big >= 2LL * h->sm_count) {
            ce = launch_igemm<T, ConvCfg<T>>(h, xp, wp, yp, g);
            h->last_kernel = "conv_igemm_128x128";
        } else {
            ce = launch_igemm<T, ConvSmallCfg<T>>(h, xp, wp, yp, g);
            h->last_kernel = "conv_igemm_64x64";
        }
        ++h->launches;
    }
    if (ce == cudaSuccess && padded) {
        int64_t blocks = ((int64_t)total + 255) / 256;
        if (blocks > 8LL * h->sm_count) blocks = 8LL * h->sm_count;
        conv_direct_fixup<T><<<(unsigned)blocks, 256, 0, h->stream>>>(xp, wp, yp, g, h->flags + kConvFlagWord);
        ce = cudaGetLastError();
        ++h->launches;
    }
    if (dev_prev >= 0 && dev_prev != h->device) cudaSetDevice(dev_prev);
    if (ce != cudaSuccess) {
        h->cuda_fail(ce);
        return cuda_err(err, h, kOp);
    }
    return KX_OK;
}

}  // namespace

extern "C" {
int kx_conv2d_f32(kx_handle *h, const kx_tensor *input, const kx_tensor *weight, const kx_conv2d_options *options,
                  const kx_tensor *out, kx_error *err) {
    return conv_impl<float>(h, input, weight, options, out, err);
}
int kx_conv2d_f64(kx_handle *h, const kx_tensor *input, const kx_tensor *weight, const kx_conv2d_options *options,
                  const kx_tensor *out, kx_error *err) {
    return conv_impl<double>(h, input, weight, options, out, err);
}
}
