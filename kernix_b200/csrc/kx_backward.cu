// Backward products: the matmul VJP and conv2d_backward on device memory.
//
// Tape::matmul's VJP (crates/kernix/src/autograd.rs:622-690) is two more
// matmuls on transposed views -- dA = G B^T, dB = A^T G -- whose results are
// summed back over the batch axes each operand was broadcast along; with a
// shared right matrix (A of rank > 2, B of rank <= 2) the leading rows of A and
// G flatten into one long contraction instead.  Here both run through the
// forward kernels (transposed operands are strided views, no copies), and a
// reduction kernel sums broadcast contributions, each output in increasing
// batch order.
//
// conv2d_backward (crates/kernix-ops/src/neural.rs:379-430) accumulates
// dx[n, c, y, x] += dy * w and dw[co, ci, ky, kx] += dy * x over output
// elements in C order.  The kernels below give every dx and dw element its
// own thread and add the same contributions in the same order, each product
// and sum separately rounded, so the results equal the reference loop's bit
// for bit.
#include <cstring>

#include "gemm_simt.cuh"
#include "kx_internal.hpp"

extern "C" int kx_matmul_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out,
                             kx_error *err);
extern "C" int kx_matmul_f64(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out,
                             kx_error *err);

namespace kx {
namespace {

template <typename T> struct MatmulFn;
template <> struct MatmulFn<float> {
    static int call(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *o, kx_error *e) {
        return kx_matmul_f32(h, a, b, o, e);
    }
};
template <> struct MatmulFn<double> {
    static int call(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *o, kx_error *e) {
        return kx_matmul_f64(h, a, b, o, e);
    }
};

// out[i] = sum of full[j] over the full-shape elements j that broadcast to
// output element i (C order over both; axis d of the full shape is summed
// when `red[d]`), in increasing j.
struct ReduceGeom {
    int rank;
    int64_t dims[KX_MAX_RANK];
    int64_t fstr[KX_MAX_RANK];    // C-order strides of the full tensor
    int red[KX_MAX_RANK];
    int64_t nout, nred;
};

template <typename T>
__global__ void unbroadcast_kernel(const T *__restrict__ full, T *__restrict__ out, const __grid_constant__ ReduceGeom g) {
    for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < g.nout; o += (int64_t)gridDim.x * blockDim.x) {
        // offset of output element o along the kept axes
        int64_t rem = o, base = 0;
        for (int d = g.rank - 1; d >= 0; --d) {
            if (g.red[d]) continue;
            base += (rem % g.dims[d]) * g.fstr[d];
            rem /= g.dims[d];
        }
        T acc = T(0);
        for (int64_t r = 0; r < g.nred; ++r) {
            int64_t rr = r, off = base;
            for (int d = g.rank - 1; d >= 0; --d) {
                if (!g.red[d]) continue;
                off += (rr % g.dims[d]) * g.fstr[d];
                rr /= g.dims[d];
            }
            acc = acc + full[off];
        }
        out[o] = acc;
    }
}

// A C-contiguous descriptor.
kx_tensor dense(void *data, const uint64_t *dims, uint32_t rank) {
    kx_tensor t;
    std::memset(&t, 0, sizeof(t));
    t.data = data;
    t.rank = rank;
    int64_t st = 1;
    for (int d = (int)rank - 1; d >= 0; --d) {
        t.dims[d] = dims[d];
        t.strides[d] = st;
        st *= (int64_t)(dims[d] ? dims[d] : 1);
    }
    t.storage_len = 1;
    for (uint32_t d = 0; d < rank; ++d) t.storage_len *= dims[d];
    return t;
}

// Swap the last two axes of a view.
kx_tensor swap_last(const kx_tensor &t) {
    kx_tensor s = t;
    std::swap(s.dims[t.rank - 1], s.dims[t.rank - 2]);
    std::swap(s.strides[t.rank - 1], s.strides[t.rank - 2]);
    return s;
}

// Leading axes (all but the last) nest in C order: the view reshapes to
// [rows, last] with row stride strides[rank - 2].
bool rows_collapse(const kx_tensor &t) {
    for (int d = 0; d + 2 < (int)t.rank; ++d)
        if (t.dims[d] > 1 && t.strides[d] != t.strides[d + 1] * (int64_t)t.dims[d + 1]) return false;
    return true;
}

// Write the full-shape gradient `fullg` (dims fdims) into `dst` (dims odims,
// right-aligned, C-contiguous), summing over broadcast axes; when no axis is
// summed the product is computed straight into `dst` by the caller instead.
template <typename T>
int reduce_into(Handle *h, const T *fullg, const uint64_t *fdims, uint32_t frank, const kx_tensor *dst,
                const uint64_t *odims, uint32_t orank) {
    ReduceGeom g;
    std::memset(&g, 0, sizeof(g));
    g.rank = (int)frank;
    int64_t st = 1;
    g.nout = 1;
    g.nred = 1;
    for (int d = (int)frank - 1; d >= 0; --d) {
        g.dims[d] = (int64_t)fdims[d];
        g.fstr[d] = st;
        st *= (int64_t)fdims[d];
        const int od = d - ((int)frank - (int)orank);
        const uint64_t ext = od >= 0 ? odims[od] : 1;
        g.red[d] = (ext == 1 && fdims[d] != 1) || od < 0 ? 1 : 0;
        if (g.red[d]) g.nred *= (int64_t)fdims[d];
        else g.nout *= (int64_t)fdims[d];
    }
    if (g.nout == 0) return KX_OK;
    T *out = static_cast<T *>(dst->data) + dst->origin;
    const int64_t blocks = (g.nout + 255) / 256 < 4 * h->sm_count ? (g.nout + 255) / 256 : 4 * h->sm_count;
    unbroadcast_kernel<T><<<(unsigned)blocks, 256, 0, h->stream>>>(fullg, out, g);
    ++h->launches;
    cudaError_t ce = cudaGetLastError();
    return ce == cudaSuccess ? KX_OK : h->cuda_fail(ce);
}

template <typename T>
int check_grad_out(const kx_tensor *t, const kx_tensor *like, const char *op, kx_error *err) {
    Span s;
    int rc = validate_tensor(t, sizeof(T), &s, err);
    if (rc) return rc;
    if (t->rank != like->rank) return set_err(err, KX_E_LAYOUT, op, "gradient shape mismatch", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
    for (uint32_t d = 0; d < t->rank; ++d)
        if (t->dims[d] != like->dims[d])
            return set_err(err, KX_E_LAYOUT, op, "gradient shape mismatch", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
    if (!is_c_contiguous(t))
        return set_err(err, KX_E_LAYOUT, op, "gradient must be C-contiguous", KX_LAYOUT_OUTPUT_NOT_C_CONTIGUOUS);
    return KX_OK;
}

}  // namespace
}  // namespace kx

namespace kx {
namespace {

template <typename T>
int matmul_backward(kx_handle *hh, const kx_tensor *a, const kx_tensor *b, const kx_tensor *g, const kx_tensor *da,
                    const kx_tensor *db, kx_error *err) {
    static const char *kOp = "matmul_backward";
    if (!hh) return set_err(err, KX_E_PARAM, kOp, "null handle");
    Handle *h = &hh->impl;
    Span sa, sb, sg;
    int rc = validate_tensor(a, sizeof(T), &sa, err);
    if (rc) return rc;
    rc = validate_tensor(b, sizeof(T), &sb, err);
    if (rc) return rc;
    MatmulPlan pl;
    rc = matmul_shape(a->dims, a->rank, b->dims, b->rank, &pl, err);
    if (rc) return rc;
    rc = validate_tensor(g, sizeof(T), &sg, err);
    if (rc) return rc;
    bool same = g->rank == pl.out_rank;
    for (uint32_t d = 0; same && d < g->rank; ++d) same = g->dims[d] == pl.out_dims[d];
    if (!same) return set_err(err, KX_E_PARAM, kOp, "gradient shape differs from forward output");
    if (da && (rc = check_grad_out<T>(da, a, kOp, err))) return rc;
    if (db && (rc = check_grad_out<T>(db, b, kOp, err))) return rc;
    DeviceGuard guard(h->device);
    if (!guard.ok) return set_err(err, KX_E_NO_DEVICE, kOp, "cannot select device");
    const uint64_t m = pl.m, k = pl.k, n = pl.n;

    // Shared right operand: the leading rows of A and G flatten into one
    // contraction (autograd.rs:636-650).
    if (a->rank > 2 && b->rank <= 2 && k > 0 && n > 0 && rows_collapse(*a) && rows_collapse(*g)) {
        const uint64_t rows = numel(a->dims, a->rank) / k;
        kx_tensor left = *a, seed = *g, right = *b;
        left.rank = 2;
        left.dims[0] = rows;
        left.dims[1] = k;
        left.strides[0] = a->strides[a->rank - 2];
        left.strides[1] = a->strides[a->rank - 1];
        seed.rank = 2;
        seed.dims[0] = rows;
        seed.dims[1] = n;
        if (pl.b_vector) {     // G [.., m] as [rows, 1]
            seed.strides[0] = g->strides[g->rank - 1];
            seed.strides[1] = 0;
            right.rank = 2;
            right.dims[0] = k;
            right.dims[1] = 1;
            right.strides[0] = b->strides[0];
            right.strides[1] = 0;
        } else {
            seed.strides[0] = g->strides[g->rank - 2];
            seed.strides[1] = g->strides[g->rank - 1];
        }
        if (da) {   // [rows, k] = seed [rows, n] . right^T [n, k]
            const uint64_t dd[2] = {rows, k};
            kx_tensor o = dense(static_cast<T *>(da->data) + da->origin, dd, 2);
            kx_tensor rt = swap_last(right);
            if ((rc = MatmulFn<T>::call(hh, &seed, &rt, &o, err))) return rc;
        }
        if (db) {   // [k, n] = left^T [k, rows] . seed [rows, n]
            const uint64_t dd[2] = {k, n};
            kx_tensor o = dense(static_cast<T *>(db->data) + db->origin, dd, 2);
            kx_tensor lt = swap_last(left);
            if ((rc = MatmulFn<T>::call(hh, &lt, &seed, &o, err))) return rc;
        }
        return KX_OK;
    }

    // General case (autograd.rs:651-690): vectors as [1, k] / [k, 1], the seed
    // with the same singleton axes, products over the broadcast batch, summed
    // back to each operand's dims.
    kx_tensor left = *a, right = *b;
    if (pl.a_vector) {
        left.rank = 2;
        left.dims[0] = 1;
        left.dims[1] = k;
        left.strides[0] = 0;
        left.strides[1] = a->strides[0];
    }
    if (pl.b_vector) {
        right.rank = 2;
        right.dims[0] = k;
        right.dims[1] = 1;
        right.strides[0] = b->strides[0];
        right.strides[1] = 0;
    }
    kx_tensor seed = *g;
    {
        const uint32_t br = pl.batch_rank;
        seed.rank = br + 2;
        for (uint32_t d = 0; d < br; ++d) {
            seed.dims[d] = g->dims[d];
            seed.strides[d] = g->strides[d];
        }
        uint32_t gi = br;
        seed.dims[br] = m;
        seed.strides[br] = pl.a_vector ? 0 : g->strides[gi++];
        seed.dims[br + 1] = n;
        seed.strides[br + 1] = pl.b_vector ? 0 : g->strides[gi++];
    }
    // full-shape gradients: batch dims + [m, k] and batch dims + [k, n]
    uint64_t fa[KX_MAX_RANK], fb[KX_MAX_RANK];
    const uint32_t fr = pl.batch_rank + 2;
    for (uint32_t d = 0; d < pl.batch_rank; ++d) fa[d] = fb[d] = pl.batch[d];
    fa[fr - 2] = m;
    fa[fr - 1] = k;
    fb[fr - 2] = k;
    fb[fr - 1] = n;
    // operand dims with vectors as matrices
    uint64_t oa[KX_MAX_RANK], ob[KX_MAX_RANK];
    for (uint32_t d = 0; d < left.rank; ++d) oa[d] = left.dims[d];
    for (uint32_t d = 0; d < right.rank; ++d) ob[d] = right.dims[d];
    auto direct = [&](const uint64_t *full, const uint64_t *op, uint32_t orank) {
        if (orank != fr) return false;
        for (uint32_t d = 0; d < fr; ++d)
            if (full[d] != op[d]) return false;
        return true;
    };
    const bool da_direct = da && direct(fa, oa, left.rank), db_direct = db && direct(fb, ob, right.rank);
    const uint64_t na = numel(fa, fr), nb = numel(fb, fr);
    const uint64_t need = ((da && !da_direct) ? na : 0) + ((db && !db_direct) ? nb : 0);
    T *tmp = nullptr;
    if (need) {
        if ((rc = h->grow(&h->bwd, &h->bwd_bytes, need * sizeof(T)))) return cuda_err(err, h, kOp);
        tmp = static_cast<T *>(h->bwd);
    }
    if (da) {
        T *dst = da_direct ? static_cast<T *>(da->data) + da->origin : tmp;
        kx_tensor o = dense(dst, fa, fr);
        kx_tensor rt = swap_last(right);
        if ((rc = MatmulFn<T>::call(hh, &seed, &rt, &o, err))) return rc;
        if (!da_direct && (rc = reduce_into<T>(h, tmp, fa, fr, da, oa, left.rank))) return cuda_err(err, h, kOp);
    }
    if (db) {
        T *dst = db_direct ? static_cast<T *>(db->data) + db->origin : tmp + ((da && !da_direct) ? na : 0);
        kx_tensor o = dense(dst, fb, fr);
        kx_tensor lt = swap_last(left);
        if ((rc = MatmulFn<T>::call(hh, &lt, &seed, &o, err))) return rc;
        if (!db_direct && (rc = reduce_into<T>(h, dst, fb, fr, db, ob, right.rank))) return cuda_err(err, h, kOp);
    }
    return KX_OK;
}

// ---- conv2d_backward ------------------------------------------------------
// acc + g * v with the product and the sum rounded separately (the reference
// never fuses them; left to itself the compiler would).
__device__ __forceinline__ float mul_add_rn(float acc, float g, float v) { return __fadd_rn(acc, __fmul_rn(g, v)); }
__device__ __forceinline__ double mul_add_rn(double acc, double g, double v) { return __dadd_rn(acc, __dmul_rn(g, v)); }

struct ConvBwdGeom {
    int64_t n, c, ih, iw;          // input
    int64_t co, cg, kh, kw;        // weight
    int64_t oh, ow;                // output
    int64_t sy, sx, py, px, dy, dx, cpg;
    int64_t xs[4], ws[4], gs[4];   // element strides of x, w, dy
};

// dx[n, c, y, x]: for co in the group, then the taps with output positions
// ascending (ky, kx descending), dy[n, co, oy, ox] * w[co, ci, ky, kx]
// added in that order -- the order the reference loop reaches them.
template <typename T>
__global__ void conv_bwd_dx_kernel(const T *__restrict__ w, const T *__restrict__ gy, T *__restrict__ dxo,
                                   const __grid_constant__ ConvBwdGeom g) {
    const int64_t total = g.n * g.c * g.ih * g.iw;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t xx = e % g.iw, y = (e / g.iw) % g.ih, c = (e / (g.iw * g.ih)) % g.c, n = e / (g.iw * g.ih * g.c);
        const int64_t grp = c / g.cg, ci = c % g.cg;
        T acc = T(0);
        for (int64_t co = grp * g.cpg; co < (grp + 1) * g.cpg; ++co) {
            for (int64_t ky = g.kh - 1; ky >= 0; --ky) {
                const int64_t ty = y + g.py - ky * g.dy;
                if (ty < 0 || ty % g.sy) continue;
                const int64_t oy = ty / g.sy;
                if (oy >= g.oh) continue;
                for (int64_t kx = g.kw - 1; kx >= 0; --kx) {
                    const int64_t tx = xx + g.px - kx * g.dx;
                    if (tx < 0 || tx % g.sx) continue;
                    const int64_t ox = tx / g.sx;
                    if (ox >= g.ow) continue;
                    const T gv = gy[n * g.gs[0] + co * g.gs[1] + oy * g.gs[2] + ox * g.gs[3]];
                    const T wv = w[co * g.ws[0] + ci * g.ws[1] + ky * g.ws[2] + kx * g.ws[3]];
                    acc = mul_add_rn(acc, gv, wv);
                }
            }
        }
        dxo[e] = acc;
    }
}

// dw[co, ci, ky, kx]: over (n, oy, ox) in C order, dy * x where the tap is
// inside the padded input.
template <typename T>
__global__ void conv_bwd_dw_kernel(const T *__restrict__ x, const T *__restrict__ gy, T *__restrict__ dwo,
                                   const __grid_constant__ ConvBwdGeom g) {
    const int64_t total = g.co * g.cg * g.kh * g.kw;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t kx = e % g.kw, ky = (e / g.kw) % g.kh, ci = (e / (g.kw * g.kh)) % g.cg, co = e / (g.kw * g.kh * g.cg);
        const int64_t c = (co / g.cpg) * g.cg + ci;
        T acc = T(0);
        for (int64_t n = 0; n < g.n; ++n)
            for (int64_t oy = 0; oy < g.oh; ++oy) {
                const int64_t y = oy * g.sy + ky * g.dy - g.py;
                if (y < 0 || y >= g.ih) continue;
                for (int64_t ox = 0; ox < g.ow; ++ox) {
                    const int64_t xx = ox * g.sx + kx * g.dx - g.px;
                    if (xx < 0 || xx >= g.iw) continue;
                    const T gv = gy[n * g.gs[0] + co * g.gs[1] + oy * g.gs[2] + ox * g.gs[3]];
                    acc = mul_add_rn(acc, gv, x[n * g.xs[0] + c * g.xs[1] + y * g.xs[2] + xx * g.xs[3]]);
                }
            }
        dwo[e] = acc;
    }
}

template <typename T>
int conv2d_backward(kx_handle *hh, const kx_tensor *x, const kx_tensor *w, const kx_tensor *gy,
                    const kx_conv2d_options *o, const kx_tensor *dx, const kx_tensor *dw, kx_error *err) {
    static const char *kOp = "conv2d_backward";
    if (!hh) return set_err(err, KX_E_PARAM, kOp, "null handle");
    Handle *h = &hh->impl;
    Span s;
    int rc = validate_tensor(x, sizeof(T), &s, err);
    if (rc) return rc;
    rc = validate_tensor(w, sizeof(T), &s, err);
    if (rc) return rc;
    uint64_t od[4];
    rc = conv_shape(x->dims, x->rank, w->dims, w->rank, o, od, err);
    if (rc) return rc;
    rc = validate_tensor(gy, sizeof(T), &s, err);
    if (rc) return rc;
    bool same = gy->rank == 4;
    for (int d = 0; same && d < 4; ++d) same = gy->dims[d] == od[d];
    if (!same) return set_err(err, KX_E_PARAM, kOp, "gradient shape differs from forward output");
    if (dx && (rc = check_grad_out<T>(dx, x, kOp, err))) return rc;
    if (dw && (rc = check_grad_out<T>(dw, w, kOp, err))) return rc;
    DeviceGuard guard(h->device);
    if (!guard.ok) return set_err(err, KX_E_NO_DEVICE, kOp, "cannot select device");
    ConvBwdGeom g;
    g.n = (int64_t)x->dims[0];
    g.c = (int64_t)x->dims[1];
    g.ih = (int64_t)x->dims[2];
    g.iw = (int64_t)x->dims[3];
    g.co = (int64_t)w->dims[0];
    g.cg = (int64_t)w->dims[1];
    g.kh = (int64_t)w->dims[2];
    g.kw = (int64_t)w->dims[3];
    g.oh = (int64_t)od[2];
    g.ow = (int64_t)od[3];
    g.sy = (int64_t)o->stride[0];
    g.sx = (int64_t)o->stride[1];
    g.py = (int64_t)o->padding[0];
    g.px = (int64_t)o->padding[1];
    g.dy = (int64_t)o->dilation[0];
    g.dx = (int64_t)o->dilation[1];
    g.cpg = g.co / (int64_t)o->groups;
    for (int d = 0; d < 4; ++d) {
        g.xs[d] = x->dims[d] == 1 ? 0 : x->strides[d];
        g.ws[d] = w->dims[d] == 1 ? 0 : w->strides[d];
        g.gs[d] = gy->dims[d] == 1 ? 0 : gy->strides[d];
    }
    const T *xp = static_cast<const T *>(x->data) + x->origin;
    const T *wp = static_cast<const T *>(w->data) + w->origin;
    const T *gp = static_cast<const T *>(gy->data) + gy->origin;
    const bool empty = numel(od, 4) == 0;
    cudaError_t ce = cudaSuccess;
    auto grid = [&](int64_t total) {
        const int64_t b = (total + 255) / 256;
        return (unsigned)(b < 8 * h->sm_count ? (b > 0 ? b : 1) : 8 * h->sm_count);
    };
    if (dx) {
        T *dp = static_cast<T *>(dx->data) + dx->origin;
        const uint64_t nx = numel(x->dims, 4);
        if (nx) {
            if (empty) ce = cudaMemsetAsync(dp, 0, nx * sizeof(T), h->stream);
            else {
                conv_bwd_dx_kernel<T><<<grid((int64_t)nx), 256, 0, h->stream>>>(wp, gp, dp, g);
                ++h->launches;
                ce = cudaGetLastError();
            }
        }
    }
    if (dw && ce == cudaSuccess) {
        T *dp = static_cast<T *>(dw->data) + dw->origin;
        const uint64_t nw = numel(w->dims, 4);
        if (nw) {
            if (empty) ce = cudaMemsetAsync(dp, 0, nw * sizeof(T), h->stream);
            else {
                conv_bwd_dw_kernel<T><<<grid((int64_t)nw), 256, 0, h->stream>>>(xp, gp, dp, g);
                ++h->launches;
                ce = cudaGetLastError();
            }
        }
    }
    h->last_kernel = "conv_backward_ordered";
    if (ce != cudaSuccess) {
        h->cuda_fail(ce);
        return cuda_err(err, h, kOp);
    }
    return KX_OK;
}

}  // namespace
}  // namespace kx

using namespace kx;

extern "C" {
int kx_matmul_backward_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *grad,
                           const kx_tensor *grad_a, const kx_tensor *grad_b, kx_error *err) {
    return matmul_backward<float>(h, a, b, grad, grad_a, grad_b, err);
}
int kx_matmul_backward_f64(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *grad,
                           const kx_tensor *grad_a, const kx_tensor *grad_b, kx_error *err) {
    return matmul_backward<double>(h, a, b, grad, grad_a, grad_b, err);
}
int kx_conv2d_backward_f32(kx_handle *h, const kx_tensor *input, const kx_tensor *weight, const kx_tensor *grad,
                           const kx_conv2d_options *options, const kx_tensor *grad_input, const kx_tensor *grad_weight,
                           kx_error *err) {
    return conv2d_backward<float>(h, input, weight, grad, options, grad_input, grad_weight, err);
}
int kx_conv2d_backward_f64(kx_handle *h, const kx_tensor *input, const kx_tensor *weight, const kx_tensor *grad,
                           const kx_conv2d_options *options, const kx_tensor *grad_input, const kx_tensor *grad_weight,
                           kx_error *err) {
    return conv2d_backward<double>(h, input, weight, grad, options, grad_input, grad_weight, err);
}
}
