// tensordot lowered to one GEMM on device memory.
//
// tensordot (crates/kernix-ops/src/ops/linalg_extra.rs:164-276) contracts
// pairs of axes: every output element (left free axes, then right free axes,
// C order) is the sum over the contraction index space, in C order over the
// contracted extents taken in pairing order, of left * right.  That is a
// matrix product of A' [M = free(left), K = contracted] and B' [K, N =
// free(right)] whose k index runs in exactly that order, so the forward GEMM
// kernels compute it; in ordered mode (kx_set_ordered_matmul) they add
// a * b in increasing k with separate rounding, the reference loop's sums bit
// for bit.  A' and B' are strided views when the free axes and the contracted
// axes each nest into one stride (the common case: adjacent axes of a
// contiguous tensor, including transposed or sliced views); otherwise the
// operand is first gathered into a contiguous buffer in that axis order.
#include <cstring>

#include "kx_internal.hpp"

extern "C" int kx_matmul_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out,
                             kx_error *err);
extern "C" int kx_matmul_f64(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out,
                             kx_error *err);

namespace kx {
namespace {

struct PermGeom {
    int rank;
    int64_t dims[KX_MAX_RANK];      // in the new axis order
    int64_t str[KX_MAX_RANK];       // source strides in the new axis order
    int64_t total;
};

// dst (contiguous, new axis order) = src read through its strides.
template <typename T>
__global__ void permute_copy_kernel(const T *__restrict__ src, T *__restrict__ dst, const __grid_constant__ PermGeom g) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < g.total; e += (int64_t)gridDim.x * blockDim.x) {
        int64_t rem = e, off = 0;
        for (int d = g.rank - 1; d >= 0; --d) {
            off += (rem % g.dims[d]) * g.str[d];
            rem /= g.dims[d];
        }
        dst[e] = src[off];
    }
}

// Product of the extents of `axes` (outermost first) and, when the flat
// index over them maps to one stride -- every non-singleton axis's stride is
// the innermost one times the extents inside it -- that stride (0 if all are
// singletons).  An empty extent makes the product 0 with any stride.
bool merge_axes(const kx_tensor *t, const int *axes, int n, uint64_t *extent, int64_t *stride) {
    uint64_t e = 1;
    int64_t s = 0;
    bool have = false;
    for (int i = n - 1; i >= 0; --i) {
        const uint64_t d = t->dims[axes[i]];
        if (d == 0) {
            *extent = 0;
            *stride = 0;
            return true;
        }
        if (d != 1) {
            if (!have) {
                s = t->strides[axes[i]];
                have = true;
            } else if (t->strides[axes[i]] != s * (int64_t)e) {
                return false;
            }
        }
        e *= d;
    }
    *extent = e;
    *stride = have ? s : 0;
    return true;
}

template <typename T>
int tensordot(kx_handle *hh, const kx_tensor *a, const kx_tensor *b, const int64_t *a_axes, uint32_t na,
              const int64_t *b_axes, uint32_t nb, const kx_tensor *out, kx_error *err) {
    static const char *kOp = "tensordot";
    if (!hh) return set_err(err, KX_E_PARAM, kOp, "null handle");
    Handle *h = &hh->impl;
    Span sa, sb, so;
    int rc = validate_tensor(a, sizeof(T), &sa, err);
    if (rc) return rc;
    rc = validate_tensor(b, sizeof(T), &sb, err);
    if (rc) return rc;
    if (na != nb) return set_err(err, KX_E_AXES_MISMATCH, kOp, "contraction axis counts", na, nb);
    if (na && (!a_axes || !b_axes)) return set_err(err, KX_E_PARAM, kOp, "null axis list");
    bool cl[KX_MAX_RANK] = {}, cr[KX_MAX_RANK] = {};
    int axl[KX_MAX_RANK], axr[KX_MAX_RANK];
    for (uint32_t i = 0; i < na; ++i) {
        int64_t l = a_axes[i] < 0 ? a_axes[i] + (int64_t)a->rank : a_axes[i];
        if (l < 0 || l >= (int64_t)a->rank)
            return set_err(err, KX_E_AXIS, kOp, "axis", (uint64_t)a_axes[i], a->rank);
        int64_t r = b_axes[i] < 0 ? b_axes[i] + (int64_t)b->rank : b_axes[i];
        if (r < 0 || r >= (int64_t)b->rank)
            return set_err(err, KX_E_AXIS, kOp, "axis", (uint64_t)b_axes[i], b->rank);
        if (cl[l] || cr[r]) return set_err(err, KX_E_DUPLICATE_AXIS, kOp, "duplicate axis", cl[l] ? l : r);
        if (a->dims[l] != b->dims[r])
            return set_err(err, KX_E_CONTRACT, kOp, "contracted dimensions", a->dims[l], b->dims[r]);
        cl[l] = cr[r] = true;
        axl[i] = (int)l;
        axr[i] = (int)r;
    }
    int fl[KX_MAX_RANK], fr[KX_MAX_RANK], nfl = 0, nfr = 0;
    uint64_t od[2 * KX_MAX_RANK];
    uint32_t orank = 0;
    for (uint32_t i = 0; i < a->rank; ++i)
        if (!cl[i]) { fl[nfl++] = (int)i; od[orank++] = a->dims[i]; }
    for (uint32_t i = 0; i < b->rank; ++i)
        if (!cr[i]) { fr[nfr++] = (int)i; od[orank++] = b->dims[i]; }
    if (orank > KX_MAX_RANK) return set_err(err, KX_E_UNSUPPORTED, kOp, "output rank above KX_MAX_RANK", orank);
    rc = validate_dims(od, orank, err);
    if (rc) return rc;
    rc = validate_tensor(out, sizeof(T), &so, err);
    if (rc) return rc;
    bool same = out->rank == orank;
    for (uint32_t d = 0; same && d < orank; ++d) same = out->dims[d] == od[d];
    if (!same) return set_err(err, KX_E_LAYOUT, kOp, "output shape mismatch", KX_LAYOUT_OUTPUT_SHAPE_MISMATCH);
    if (!is_c_contiguous(out))
        return set_err(err, KX_E_LAYOUT, kOp, "output must be C-contiguous", KX_LAYOUT_OUTPUT_NOT_C_CONTIGUOUS);
    if (spans_overlap(out->data, so, a->data, sa, sizeof(T)) || spans_overlap(out->data, so, b->data, sb, sizeof(T)))
        return set_err(err, KX_E_ALIAS, kOp, "output overlaps an input");
    if (numel(od, orank) == 0) return KX_OK;
    DeviceGuard guard(h->device);
    if (!guard.ok) return set_err(err, KX_E_NO_DEVICE, kOp, "cannot select device");

    // A' [M, K] over (free(left), contracted); B' [K, N] over (contracted, free(right))
    uint64_t m, k, kb, n;
    int64_t sm, sk, skb, sn;
    const bool a_view = merge_axes(a, fl, nfl, &m, &sm) && merge_axes(a, axl, (int)na, &k, &sk);
    const bool b_view = merge_axes(b, axr, (int)nb, &kb, &skb) && merge_axes(b, fr, nfr, &n, &sn);
    m = k = n = 1;
    for (int i = 0; i < nfl; ++i) m *= a->dims[fl[i]];
    for (uint32_t i = 0; i < na; ++i) k *= a->dims[axl[i]];
    for (int i = 0; i < nfr; ++i) n *= b->dims[fr[i]];
    const uint64_t need = (a_view ? 0 : m * k) + (b_view ? 0 : k * n);
    T *buf = nullptr;
    if (need) {
        if ((rc = h->grow(&h->perm, &h->perm_bytes, need * sizeof(T)))) return cuda_err(err, h, kOp);
        buf = static_cast<T *>(h->perm);
    }
    auto gather = [&](const kx_tensor *t, const int *first, int nf, const int *second, int ns, T *dst) -> int {
        PermGeom g;
        std::memset(&g, 0, sizeof(g));
        g.rank = nf + ns;
        g.total = 1;
        for (int i = 0; i < nf; ++i) {
            g.dims[i] = (int64_t)t->dims[first[i]];
            g.str[i] = t->strides[first[i]];
        }
        for (int i = 0; i < ns; ++i) {
            g.dims[nf + i] = (int64_t)t->dims[second[i]];
            g.str[nf + i] = t->strides[second[i]];
        }
        for (int d = 0; d < g.rank; ++d) g.total *= g.dims[d];
        if (g.rank == 0) {
            g.rank = 1;
            g.dims[0] = 1;
        }
        const T *src = static_cast<const T *>(t->data) + t->origin;
        const int64_t blocks = (g.total + 255) / 256 < 8 * h->sm_count ? (g.total + 255) / 256 : 8 * h->sm_count;
        permute_copy_kernel<T><<<(unsigned)(blocks > 0 ? blocks : 1), 256, 0, h->stream>>>(src, dst, g);
        ++h->launches;
        cudaError_t ce = cudaGetLastError();
        return ce == cudaSuccess ? KX_OK : h->cuda_fail(ce);
    };
    kx_tensor A, B, O;
    std::memset(&A, 0, sizeof(A));
    std::memset(&B, 0, sizeof(B));
    A.rank = B.rank = 2;
    A.dims[0] = m;
    A.dims[1] = k;
    B.dims[0] = k;
    B.dims[1] = n;
    if (a_view) {
        A.data = a->data;
        A.storage_len = a->storage_len;
        A.origin = a->origin;
        A.strides[0] = sm;
        A.strides[1] = sk;
    } else {
        if ((rc = gather(a, fl, nfl, axl, (int)na, buf))) return cuda_err(err, h, kOp);
        A.data = buf;
        A.storage_len = m * k;
        A.strides[0] = (int64_t)k;
        A.strides[1] = 1;
    }
    if (b_view) {
        B.data = b->data;
        B.storage_len = b->storage_len;
        B.origin = b->origin;
        B.strides[0] = skb;
        B.strides[1] = sn;
    } else {
        T *dst = buf + (a_view ? 0 : m * k);
        if ((rc = gather(b, axr, (int)nb, fr, nfr, dst))) return cuda_err(err, h, kOp);
        B.data = dst;
        B.storage_len = k * n;
        B.strides[0] = (int64_t)n;
        B.strides[1] = 1;
    }
    O = *out;
    O.rank = 2;
    O.dims[0] = m;
    O.dims[1] = n;
    O.strides[0] = (int64_t)n;
    O.strides[1] = 1;
    if constexpr (sizeof(T) == 4) return kx_matmul_f32(hh, &A, &B, &O, err);
    else return kx_matmul_f64(hh, &A, &B, &O, err);
}

}  // namespace
}  // namespace kx

extern "C" {
int kx_tensordot_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const int64_t *a_axes, uint32_t na,
                     const int64_t *b_axes, uint32_t nb, const kx_tensor *out, kx_error *err) {
    return kx::tensordot<float>(h, a, b, a_axes, na, b_axes, nb, out, err);
}
int kx_tensordot_f64(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const int64_t *a_axes, uint32_t na,
                     const int64_t *b_axes, uint32_t nb, const kx_tensor *out, kx_error *err) {
    return kx::tensordot<double>(h, a, b, a_axes, na, b_axes, nb, out, err);
}
}
