// Host-side validation and shape planning shared by every C-ABI entry point.
// Pure C++ (no CUDA calls): runs without a GPU and is unit-tested on the CPU.
//
// Each function restates one reference check with the same order of failures:
//   span_of / validate_storage  <- kernix-core layout/geometry.rs:40-80 (checked_span)
//                                  and layout/affine.rs:175-199 (validate_storage_len,
//                                  validate_cpu_storage)
//   validate_dims               <- kernix-core shape/utils.rs:3-21 (Kahen::new)
//   broadcast_shape             <- kernix-ops ops/broadcast.rs:6-34
//   matmul_shape                <- kernix-ops ops/linalg.rs:77-119
//   conv_shape / conv_extent    <- kernix-ops neural.rs:49-125
#pragma once
#include <cstdint>
#include <cstring>
#include <cstdio>

#include "../../include/kernix_b200.h"

namespace kx {

using i128 = __int128;
constexpr uint64_t kUsizeMax = UINT64_MAX;
constexpr uint64_t kIsizeMax = (uint64_t)INT64_MAX;

inline int set_err(kx_error *e, int status, const char *op = nullptr, const char *param = nullptr,
                   uint64_t v0 = 0, uint64_t v1 = 0, uint64_t v2 = 0, uint64_t v3 = 0) {
    if (e) {
        std::memset(e, 0, sizeof(*e));
        e->status = status;
        if (op) std::snprintf(e->operation, sizeof(e->operation), "%s", op);
        if (param) std::snprintf(e->parameter, sizeof(e->parameter), "%s", param);
        e->values[0] = v0;
        e->values[1] = v1;
        e->values[2] = v2;
        e->values[3] = v3;
    }
    return status;
}

struct Span {
    bool empty;       // a zero dimension: no element is addressed
    uint64_t start;   // lowest reachable element
    uint64_t end;     // one past the highest reachable element
};

// checked_span: the half-open range of storage elements a layout can address.
inline int span_of(const uint64_t *dims, const int64_t *strides, uint32_t rank, uint64_t origin,
                   Span *out, kx_error *e) {
    for (uint32_t i = 0; i < rank; ++i) {
        if (dims[i] == 0) {
            out->empty = true;
            out->start = out->end = 0;
            return KX_OK;
        }
    }
    i128 lo = (i128)origin, hi = (i128)origin;
    for (uint32_t i = 0; i < rank; ++i) {
        // (2^64-1) * |i64| < 2^127: the product itself never overflows i128.
        i128 contribution = (i128)(dims[i] - 1) * (i128)strides[i];
        i128 *side = contribution < 0 ? &lo : &hi;
        if (__builtin_add_overflow(*side, contribution, side))
            return set_err(e, KX_E_LAYOUT, "layout", "address overflow", KX_LAYOUT_ADDRESS_OVERFLOW);
    }
    if (lo < 0) return set_err(e, KX_E_LAYOUT, "layout", "negative storage offset", KX_LAYOUT_NEGATIVE_STORAGE_OFFSET);
    i128 end = hi + 1;
    if (end > (i128)kUsizeMax) return set_err(e, KX_E_LAYOUT, "layout", "address overflow", KX_LAYOUT_ADDRESS_OVERFLOW);
    out->empty = false;
    out->start = (uint64_t)lo;
    out->end = (uint64_t)end;
    return KX_OK;
}

// validate_cpu_storage: the span fits the available elements and the byte
// extent of the allocation stays within isize::MAX.
inline int validate_storage(const Span &s, uint64_t available, uint32_t elem_bytes, kx_error *e) {
    uint64_t required = s.empty ? 0 : s.end;
    if (available < required)
        return set_err(e, KX_E_LAYOUT, "layout", "storage too small", KX_LAYOUT_STORAGE_TOO_SMALL, required, available);
    i128 bytes = (i128)available * (i128)elem_bytes;
    if (bytes > (i128)kIsizeMax)
        return set_err(e, KX_E_LAYOUT, "layout", "storage byte extent overflow", KX_LAYOUT_BYTE_EXTENT_OVERFLOW);
    return KX_OK;
}

// Kahen::new: a nonzero dimension product must fit usize.
inline int validate_dims(const uint64_t *dims, uint32_t rank, kx_error *e) {
    for (uint32_t i = 0; i < rank; ++i)
        if (dims[i] == 0) return KX_OK;
    uint64_t acc = 1;
    for (uint32_t i = 0; i < rank; ++i) {
        unsigned __int128 next = (unsigned __int128)acc * dims[i];
        if (next > kUsizeMax)
            return set_err(e, KX_E_SHAPE_OVERFLOW, "shape", "element count overflow", i, acc, dims[i]);
        acc = (uint64_t)next;
    }
    return KX_OK;
}

inline uint64_t numel(const uint64_t *dims, uint32_t rank) {
    uint64_t n = 1;
    for (uint32_t i = 0; i < rank; ++i) {
        if (dims[i] == 0) return 0;
        n *= dims[i];
    }
    return n;
}

inline int validate_tensor(const kx_tensor *t, uint32_t elem_bytes, Span *span, kx_error *e) {
    if (!t) return set_err(e, KX_E_PARAM, "tensor", "null descriptor");
    if (t->rank > KX_MAX_RANK) return set_err(e, KX_E_UNSUPPORTED, "tensor", "rank above KX_MAX_RANK", t->rank);
    int rc = validate_dims(t->dims, t->rank, e);
    if (rc) return rc;
    Span s;
    rc = span_of(t->dims, t->strides, t->rank, t->origin, &s, e);
    if (rc) return rc;
    rc = validate_storage(s, t->storage_len, elem_bytes, e);
    if (rc) return rc;
    if (!s.empty && !t->data) return set_err(e, KX_E_PARAM, "tensor", "null data pointer for a nonempty tensor");
    if (t->data && (reinterpret_cast<uintptr_t>(t->data) % elem_bytes) != 0)
        return set_err(e, KX_E_LAYOUT, "layout", "misaligned data pointer", KX_LAYOUT_MISALIGNED_POINTER);
    if (span) *span = s;
    return KX_OK;
}

// is_c_contiguous (layout/geometry.rs:111-137): singleton strides are ignored.
inline bool is_c_contiguous(const kx_tensor *t) {
    for (uint32_t i = 0; i < t->rank; ++i)
        if (t->dims[i] == 0) return true;
    unsigned __int128 expected = 1;
    for (int i = (int)t->rank - 1; i >= 0; --i) {
        if (t->dims[i] <= 1) continue;
        if (t->strides[i] <= 0 || (unsigned __int128)t->strides[i] != expected) return false;
        expected *= t->dims[i];
    }
    return true;
}

// Byte ranges of two validated spans overlap.
inline bool spans_overlap(const void *pa, const Span &a, const void *pb, const Span &b, uint32_t es) {
    if (a.empty || b.empty) return false;
    uintptr_t a0 = reinterpret_cast<uintptr_t>(pa) + a.start * es, a1 = reinterpret_cast<uintptr_t>(pa) + a.end * es;
    uintptr_t b0 = reinterpret_cast<uintptr_t>(pb) + b.start * es, b1 = reinterpret_cast<uintptr_t>(pb) + b.end * es;
    return a0 < b1 && b0 < a1;
}

// broadcast_shape: right-aligned NumPy broadcasting; 0 with 1 gives 0.
inline int broadcast_shape(const uint64_t *l, uint32_t lr, const uint64_t *r, uint32_t rr,
                           uint64_t *out, uint32_t *out_rank, kx_error *e) {
    uint32_t rank = lr > rr ? lr : rr;
    for (uint32_t axis = 0; axis < rank; ++axis) {
        uint64_t a = (axis + lr >= rank) ? l[axis + lr - rank] : 1;
        uint64_t b = (axis + rr >= rank) ? r[axis + rr - rank] : 1;
        uint64_t dim;
        if (a == b || b == 1) dim = a;
        else if (a == 1) dim = b;
        else return set_err(e, KX_E_BROADCAST, "matmul", "batch broadcast", axis, a, b);
        out[axis] = dim;
    }
    *out_rank = rank;
    return KX_OK;
}

// Everything the device launch needs, derived from the two operand shapes.
struct MatmulPlan {
    bool a_vector, b_vector;
    uint32_t a_batch_rank, b_batch_rank;
    uint64_t m, k, n;
    uint32_t batch_rank;
    uint64_t batch[KX_MAX_RANK];
    uint32_t out_rank;
    uint64_t out_dims[KX_MAX_RANK];
};

// matmul_impl's validation prefix, in the reference order: rank-0 left,
// rank-0 right, contraction mismatch, batch broadcast, output shape overflow.
inline int matmul_shape(const uint64_t *a, uint32_t ar, const uint64_t *b, uint32_t br, MatmulPlan *p,
                        kx_error *e) {
    if (ar == 0) return set_err(e, KX_E_INVALID_RANK, "matmul", "rank", 1, 0);
    if (br == 0) return set_err(e, KX_E_INVALID_RANK, "matmul", "rank", 1, 0);
    if (ar > KX_MAX_RANK || br > KX_MAX_RANK)
        return set_err(e, KX_E_UNSUPPORTED, "matmul", "rank above KX_MAX_RANK", ar > br ? ar : br);
    p->a_vector = ar == 1;
    p->b_vector = br == 1;
    p->a_batch_rank = p->a_vector ? 0 : ar - 2;
    p->b_batch_rank = p->b_vector ? 0 : br - 2;
    p->m = p->a_vector ? 1 : a[ar - 2];
    p->k = a[ar - 1];
    uint64_t kb = p->b_vector ? b[0] : b[br - 2];
    p->n = p->b_vector ? 1 : b[br - 1];
    if (p->k != kb) return set_err(e, KX_E_CONTRACT, "matmul", "contracted dimensions", p->k, kb);
    int rc = broadcast_shape(a, p->a_batch_rank, b, p->b_batch_rank, p->batch, &p->batch_rank, e);
    if (rc) return rc;
    uint32_t r = 0;
    for (uint32_t i = 0; i < p->batch_rank; ++i) p->out_dims[r++] = p->batch[i];
    if (!p->a_vector) p->out_dims[r++] = p->m;
    if (!p->b_vector) p->out_dims[r++] = p->n;
    if (r > KX_MAX_RANK) return set_err(e, KX_E_UNSUPPORTED, "matmul", "output rank above KX_MAX_RANK", r);
    p->out_rank = r;
    return validate_dims(p->out_dims, r, e);
}

// extent (neural.rs:57-83): one spatial output extent, or 0 when the effective
// kernel exceeds the padded input.
inline int conv_extent(uint64_t size, uint64_t kernel, uint64_t stride, uint64_t padding, uint64_t dilation,
                       uint64_t *out, kx_error *e) {
    if (kernel == 0 || stride == 0 || dilation == 0)
        return set_err(e, KX_E_PARAM, "spatial geometry", "kernel, stride and dilation must be positive");
    unsigned __int128 effective = (unsigned __int128)(kernel - 1) * dilation + 1;
    if (effective > kUsizeMax) return set_err(e, KX_E_DIM_OVERFLOW, "conv2d", "dimension overflow", 2);
    unsigned __int128 padded = (unsigned __int128)padding * 2;
    if (padded > kUsizeMax) return set_err(e, KX_E_DIM_OVERFLOW, "conv2d", "dimension overflow", 2);
    padded += size;
    if (padded > kUsizeMax) return set_err(e, KX_E_DIM_OVERFLOW, "conv2d", "dimension overflow", 2);
    *out = (padded < effective) ? 0 : (uint64_t)((padded - effective) / stride + 1);
    return KX_OK;
}

// ConvGeometry::new (neural.rs:91-125).
inline int conv_shape(const uint64_t *in, uint32_t in_rank, const uint64_t *w, uint32_t w_rank,
                      const kx_conv2d_options *o, uint64_t *out, kx_error *e) {
    int rc = validate_dims(in, in_rank, e);
    if (rc) return rc;
    if (in_rank != 4) return set_err(e, KX_E_EXACT_RANK, "conv2d", "rank", 4, in_rank);
    rc = validate_dims(w, w_rank, e);
    if (rc) return rc;
    if (w_rank != 4) return set_err(e, KX_E_EXACT_RANK, "conv2d weights", "rank", 4, w_rank);
    if (!o) return set_err(e, KX_E_PARAM, "conv2d", "null options");
    uint64_t n = in[0], ci = in[1], h = in[2], wd = in[3];
    uint64_t co = w[0], cg = w[1], kh = w[2], kw = w[3];
    uint64_t g = o->groups;
    if (g == 0 || ci == 0 || co == 0 || ci % g != 0 || co % g != 0 || cg != ci / g)
        return set_err(e, KX_E_PARAM, "conv2d", "groups and input/output channels must agree");
    uint64_t oh, ow;
    rc = conv_extent(h, kh, o->stride[0], o->padding[0], o->dilation[0], &oh, e);
    if (rc) return rc;
    rc = conv_extent(wd, kw, o->stride[1], o->padding[1], o->dilation[1], &ow, e);
    if (rc) return rc;
    out[0] = n;
    out[1] = co;
    out[2] = oh;
    out[3] = ow;
    return validate_dims(out, 4, e);
}

}  // namespace kx
