// kernix_b200.hpp -- C++ host mirror of Kernix's matmul plug points over the C ABI.
//
// Header-only.  Names and contracts follow the reference crate so host code
// (and tests) read like Kernix's own:
//   kernix::MatmulElement<T>::try_dense_matmul / try_strided_matmul
//                                  crates/kernix-ops/src/ops/matmul_element.rs:14-44
//   kernix::MatrixInput<T>         crates/kernix-ops/src/ops/matmul_element.rs:262-317
//   kernix::CudaExecutor           the Device<T> + MatmulDevice<T> backend
//                                  (crates/kernix-core/src/device.rs:22-35,
//                                   crates/kernix-ops/src/execution.rs:25-36)
//   kernix::DeviceTensor<T>        Tensor<T, Kahen, Buffer> with an opaque device buffer
//                                  and an affine layout (dims, signed strides, origin)
//   kernix::OpsError               crates/kernix-ops/src/ops/error.rs:8-140
//   kernix::CudaConfig / Context   the [cuda] table of kernix::config (config.rs:28-40, 133-137)
//   CudaExecutor::{softmax, softmax_temperature, attention, tensordot,
//                  matmul_backward, conv2d_backward, matmul_into}
//                                  math.rs:531-536, math_extra.rs:544-557,
//                                  linalg_extra.rs:164-276, autograd.rs:622-690,
//                                  neural.rs:379-430, execution.rs:149-240
//   kernix::shard_window / row_piece   the work split across the GPUs of a node
//   kernix::gemm_sharded           one process over several GPUs (kx_gemm_sharded_f32)
// Errors are exceptions carrying the C ABI's kx_error record; hooks return bool
// exactly like the reference (false => nothing written).
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

#include "kernix_b200.h"

namespace kernix {

// OpsError: the C status plus the variant's fields (kx_error::values).
class OpsError : public std::runtime_error {
  public:
    explicit OpsError(int status, const kx_error &e = kx_error{})
        : std::runtime_error(std::string(kx_status_name(status)) + (e.operation[0] ? ": " : "") + e.operation +
                             (e.parameter[0] ? std::string(" (") + e.parameter + ")" : std::string())),
          status_(status), record_(e) {}
    int status() const { return status_; }
    const kx_error &record() const { return record_; }

  private:
    int status_;
    kx_error record_;
};

inline void check(int rc, const kx_error &e) {
    if (rc != KX_OK) throw OpsError(rc, e);
}

namespace detail {
template <typename T> struct Fns;
template <> struct Fns<float> {
    static constexpr auto dense = kx_try_dense_matmul_f32;
    static constexpr auto strided = kx_try_strided_matmul_f32;
    static constexpr auto matmul = kx_matmul_f32;
    static constexpr auto conv2d = kx_conv2d_f32;
    static constexpr auto softmax = kx_softmax_f32;
    static constexpr auto softmax_temperature = kx_softmax_temperature_f32;
    static constexpr auto tensordot = kx_tensordot_f32;
    static constexpr auto matmul_backward = kx_matmul_backward_f32;
    static constexpr auto conv2d_backward = kx_conv2d_backward_f32;
};
template <> struct Fns<double> {
    static constexpr auto dense = kx_try_dense_matmul_f64;
    static constexpr auto strided = kx_try_strided_matmul_f64;
    static constexpr auto matmul = kx_matmul_f64;
    static constexpr auto conv2d = kx_conv2d_f64;
    static constexpr auto softmax = kx_softmax_f64;
    static constexpr auto softmax_temperature = kx_softmax_temperature_f64;
    static constexpr auto tensordot = kx_tensordot_f64;
    static constexpr auto matmul_backward = kx_matmul_backward_f64;
    static constexpr auto conv2d_backward = kx_conv2d_backward_f64;
};
}  // namespace detail

// Validated borrowed rank-two host matrix (MatrixInput::new): the span is
// checked against the storage and singleton strides are normalised to zero.
template <typename T>
class MatrixInput {
  public:
    static MatrixInput create(const T *data, size_t len, std::array<size_t, 2> dims,
                              std::array<std::ptrdiff_t, 2> strides, size_t origin) {
        kx_matrix m{data, len, {dims[0], dims[1]}, {strides[0], strides[1]}, origin};
        kx_error e{};
        check(kx_matrix_validate(&m, sizeof(T), &e), e);
        for (int axis = 0; axis < 2; ++axis)
            if (dims[axis] <= 1) m.strides[axis] = 0;
        return MatrixInput(m);
    }
    std::array<size_t, 2> dims() const { return {m_.dims[0], m_.dims[1]}; }
    std::array<std::ptrdiff_t, 2> strides() const { return {m_.strides[0], m_.strides[1]}; }
    const T *storage() const { return static_cast<const T *>(m_.data); }
    size_t origin() const { return m_.origin; }
    const kx_matrix &raw() const { return m_; }

  private:
    explicit MatrixInput(const kx_matrix &m) : m_(m) {}
    kx_matrix m_;
};

// The [cuda] table of a configuration (kx_cuda_config); defaults as an
// absent table: device 0, automatic kernel families, native products.
struct CudaConfig {
    kx_cuda_config c;
    CudaConfig() { kx_cuda_config_default(&c); }
};

// One handle per device; movable, not copyable.
class Handle {
  public:
    explicit Handle(int device = 0) {
        kx_error e{};
        check(kx_create(device, &h_, &e), e);
    }
    // Context::new for the [cuda] table: every key is validated before any
    // device work (OpsError with KX_E_PARAM naming the key).
    explicit Handle(const CudaConfig &cfg) {
        kx_error e{};
        check(kx_context_create(&cfg.c, &h_, &e), e);
    }
    ~Handle() { kx_destroy(h_); }
    Handle(const Handle &) = delete;
    Handle &operator=(const Handle &) = delete;
    Handle(Handle &&o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    kx_handle *get() const { return h_; }
    CudaConfig config() const {
        CudaConfig cfg;
        kx_handle_config(h_, &cfg.c);
        return cfg;
    }

  private:
    kx_handle *h_ = nullptr;
};

// Work split across the GPUs of one node (kx_shard_window, kx_row_piece).
inline std::pair<uint64_t, uint64_t> shard_window(uint64_t total, uint32_t rank, uint32_t world) {
    uint64_t start = 0, count = 0;
    check(kx_shard_window(total, rank, world, &start, &count), kx_error{});
    return {start, count};
}
inline std::pair<uint64_t, uint64_t> row_piece(uint64_t m, uint32_t world, uint64_t target) {
    uint64_t piece = 0, pieces = 0;
    check(kx_row_piece(m, world, target, &piece, &pieces), kx_error{});
    return {piece, pieces};
}

// MatmulElement hooks on HOST buffers.  The handle is the device the product
// runs on; false means nothing was written.
template <typename T>
struct MatmulElement {
    static_assert(std::is_same<T, float>::value || std::is_same<T, double>::value, "f32 and f64 only");
    static constexpr bool HAS_NATIVE_MATMUL = true;
    static bool try_dense_matmul(const Handle &h, const T *a, size_t a_len, const T *b, size_t b_len, T *out,
                                 size_t out_len, size_t m, size_t k, size_t n) {
        return detail::Fns<T>::dense(h.get(), a, a_len, b, b_len, out, out_len, m, k, n) == KX_OK;
    }
    static bool try_strided_matmul(const Handle &h, const MatrixInput<T> &a, const MatrixInput<T> &b, T *out,
                                   size_t out_len) {
        return detail::Fns<T>::strided(h.get(), &a.raw(), &b.raw(), out, out_len) == KX_OK;
    }
};

// Device buffer shared by views.
template <typename T>
class DeviceBuffer {
  public:
    DeviceBuffer(kx_handle *h, size_t len) : h_(h), len_(len) {
        kx_error e{};
        check(kx_alloc(h, len * sizeof(T), &ptr_, &e), e);
    }
    ~DeviceBuffer() { kx_free(h_, ptr_); }
    DeviceBuffer(const DeviceBuffer &) = delete;
    DeviceBuffer &operator=(const DeviceBuffer &) = delete;
    T *data() const { return static_cast<T *>(ptr_); }
    size_t len() const { return len_; }
    kx_handle *owner() const { return h_; }

  private:
    kx_handle *h_;
    void *ptr_ = nullptr;
    size_t len_;
};

// Tensor<T, Kahen, DeviceBuffer>: an affine layout over a shared device buffer.
template <typename T>
class DeviceTensor {
  public:
    DeviceTensor(std::shared_ptr<DeviceBuffer<T>> buf, std::vector<uint64_t> dims, std::vector<int64_t> strides,
                 uint64_t origin)
        : buf_(std::move(buf)), dims_(std::move(dims)), strides_(std::move(strides)), origin_(origin) {}
    const std::vector<uint64_t> &dims() const { return dims_; }
    const std::vector<int64_t> &strides() const { return strides_; }
    uint64_t origin() const { return origin_; }
    const std::shared_ptr<DeviceBuffer<T>> &buffer() const { return buf_; }
    kx_tensor desc() const {
        kx_tensor t{};
        t.data = buf_->data();
        t.storage_len = buf_->len();
        t.origin = origin_;
        t.rank = static_cast<uint32_t>(dims_.size());
        for (size_t i = 0; i < dims_.size() && i < KX_MAX_RANK; ++i) {
            t.dims[i] = dims_[i];
            t.strides[i] = strides_[i];
        }
        return t;
    }
    // Layout::swap_axes (layout/affine.rs:247-255): no data movement.
    DeviceTensor swap_axes(size_t a, size_t b) const {
        auto d = dims_;
        auto s = strides_;
        std::swap(d.at(a), d.at(b));
        std::swap(s.at(a), s.at(b));
        return DeviceTensor(buf_, d, s, origin_);
    }
    DeviceTensor transpose() const { return swap_axes(0, 1); }
    // Layout::reverse_axis (layout/affine.rs:270-292): negative stride, moved origin.
    DeviceTensor reverse_axis(size_t axis) const {
        auto s = strides_;
        uint64_t origin = origin_;
        if (dims_.at(axis) > 1) {
            origin = (uint64_t)((int64_t)origin + (int64_t)(dims_[axis] - 1) * s[axis]);
            s[axis] = -s[axis];
        }
        return DeviceTensor(buf_, dims_, s, origin);
    }

  private:
    std::shared_ptr<DeviceBuffer<T>> buf_;
    std::vector<uint64_t> dims_;
    std::vector<int64_t> strides_;
    uint64_t origin_;
};

// Device<T> + MatmulDevice<T> for one GPU.  Transfers are synchronous and in
// physical order; matmul never changes devices or layouts behind the caller.
class CudaExecutor {
  public:
    explicit CudaExecutor(int device = 0) : h_(device), device_(device) {}
    // A context's executor: the [cuda] table's device, kernel families and
    // ordered mode (Context::new, config.rs:133-137).
    explicit CudaExecutor(const CudaConfig &cfg) : h_(cfg), device_(cfg.c.device) {}
    const char *name() const { return "cuda"; }
    int device() const { return device_; }
    kx_handle *handle() const { return h_.get(); }
    CudaExecutor &with_ordered_matmul(bool ordered) {
        kx_set_ordered_matmul(h_.get(), ordered ? 1 : 0);
        return *this;
    }
    bool ordered_matmul() const { return kx_ordered_matmul(h_.get()) != 0; }

    template <typename T>
    DeviceTensor<T> upload(const std::vector<T> &values, std::vector<uint64_t> dims) const {
        auto buf = std::make_shared<DeviceBuffer<T>>(h_.get(), values.size());
        kx_error e{};
        check(kx_upload(h_.get(), buf->data(), values.data(), values.size() * sizeof(T), &e), e);
        std::vector<int64_t> strides(dims.size());
        int64_t acc = 1;
        for (size_t i = dims.size(); i-- > 0;) {
            strides[i] = acc;
            acc *= (int64_t)dims[i];
        }
        return DeviceTensor<T>(buf, std::move(dims), std::move(strides), 0);
    }
    // Physical buffer contents (download, device.rs:31-32); rejects buffers of another context.
    template <typename T>
    std::vector<T> download(const DeviceTensor<T> &t) const {
        if (t.buffer()->owner() != h_.get()) throw OpsError(KX_E_PARAM);
        std::vector<T> out(t.buffer()->len());
        kx_error e{};
        check(kx_download(h_.get(), out.data(), t.buffer()->data(), out.size() * sizeof(T), &e), e);
        return out;
    }
    void synchronize() const {
        kx_error e{};
        check(kx_synchronize(h_.get(), &e), e);
    }
    // A fresh C-order device tensor of `dims` (Kernix allocates every result so).
    template <typename T>
    DeviceTensor<T> empty(std::vector<uint64_t> dims) const {
        size_t n = 1;
        for (auto d : dims) n *= d;
        auto buf = std::make_shared<DeviceBuffer<T>>(h_.get(), n ? n : 1);
        std::vector<int64_t> strides(dims.size());
        int64_t acc = 1;
        for (size_t i = dims.size(); i-- > 0;) {
            strides[i] = acc;
            acc *= (int64_t)(dims[i] ? dims[i] : 1);
        }
        return DeviceTensor<T>(buf, std::move(dims), std::move(strides), 0);
    }
    // MatmulDevice::matmul: NumPy matmul semantics into a fresh C-order tensor.
    template <typename T>
    DeviceTensor<T> matmul(const DeviceTensor<T> &a, const DeviceTensor<T> &b) const {
        kx_error e{};
        uint32_t rank = 0;
        uint64_t od[KX_MAX_RANK];
        check(kx_matmul_shape(a.dims().data(), (uint32_t)a.dims().size(), b.dims().data(),
                              (uint32_t)b.dims().size(), &rank, od, &e),
              e);
        auto out = empty<T>(std::vector<uint64_t>(od, od + rank));
        matmul_into(a, b, out);
        return out;
    }
    // CpuExecutor::matmul_into's contract: the caller's C-contiguous output is
    // reused, nothing allocated (execution.rs:149-240).
    template <typename T>
    void matmul_into(const DeviceTensor<T> &a, const DeviceTensor<T> &b, const DeviceTensor<T> &out) const {
        kx_error e{};
        kx_tensor da = a.desc(), db = b.desc(), dc = out.desc();
        check(detail::Fns<T>::matmul(h_.get(), &da, &db, &dc, &e), e);
    }
    // softmax (math.rs:531-536) and softmax_temperature (math_extra.rs:544-557).
    template <typename T>
    DeviceTensor<T> softmax(const DeviceTensor<T> &src, int64_t axis) const {
        auto out = empty<T>(src.dims());
        kx_error e{};
        kx_tensor ds = src.desc(), dout = out.desc();
        check(detail::Fns<T>::softmax(h_.get(), &ds, axis, &dout, &e), e);
        return out;
    }
    template <typename T>
    DeviceTensor<T> softmax_temperature(const DeviceTensor<T> &src, int64_t axis, T temperature) const {
        auto out = empty<T>(src.dims());
        kx_error e{};
        kx_tensor ds = src.desc(), dout = out.desc();
        check(detail::Fns<T>::softmax_temperature(h_.get(), &ds, axis, temperature, &dout, &e), e);
        return out;
    }
    // matmul(softmax_temperature(matmul(q, kt), -1, t), v) in one call (f32).
    DeviceTensor<float> attention(const DeviceTensor<float> &q, const DeviceTensor<float> &kt,
                                  const DeviceTensor<float> &v, float temperature) const {
        kx_error e{};
        uint32_t r1 = 0, r2 = 0;
        uint64_t sd[KX_MAX_RANK], od[KX_MAX_RANK];
        check(kx_matmul_shape(q.dims().data(), (uint32_t)q.dims().size(), kt.dims().data(),
                              (uint32_t)kt.dims().size(), &r1, sd, &e),
              e);
        check(kx_matmul_shape(sd, r1, v.dims().data(), (uint32_t)v.dims().size(), &r2, od, &e), e);
        auto out = empty<float>(std::vector<uint64_t>(od, od + r2));
        kx_tensor dq = q.desc(), dk = kt.desc(), dv = v.desc(), dout = out.desc();
        check(kx_attention_f32(h_.get(), &dq, &dk, &dv, temperature, &dout, &e), e);
        return out;
    }
    // tensordot (linalg_extra.rs:164-276): a's free axes, then b's.
    template <typename T>
    DeviceTensor<T> tensordot(const DeviceTensor<T> &a, const DeviceTensor<T> &b, const std::vector<int64_t> &a_axes,
                              const std::vector<int64_t> &b_axes) const {
        std::vector<bool> ca(a.dims().size()), cb(b.dims().size());
        for (auto x : a_axes) {
            const int64_t i = x < 0 ? x + (int64_t)ca.size() : x;
            if (i >= 0 && i < (int64_t)ca.size()) ca[i] = true;
        }
        for (auto x : b_axes) {
            const int64_t i = x < 0 ? x + (int64_t)cb.size() : x;
            if (i >= 0 && i < (int64_t)cb.size()) cb[i] = true;
        }
        std::vector<uint64_t> dims;
        for (size_t i = 0; i < ca.size(); ++i)
            if (!ca[i]) dims.push_back(a.dims()[i]);
        for (size_t i = 0; i < cb.size(); ++i)
            if (!cb[i]) dims.push_back(b.dims()[i]);
        auto out = empty<T>(dims.size() <= KX_MAX_RANK ? dims : std::vector<uint64_t>{});
        kx_error e{};
        kx_tensor da = a.desc(), db = b.desc(), dout = out.desc();
        check(detail::Fns<T>::tensordot(h_.get(), &da, &db, a_axes.data(), (uint32_t)a_axes.size(), b_axes.data(),
                                        (uint32_t)b_axes.size(), &dout, &e),
              e);
        return out;
    }
    // Tape::matmul's VJP (autograd.rs:622-690): (grad b^T, a^T grad) with
    // broadcast batches summed back.
    template <typename T>
    std::pair<DeviceTensor<T>, DeviceTensor<T>> matmul_backward(const DeviceTensor<T> &a, const DeviceTensor<T> &b,
                                                                const DeviceTensor<T> &grad) const {
        auto ga = empty<T>(a.dims()), gb = empty<T>(b.dims());
        kx_error e{};
        kx_tensor da = a.desc(), db = b.desc(), dg = grad.desc(), dga = ga.desc(), dgb = gb.desc();
        check(detail::Fns<T>::matmul_backward(h_.get(), &da, &db, &dg, &dga, &dgb, &e), e);
        return {ga, gb};
    }
    // conv2d_backward (neural.rs:379-430): input and weight gradients.
    template <typename T>
    std::pair<DeviceTensor<T>, DeviceTensor<T>> conv2d_backward(const DeviceTensor<T> &x, const DeviceTensor<T> &w,
                                                                const DeviceTensor<T> &grad,
                                                                const kx_conv2d_options &opts) const {
        auto gx = empty<T>(x.dims()), gw = empty<T>(w.dims());
        kx_error e{};
        kx_tensor dx = x.desc(), dw = w.desc(), dg = grad.desc(), dgx = gx.desc(), dgw = gw.desc();
        check(detail::Fns<T>::conv2d_backward(h_.get(), &dx, &dw, &dg, &opts, &dgx, &dgw, &e), e);
        return {gx, gw};
    }

  private:
    Handle h_;
    int device_;
};

// The row-sharded f32 product from one process over several executors, one
// per GPU (kx_gemm_sharded_f32): executor r multiplies a_windows[r] (window r
// of A's rows, shard_window(M, r, n)) by b[r] into the same rows of out[r];
// with `gather` every output holds the whole product once each executor has
// synchronized.  Reference counterpart: CpuExecutor::matmul_into's row chunks
// per worker (execution.rs:188-233).
inline void gemm_sharded(const std::vector<const CudaExecutor *> &execs,
                         const std::vector<DeviceTensor<float>> &a_windows, const std::vector<DeviceTensor<float>> &b,
                         const std::vector<DeviceTensor<float>> &out, bool gather = true) {
    const size_t n = execs.size();
    if (a_windows.size() != n || b.size() != n || out.size() != n) throw OpsError(KX_E_PARAM);
    std::vector<kx_handle *> hs(n);
    std::vector<kx_tensor> da(n), db(n), dout(n);
    for (size_t r = 0; r < n; ++r) {
        if (!execs[r]) throw OpsError(KX_E_PARAM);
        hs[r] = execs[r]->handle();
        da[r] = a_windows[r].desc();
        db[r] = b[r].desc();
        dout[r] = out[r].desc();
    }
    kx_error e{};
    check(kx_gemm_sharded_f32(hs.data(), (uint32_t)n, da.data(), db.data(), dout.data(), gather ? 1 : 0, &e), e);
}

}  // namespace kernix
