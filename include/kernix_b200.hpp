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
};
template <> struct Fns<double> {
    static constexpr auto dense = kx_try_dense_matmul_f64;
    static constexpr auto strided = kx_try_strided_matmul_f64;
    static constexpr auto matmul = kx_matmul_f64;
    static constexpr auto conv2d = kx_conv2d_f64;
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

// One handle per device; movable, not copyable.
class Handle {
  public:
    explicit Handle(int device = 0) {
        kx_error e{};
        check(kx_create(device, &h_, &e), e);
    }
    ~Handle() { kx_destroy(h_); }
    Handle(const Handle &) = delete;
    Handle &operator=(const Handle &) = delete;
    Handle(Handle &&o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    kx_handle *get() const { return h_; }

  private:
    kx_handle *h_ = nullptr;
};

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
    // MatmulDevice::matmul: NumPy matmul semantics into a fresh C-order tensor.
    template <typename T>
    DeviceTensor<T> matmul(const DeviceTensor<T> &a, const DeviceTensor<T> &b) const {
        kx_error e{};
        uint32_t rank = 0;
        uint64_t od[KX_MAX_RANK];
        check(kx_matmul_shape(a.dims().data(), (uint32_t)a.dims().size(), b.dims().data(),
                              (uint32_t)b.dims().size(), &rank, od, &e),
              e);
        std::vector<uint64_t> dims(od, od + rank);
        size_t n = 1;
        for (auto d : dims) n *= d;
        auto buf = std::make_shared<DeviceBuffer<T>>(h_.get(), n ? n : 1);
        std::vector<int64_t> strides(rank);
        int64_t acc = 1;
        for (size_t i = rank; i-- > 0;) {
            strides[i] = acc;
            acc *= (int64_t)(dims[i] ? dims[i] : 1);
        }
        DeviceTensor<T> out(buf, dims, strides, 0);
        kx_tensor da = a.desc(), db = b.desc(), dc = out.desc();
        dc.storage_len = n;
        check(detail::Fns<T>::matmul(h_.get(), &da, &db, &dc, &e), e);
        return out;
    }

  private:
    Handle h_;
    int device_;
};

}  // namespace kernix
