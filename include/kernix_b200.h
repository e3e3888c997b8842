/*
 * kernix_b200.h -- C ABI of the B200 (sm_100a) dense-matmul path for Kernix.
 *
 * This is the drop-in boundary that a thin Rust FFI crate binds.  Every entry
 * point takes plain pointers, sizes and layout descriptors (no C++ or torch
 * types), returns an int status, and performs all validation on the host
 * BEFORE any device work: a call that fails validation writes nothing.
 *
 * Reference interfaces replaced (paths inside the kernix repository):
 *   - MatmulElement::try_dense_matmul   crates/kernix-ops/src/ops/matmul_element.rs:28-44,139-251
 *   - MatmulElement::try_strided_matmul crates/kernix-ops/src/ops/matmul_element.rs:17-23,53-138
 *   - MatrixInput::new                  crates/kernix-ops/src/ops/matmul_element.rs:262-300
 *   - matmul / matmul_impl              crates/kernix-ops/src/ops/linalg.rs:31-44,68-214
 *   - MatmulDevice<T>::matmul           crates/kernix-ops/src/execution.rs:25-36
 *   - Device<T> upload/download/sync    crates/kernix-core/src/device.rs:22-35
 *   - neural::conv2d / ConvGeometry     crates/kernix-ops/src/neural.rs:22-133,177-183
 *   - softmax_temperature               crates/kernix-ops/src/ops/math_extra.rs:394-401,425-500,544-557
 *   - softmax                           crates/kernix-ops/src/ops/math.rs:398-465,531-536
 *   - tensordot                         crates/kernix-ops/src/ops/linalg_extra.rs:164-276
 *   - CpuExecutor::matmul_into          crates/kernix-ops/src/execution.rs:149-240
 *     (its row chunks per worker, execution.rs:188-233: the sharded entries)
 *   - Config / Context::new ([cuda])    crates/kernix/src/config.rs:28-40,84-95,133-137
 *   - Tape::matmul backward (VJP)       crates/kernix/src/autograd.rs:622-690
 *   - conv2d_backward                   crates/kernix-ops/src/neural.rs:379-430
 *   - the C bridge convention           crates/kernix-ops/src/accelerate.c:15-30
 *     (int status, caller-owned buffers, row-major output)
 *
 * Element units: every length, stride and origin is counted in ELEMENTS of the
 * call's scalar type, as in kernix_core::Layout (layout/affine.rs:15-58).
 */
#ifndef KERNIX_B200_H
#define KERNIX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KX_ABI_VERSION 1
#define KX_MAX_RANK 8

/* Status codes.  KX_OK: success, every output element written.
 * KX_DECLINED mirrors a hook returning `false`: nothing was written and the
 * caller may fall back (matmul_element.rs:17-44).  Codes 2..11 map 1:1 onto
 * kernix OpsError / LayoutError variants (ops/error.rs:8-140). */
typedef enum kx_status {
    KX_OK = 0,
    KX_DECLINED = 1,
    KX_E_INVALID_RANK = 2,      /* OpsError::InvalidRank {operation, minimum, actual} */
    KX_E_CONTRACT = 3,          /* OpsError::ContractDimensionMismatch {left, right} */
    KX_E_BROADCAST = 4,         /* OpsError::BroadcastIncompatible {axis, left, right} */
    KX_E_SHAPE_OVERFLOW = 5,    /* ShapeError::ElementCountOverflow {axis, accumulated, dim} */
    KX_E_DIM_OVERFLOW = 6,      /* OpsError::DimensionOverflow {axis} */
    KX_E_LAYOUT = 7,            /* LayoutError: span/storage/stride validation (values[0] = kx_layout_error) */
    KX_E_PARAM = 8,             /* OpsError::InvalidParameter {operation, parameter} */
    KX_E_EXACT_RANK = 9,        /* OpsError::ExactRank {operation, expected, actual} */
    KX_E_NONFINITE = 10,        /* OpsError::NonFiniteInput {operation, indices} */
    KX_E_AXIS = 11,             /* OpsError::AxisOutOfBounds {axis, rank} */
    KX_E_ALIAS = 12,            /* output storage overlaps an input (Rust borrow rules forbid it) */
    KX_E_CUDA = 13,             /* a CUDA runtime call failed (kx_error.cuda_error) */
    KX_E_NO_DEVICE = 14,        /* no usable sm_100 device for this handle */
    KX_E_TIMEOUT = 15,          /* a bounded device-side wait expired */
    KX_E_UNSUPPORTED = 16,      /* valid request outside this library's scope (e.g. rank > 8) */
    KX_E_AXES_MISMATCH = 17,    /* OpsError::ContractAxesMismatch {left, right} (axis counts) */
    KX_E_DUPLICATE_AXIS = 18    /* OpsError::DuplicateAxis {axis} */
} kx_status;

/* Sub-codes in kx_error.values[0] for KX_E_LAYOUT (layout/geometry.rs:40-80, affine.rs:186-199). */
typedef enum kx_layout_error {
    KX_LAYOUT_STRIDE_RANK_MISMATCH = 1,
    KX_LAYOUT_ADDRESS_OVERFLOW = 2,
    KX_LAYOUT_NEGATIVE_STORAGE_OFFSET = 3,
    KX_LAYOUT_STORAGE_TOO_SMALL = 4,    /* values[1] = required, values[2] = available */
    KX_LAYOUT_BYTE_EXTENT_OVERFLOW = 5,
    KX_LAYOUT_OUTPUT_NOT_C_CONTIGUOUS = 6,
    KX_LAYOUT_OUTPUT_SHAPE_MISMATCH = 7,
    KX_LAYOUT_MISALIGNED_POINTER = 8
} kx_layout_error;

/* Structured error record (optional out-parameter, may be NULL).
 * `values` carries the variant's integer fields in declaration order, e.g.
 * InvalidRank -> {minimum, actual}, BroadcastIncompatible -> {axis, left, right},
 * ElementCountOverflow -> {axis, accumulated, dim}. */
typedef struct kx_error {
    int32_t status;
    int32_t cuda_error;
    char operation[40];
    char parameter[96];
    uint64_t values[4];
    uint32_t nindices;
    uint64_t indices[KX_MAX_RANK];
} kx_error;

/* N-d strided tensor descriptor (mirror of kernix_core::Layout + storage).
 * Element (i0..ir-1) lives at data[origin + sum_j i_j * strides[j]].
 * `storage_len` is the number of elements addressable from `data`; the layout's
 * reachable span must lie inside [0, storage_len) (Layout::validate_cpu_storage). */
typedef struct kx_tensor {
    void *data;
    uint64_t storage_len;
    uint64_t origin;
    uint32_t rank;
    uint32_t reserved;
    uint64_t dims[KX_MAX_RANK];
    int64_t strides[KX_MAX_RANK];
} kx_tensor;

/* Rank-2 strided matrix (mirror of MatrixInput {data, dims, strides, origin},
 * matmul_element.rs:262-300).  Singleton strides are ignored, as MatrixInput::new
 * normalises them to zero. */
typedef struct kx_matrix {
    const void *data;
    uint64_t storage_len;
    uint64_t dims[2];
    int64_t strides[2];
    uint64_t origin;
} kx_matrix;

/* Conv2dOptions (neural.rs:22-42): stride/padding/dilation per (y, x). */
typedef struct kx_conv2d_options {
    uint64_t stride[2];
    uint64_t padding[2];
    uint64_t dilation[2];
    uint64_t groups;
} kx_conv2d_options;

/* Kernel family selection for f32. */
typedef enum kx_f32_variant {
    KX_F32_AUTO = 0,    /* library chooses per shape and layout */
    KX_F32_FFMA = 1,    /* SIMT FP32 FMA, fp32 accumulation */
    KX_F32_3XTF32 = 2,  /* split-TF32 tensor-core contraction (tcgen05 + TMEM) */
    KX_F32_3XTF32_1SM = 3   /* the same, one-SM tiles only (no CTA-pair kernel) */
} kx_f32_variant;

/* Kernel family selection for f64. */
typedef enum kx_f64_variant {
    KX_F64_AUTO = 0,    /* library chooses per shape and layout */
    KX_F64_DFMA = 1,    /* SIMT DFMA outer products */
    KX_F64_DMMA = 2     /* FP64 tensor pipe (mma.sync m16n8k4 .f64), f64 accumulation */
} kx_f64_variant;

typedef struct kx_handle kx_handle;

/* ---- library / handle -------------------------------------------------- */
int kx_abi_version(void);
/* Number of CUDA devices visible (0 without a GPU).  Host only. */
int kx_device_count(int *count);
/* Create a handle bound to `device`.  Selects the device, checks sm_100, and
 * creates no stream (the default stream is used until kx_set_stream). */
int kx_create(int device, kx_handle **out, kx_error *err);
int kx_destroy(kx_handle *h);
/* Subsequent work on this handle is ordered on `stream` (a cudaStream_t). */
int kx_set_stream(kx_handle *h, void *stream);
int kx_set_f32_variant(kx_handle *h, int variant);
int kx_set_f64_variant(kx_handle *h, int variant);
/* Ordered mode (CpuExecutor::with_ordered_matmul, execution.rs:76-84): every
 * output is accumulated in increasing k with separately rounded multiply and
 * add, so device matmul results equal matmul_reference (linalg.rs:57-64,
 * 236-316) bit for bit.  Slower: no FMA, no split-K. */
int kx_set_ordered_matmul(kx_handle *h, int ordered);
int kx_ordered_matmul(const kx_handle *h);
/* Wait for outstanding work on the handle's stream (Device::synchronize).
 * Returns KX_E_TIMEOUT (once, then clears it) when a kernel's bounded
 * device-side wait expired since the last call: such a kernel stops, frees its
 * tensor memory and leaves its output unspecified instead of hanging. */
int kx_synchronize(kx_handle *h, kx_error *err);
/* Diagnostic, no counterpart in the reference: the next launch of the one-SM
 * split-TF32 GEMM on this handle (variant KX_F32_3XTF32_1SM, K > 1024, or the
 * automatic choice where it picks that kernel) issues no operand copies and
 * bounds each of its waits by `wait_ns` (1 ms .. 2 s), so every wait expires
 * and the call's kx_synchronize reports KX_E_TIMEOUT.  For exercising a
 * caller's handling of that status; the output of that call is unspecified. */
int kx_diag_expire_next_gemm(kx_handle *h, uint64_t wait_ns);

/* ---- execution context from configuration --------------------------------
 * The [cuda] table a Kernix configuration gains beside [cpu]
 * (config.rs:28-40 CpuConfig {threads, ordered_matmul}; kernix.toml:1-7):
 * everything a CUDA execution context fixes when it is created.  The Rust
 * side parses it with the rest of Config (serde, unknown keys rejected) and
 * passes it here from Context::new (config.rs:133-137). */
typedef struct kx_cuda_config {
    int32_t device;          /* CUDA ordinal */
    int32_t f32_variant;     /* kx_f32_variant */
    int32_t f64_variant;     /* kx_f64_variant */
    int32_t ordered_matmul;  /* 0 or 1: as [cpu] ordered_matmul, for this context's products */
    uint64_t workspace_bytes;    /* device scratch reserved at creation; 0 = grown on first use */
} kx_cuda_config;
/* Defaults: device 0, automatic variants, native (unordered) products, no
 * reserved scratch -- what an absent [cuda] table means. */
void kx_cuda_config_default(kx_cuda_config *cfg);
/* Validate `cfg` field by field (KX_E_PARAM naming the key, before any device
 * work), then create a handle on cfg->device with those settings
 * (KX_E_NO_DEVICE as kx_create) and reserve the scratch (KX_E_CUDA if the
 * device cannot hold it; no handle is returned then). */
int kx_context_create(const kx_cuda_config *cfg, kx_handle **out, kx_error *err);
/* The settings a handle runs with now (Context::config). */
int kx_handle_config(const kx_handle *h, kx_cuda_config *out);

/* ---- Device<T> buffers (device.rs:22-35) -------------------------------- */
int kx_alloc(kx_handle *h, uint64_t bytes, void **out, kx_error *err);
int kx_free(kx_handle *h, void *ptr);
/* Synchronous transfers in physical order; complete before returning. */
int kx_upload(kx_handle *h, void *dst_device, const void *src_host, uint64_t bytes, kx_error *err);
int kx_download(kx_handle *h, void *dst_host, const void *src_device, uint64_t bytes, kx_error *err);

/* ---- shape planning (host only; no device needed) ----------------------- */
/* NumPy matmul output shape with the reference's error order
 * (linalg.rs:77-116): rank-0 left, rank-0 right, contraction mismatch,
 * batch broadcast, element-count overflow.  On success writes the output rank
 * and dims (dims must hold KX_MAX_RANK entries). */
int kx_matmul_shape(const uint64_t *a_dims, uint32_t a_rank,
                    const uint64_t *b_dims, uint32_t b_rank,
                    uint32_t *out_rank, uint64_t *out_dims, kx_error *err);
/* ConvGeometry::new (neural.rs:91-125): output [n, co, oh, ow]. */
int kx_conv2d_shape(const uint64_t *input_dims, uint32_t input_rank,
                    const uint64_t *weight_dims, uint32_t weight_rank,
                    const kx_conv2d_options *options, uint64_t *out_dims, kx_error *err);
/* Validate a descriptor exactly as Layout::from_strides + validate_cpu_storage
 * (affine.rs:43-58,186-199) for elements of `elem_bytes` bytes. */
int kx_validate_tensor(const kx_tensor *t, uint32_t elem_bytes, kx_error *err);

/* ---- device-resident operations (MatmulDevice / free functions) --------- */
/* out = matmul(a, b) on device memory.  `out` must be C-contiguous with the
 * dims returned by kx_matmul_shape and must not overlap a or b.  Arbitrary
 * signed/zero strides and origins are read in place (no host copies). */
int kx_matmul_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out, kx_error *err);
int kx_matmul_f64(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out, kx_error *err);

/* conv2d on device memory: NCHW input (any strides), weight
 * [out_channels, in_channels/groups, kh, kw] (any strides), C-contiguous out.
 * im2col is fused into the operand load (no column buffer). */
int kx_conv2d_f32(kx_handle *h, const kx_tensor *input, const kx_tensor *weight,
                  const kx_conv2d_options *options, const kx_tensor *out, kx_error *err);
int kx_conv2d_f64(kx_handle *h, const kx_tensor *input, const kx_tensor *weight,
                  const kx_conv2d_options *options, const kx_tensor *out, kx_error *err);

/* softmax_temperature(src, axis, temperature) into a C-contiguous `out` of the
 * same dims.  Nonfinite input returns KX_E_NONFINITE with the C-order indices
 * of the first nonfinite element in the reference's scan order; `out` is then
 * unspecified (the reference returns no tensor). */
int kx_softmax_temperature_f32(kx_handle *h, const kx_tensor *src, int64_t axis, float temperature,
                               const kx_tensor *out, kx_error *err);
int kx_softmax_temperature_f64(kx_handle *h, const kx_tensor *src, int64_t axis, double temperature,
                               const kx_tensor *out, kx_error *err);
/* softmax(src, axis) (ops/math.rs:398-465,531-536): exp(x - max) / sum along
 * `axis` into a C-contiguous `out` of the same dims.  Axis errors come first;
 * nonfinite input returns KX_E_NONFINITE (operation "softmax") with the
 * C-order indices of the first nonfinite element in the reference scan order. */
int kx_softmax_f32(kx_handle *h, const kx_tensor *src, int64_t axis, const kx_tensor *out, kx_error *err);
int kx_softmax_f64(kx_handle *h, const kx_tensor *src, int64_t axis, const kx_tensor *out, kx_error *err);

/* Attention products in one call: out = matmul(softmax_temperature(matmul(q,
 * kt), -1, temperature), v) -- the composition Kernix users write from
 * matmul (linalg.rs:68-214) and softmax_temperature (math_extra.rs:394-401,
 * 425-500,544-557), with the same errors in the same order: matmul(q, kt)'s
 * shape errors, the temperature, matmul(P, v)'s shape errors, then
 * NonFiniteInput (operation "softmax_temperature") with the indices into the
 * scores of their first inf/NaN in the reference scan order.  `out` is
 * C-contiguous with matmul(P, v)'s dims.  When q is [B.., sq, 128], kt the
 * transposed view [B.., 128, sk] of a row-major k, v [B.., sk, 128] with equal
 * batch dims (each nesting into one stride) and unit strides along the head
 * dimension, one fused tcgen05 kernel computes it without materialising the
 * scores; other layouts, ordered mode, and inputs whose scores hold an inf or
 * NaN (or whose v does) run the three calls on a scores buffer the handle
 * allocates.  Synchronises the handle's stream (the nonfinite flag is read). */
int kx_attention_f32(kx_handle *h, const kx_tensor *q, const kx_tensor *kt, const kx_tensor *v, float temperature,
                     const kx_tensor *out, kx_error *err);

/* tensordot (ops/linalg_extra.rs:164-276): out (C-contiguous; left's free
 * axes then right's, in order) = the contraction of a and b over the axis
 * pairs (a_axes[i], b_axes[i]) (negative axes count from the end).  Errors in
 * the reference order: KX_E_AXES_MISMATCH (na != nb), then per pair
 * KX_E_AXIS (left, then right), KX_E_DUPLICATE_AXIS, KX_E_CONTRACT.  One GEMM
 * over [free(a), contracted] x [contracted, free(b)], on strided views when
 * the axes nest (else after a gather into the handle's buffer); in ordered
 * mode the sums equal the reference's bit for bit. */
int kx_tensordot_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const int64_t *a_axes, uint32_t na,
                     const int64_t *b_axes, uint32_t nb, const kx_tensor *out, kx_error *err);
int kx_tensordot_f64(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const int64_t *a_axes, uint32_t na,
                     const int64_t *b_axes, uint32_t nb, const kx_tensor *out, kx_error *err);

/* ---- backward products -------------------------------------------------- */
/* Tape::matmul's vector-Jacobian products (crates/kernix/src/autograd.rs:
 * 622-690): grad_a = grad . b^T and grad_b = a^T . grad on the operands with
 * vectors as [1, k] / [k, 1], each summed back over the batch axes its operand
 * was broadcast along.  `grad` has matmul(a, b)'s dims (else KX_E_PARAM,
 * "gradient shape differs from forward output"); grad_a / grad_b (either may
 * be NULL) are C-contiguous with a's / b's dims.  Transposed operands are read
 * as strided views; a broadcast batch is reduced on the device. */
int kx_matmul_backward_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *grad,
                           const kx_tensor *grad_a, const kx_tensor *grad_b, kx_error *err);
int kx_matmul_backward_f64(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *grad,
                           const kx_tensor *grad_a, const kx_tensor *grad_b, kx_error *err);
/* conv2d_backward (crates/kernix-ops/src/neural.rs:379-430): grad_input and
 * grad_weight (either may be NULL; C-contiguous, the input's / weight's dims)
 * of conv2d(input, weight, options) for the output gradient `grad` (the
 * forward output's dims, else KX_E_PARAM).  Every element adds the same
 * contributions in the reference loop's order, product and sum rounded
 * separately: the results equal the reference's bit for bit. */
int kx_conv2d_backward_f32(kx_handle *h, const kx_tensor *input, const kx_tensor *weight, const kx_tensor *grad,
                           const kx_conv2d_options *options, const kx_tensor *grad_input,
                           const kx_tensor *grad_weight, kx_error *err);
int kx_conv2d_backward_f64(kx_handle *h, const kx_tensor *input, const kx_tensor *weight, const kx_tensor *grad,
                           const kx_conv2d_options *options, const kx_tensor *grad_input,
                           const kx_tensor *grad_weight, kx_error *err);

/* ---- host-buffer hooks (MatmulElement) ---------------------------------- */
/* try_dense_matmul: C-order a[m*k], b[k*n] -> out[m*n] in HOST memory.
 * Returns KX_DECLINED (nothing written) on any length mismatch, exactly like
 * the reference hook's `false`; KX_OK when all m*n outputs were written. */
int kx_try_dense_matmul_f32(kx_handle *h, const float *a, uint64_t a_len, const float *b, uint64_t b_len,
                            float *out, uint64_t out_len, uint64_t m, uint64_t k, uint64_t n);
int kx_try_dense_matmul_f64(kx_handle *h, const double *a, uint64_t a_len, const double *b, uint64_t b_len,
                            double *out, uint64_t out_len, uint64_t m, uint64_t k, uint64_t n);
/* try_strided_matmul: validated signed-stride host matrices, C-order out[m*n]. */
int kx_try_strided_matmul_f32(kx_handle *h, const kx_matrix *a, const kx_matrix *b, float *out, uint64_t out_len);
int kx_try_strided_matmul_f64(kx_handle *h, const kx_matrix *a, const kx_matrix *b, double *out, uint64_t out_len);
/* MatrixInput::new validation alone (host only). */
int kx_matrix_validate(const kx_matrix *m, uint32_t elem_bytes, kx_error *err);

/* ---- allocation-free variant -------------------------------------------- */
/* No counterpart in the reference.  Split-K f32 GEMM out = a x b for callers
 * that may not call cudaMalloc while they run (a process whose device memory is
 * owned up front by its own pool, or a latency-critical loop where cudaMalloc /
 * cudaFree would synchronise the device).  It takes no handle and allocates
 * nothing: the split-K partial sums live in a file-scope 16 MiB static device
 * array that every GPU loading this library keeps until exit.
 *   - rank-two a [m,k] and b [k,n], any signed strides, device memory of the
 *     calling thread's current device; out C-contiguous [m,n], not overlapping;
 *   - rejects m*n > 2,097,152 (two splits must fit) with KX_E_UNSUPPORTED;
 *   - the first call on a device resolves the array's address on that device
 *     (and loads the module there): make it before any stream capture;
 *   - all calls share the array: calls whose kernels overlap on the GPU race,
 *     so order them on one stream.  Nothing in it needs to start at zero. */
int kx_matmul_splitk_f32_static(const kx_tensor *a, const kx_tensor *b, const kx_tensor *out, void *stream,
                                kx_error *err);

/* ---- gathered output across the GPUs of one node ------------------------ */
/* No counterpart in the reference: CpuExecutor::matmul_into
 * (execution.rs:188-233) splits output rows over threads that share one
 * buffer.  Across GPUs each process owns its device, so a row-sharded GEMM
 * gathers its output by pushing each rank's rows into every peer's copy of C:
 * the buffer is exported once (kx_ipc_export), mapped by the other processes
 * (kx_ipc_import), and rows are pushed with kx_copy_async, which runs on the
 * copy engines over NVLink and takes no SMs from the GEMMs that overlap it.
 * `device_ptr` for export must be a pointer returned by kx_alloc (the start of
 * a cudaMalloc allocation).  Imported pointers are valid in this process only
 * and are released with kx_ipc_close. */
#define KX_IPC_HANDLE_BYTES 64
int kx_ipc_export(kx_handle *h, void *device_ptr, unsigned char *handle_out, kx_error *err);
int kx_ipc_import(kx_handle *h, const unsigned char *handle, void **device_ptr, kx_error *err);
int kx_ipc_close(kx_handle *h, void *device_ptr);
/* out = matmul(a, b) as kx_matmul_*, with every element stored through
 * `out_mc`: the NVLink multicast (NVLS) address of out->data's memory, from a
 * multicast object that binds the same buffer on each GPU of the node.  One
 * store reaches all of them, so when each rank computes its own rows of C this
 * call leaves the full product on every rank once all ranks' calls have
 * completed (the caller orders that, e.g. with a collective after the call).
 * The split-TF32 kernel stores its epilogue through the address directly;
 * other kernels store locally and a multicast copy of the rows follows. */
int kx_matmul_replicated_f32(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out,
                             void *out_mc, kx_error *err);
int kx_matmul_replicated_f64(kx_handle *h, const kx_tensor *a, const kx_tensor *b, const kx_tensor *out,
                             void *out_mc, kx_error *err);
/* Store `bytes` (a multiple of 4, 4-byte aligned) from this GPU's `src`
 * through the multicast address `mc_dst` on the handle's stream. */
int kx_multicast_store(kx_handle *h, const void *src, void *mc_dst, uint64_t bytes, kx_error *err);
/* Copy `bytes` (multiple of 16, 16-byte aligned) from `src` to each of the
 * `ndst` (<= 8) destinations with a kernel on the handle's stream: all SMs
 * drive the NVLink stores.  For a step's last piece, when there is no GEMM
 * left to overlap and the copy engines' fan-out would be the slower path. */
int kx_peer_broadcast(kx_handle *h, const void *src, void *const *dsts, int ndst, uint64_t bytes, kx_error *err);
/* Enqueue a device-to-device copy of `bytes` on `stream` (a cudaStream_t of the
 * handle's device; null = the handle's stream).  Either side may be an
 * imported peer pointer.  Returns once the copy is enqueued. */
int kx_copy_async(kx_handle *h, void *dst, const void *src, uint64_t bytes, void *stream, kx_error *err);

/* ---- work split across the GPUs of one node ------------------------------ */
/* Kernix splits a product over worker threads (CpuExecutor::matmul_into,
 * execution.rs:188-233: chunks of output rows per worker).  Across GPUs each
 * process owns one device; these plans are what every rank computes alike.
 * kx_shard_window: the contiguous window [start, start + count) of `total`
 * independent units (attention heads, images) that `rank` of `world` takes;
 * the first total % world ranks take one more.  Host only. */
int kx_shard_window(uint64_t total, uint32_t rank, uint32_t world, uint64_t *start, uint64_t *count);
/* kx_row_piece: the row plan of a row-sharded product: the largest piece of
 * at most `target_piece` rows that tiles M evenly over the ranks, and the
 * number of pieces per rank.  Piece i of rank r is global rows
 * [(i * world + r) * piece, + piece).  Host only. */
int kx_row_piece(uint64_t m, uint32_t world, uint64_t target_piece, uint64_t *piece, uint64_t *pieces);
/* One rank's share of the row-sharded f32 product out = A B over the GPUs of
 * one node (one process and handle per GPU).  `a_local` holds this rank's rows
 * of A, piece after piece ([pieces * piece, K], any strides: e.g. a strided
 * slice of a wider buffer); `b` [K, N] is this rank's replica; `out` [M, N] is
 * C-contiguous.  Each piece is multiplied into its global rows of `out`; with
 * `peer_out` (world pointers: the start of every rank's `out` storage as
 * mapped in this process by kx_ipc_import, this rank's entry unused) it is
 * then written into the same rows of every peer's output -- by the copy
 * engines while the next piece multiplies, and the last piece either through
 * `out_mc`, the NVLink multicast address of `out`'s storage (one store, the
 * NVSwitch delivers it to every rank), or, when that is null, by a kernel on
 * all SMs.  Up to 4 GPUs, when the last piece's fan-out ((world - 1) x piece
 * rows) is at least 32 MB and the piece a multiple of 256 rows, the last
 * piece runs as two row halves, each one GEMM batched over its two K halves
 * into the handle's scratch plus a summing kernel, and the first half is
 * pushed while the second multiplies.  Every rank's `out` has the same
 * layout.  Returns once the work is enqueued on the handle's stream; when
 * every rank's call has completed on its
 * device (the caller orders that: a collective after the call, or
 * kx_synchronize on every rank and a host barrier), every rank's `out` holds
 * the whole product.  peer_out NULL: only this rank's rows are written. */
int kx_matmul_rows_sharded_f32(kx_handle *h, const kx_tensor *a_local, const kx_tensor *b, const kx_tensor *out,
                               uint32_t rank, uint32_t world, uint64_t piece, void *const *peer_out, void *out_mc,
                               kx_error *err);
/* The row-sharded f32 product driven from ONE process over `ngpu` (1..8)
 * handles, one per GPU (handles may share a device), for callers without one
 * process per GPU.  `a`, `b` and `out` are arrays of ngpu descriptors:
 * handle r multiplies a[r] (the rows of window r of A, as kx_shard_window(M,
 * r, ngpu) gives them, on its device) by b[r] ([K, N], its replica) into the
 * same rows of out[r] (a C-contiguous [M, N] output on its device).  With
 * gather_out != 0 every window is then copied into every other handle's output
 * by the copy engines (peer access between the devices is enabled on first
 * use), after whatever that handle's stream had queued before the call; the
 * outputs must not overlap.  With gather_out == 0 out[r] receives only its own
 * rows.  Every argument is checked before anything is enqueued.  Returns once
 * the work is enqueued: each handle's stream completes after all windows have
 * reached its output (kx_synchronize on each handle).  Reference counterpart:
 * the row chunks of CpuExecutor::matmul_into (execution.rs:188-233), one per
 * worker sharing one output. */
int kx_gemm_sharded_f32(kx_handle *const *handles, uint32_t ngpu, const kx_tensor *a, const kx_tensor *b,
                        const kx_tensor *out, int gather_out, kx_error *err);

/* ---- introspection ------------------------------------------------------ */
/* Number of kernel launches this handle has issued since creation. */
uint64_t kx_launch_count(const kx_handle *h);
/* Name of the kernel family the last GEMM on this handle used. */
const char *kx_last_kernel(const kx_handle *h);
const char *kx_status_name(int status);

#ifdef __cplusplus
}
#endif
#endif /* KERNIX_B200_H */
