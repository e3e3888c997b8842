"""conv2d on the tensor cores (split-TF32 implicit GEMM, im2col gathered into
the B operand) against the compensated oracle.

The handle is set to KX_F32_3XTF32 so every case takes the tensor-core kernel
when its weights are dense tap rows; the bound is the reference's f32 scaled
form |x - y| <= 2e-6 sum|w x| (small_matmul_tests.rs:153-186), applied to the
tiled-conv comparison of native_kernel_tests.rs:201-241.
"""
import math

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture
def tc(kx, torch_cuda):
    h = kx.handle(0)
    h.set_f32_variant(2)
    yield h
    h.set_f32_variant(0)


def to_dev(arr, torch):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def _check(kx, torch, x, w, opts, x_dev=None):
    got = kx.conv2d(x_dev if x_dev is not None else to_dev(x, torch), to_dev(w, torch),
                    kx.Conv2dOptions(**opts)).cpu().numpy().astype(np.float64)
    d2, ab = oracle.conv2d_dot2(oracle.View.of(x), oracle.View.of(w), **opts)
    assert got.shape == d2.shape
    assert (np.abs(got - d2) <= 2e-6 * ab + 1e-30).all(), float(np.max(np.abs(got - d2) / np.maximum(ab, 1e-30)))


GEOMETRIES = [
    # (n, c, h, w), (co, kh, kw), options
    ((2, 128, 20, 20), (256, 3, 3), dict(stride=(1, 1), padding=(1, 1), dilation=(1, 1), groups=1)),
    ((3, 19, 17, 23), (40, 3, 3), dict(stride=(2, 1), padding=(1, 2), dilation=(2, 1), groups=1)),
    ((2, 32, 15, 15), (48, 3, 3), dict(stride=(1, 1), padding=(1, 1), dilation=(1, 1), groups=2)),
    ((2, 64, 9, 11), (130, 1, 1), dict(stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1)),
    ((1, 8, 30, 30), (16, 5, 5), dict(stride=(3, 3), padding=(2, 2), dilation=(1, 1), groups=1)),
    ((2, 3, 40, 40), (64, 7, 7), dict(stride=(2, 2), padding=(3, 3), dilation=(1, 1), groups=1)),
    ((3, 40, 13, 11), (512, 3, 3), dict(stride=(1, 1), padding=(1, 1), dilation=(1, 1), groups=1)),
    ((2, 32, 9, 9), (512, 3, 3), dict(stride=(1, 1), padding=(0, 1), dilation=(1, 1), groups=2)),
]


# Input rows whose width is a multiple of 4 floats (16-byte rows) are boxed
# by TMA: with 256-channel groups they take the patch-staged pair kernel.
PATCH_GEOMETRIES = [
    ((2, 20, 12, 12), (256, 3, 3), dict(stride=(1, 1), padding=(1, 1), dilation=(1, 1), groups=1)),
    ((1, 24, 17, 20), (512, 3, 3), dict(stride=(2, 1), padding=(1, 2), dilation=(2, 1), groups=2)),
    ((1, 8, 30, 28), (256, 5, 5), dict(stride=(1, 1), padding=(2, 2), dilation=(1, 1), groups=1)),
    ((1, 16, 9, 8), (256, 1, 1), dict(stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1)),
    ((1, 3, 40, 40), (256, 7, 7), dict(stride=(2, 2), padding=(3, 3), dilation=(1, 1), groups=1)),
    ((1, 32, 56, 56), (256, 3, 3), dict(stride=(1, 1), padding=(1, 1), dilation=(1, 1), groups=1)),
    ((3, 64, 24, 36), (512, 3, 3), dict(stride=(1, 1), padding=(1, 1), dilation=(1, 1), groups=1)),
]


def expected_kernel(xs, ws, opts):
    if (ws[0] // opts["groups"]) % 256:
        return "conv_tc_3xtf32_128x128"
    return "conv_tc_3xtf32_patch_256x" if xs[3] % 4 == 0 else "conv_tc_3xtf32_pair_256x256"


@pytest.mark.parametrize("xs,ws,opts", GEOMETRIES + PATCH_GEOMETRIES)
def test_conv_tc_geometries(kx, torch_cuda, tc, xs, ws, opts):
    rng = np.random.default_rng(sum(xs) + sum(ws))
    n, c, h, w = xs
    co, kh, kw = ws
    x = rng.uniform(-1, 1, xs).astype(np.float32)
    wt = rng.normal(0, math.sqrt(2 / (c // opts["groups"] * kh * kw)), (co, c // opts["groups"], kh, kw)).astype(np.float32)
    _check(kx, torch_cuda, x, wt, opts)
    assert tc.last_kernel.startswith(expected_kernel(xs, ws, opts)), tc.last_kernel


def test_conv_patch_channel_and_image_strides(kx, torch_cuda, tc):
    """The patch boxes follow the caller's channel and image strides: the
    input is every other channel of a wider buffer, images two apart."""
    torch = torch_cuda
    rng = np.random.default_rng(17)
    buf = rng.uniform(-1, 1, (4, 40, 14, 16)).astype(np.float32)
    x = buf[::2, ::2]                                   # 2 images x 20 channels, strided
    wt = rng.normal(0, 0.1, (256, 20, 3, 3)).astype(np.float32)
    dev = to_dev(buf, torch).reshape(-1)
    xv = kx.TensorView(dev, (2, 20, 14, 16), (2 * 40 * 14 * 16, 2 * 14 * 16, 16, 1), 0)
    _check(kx, torch, np.ascontiguousarray(x), wt, dict(stride=(1, 1), padding=(1, 1), dilation=(1, 1), groups=1),
           x_dev=xv)
    assert tc.last_kernel.startswith("conv_tc_3xtf32_patch_256x"), tc.last_kernel


def test_conv_tc_reversed_and_strided_input(kx, torch_cuda, tc):
    """Input read through negative and gapped strides (reverse_axis(3) of a
    padded buffer), as the strided conv tests do."""
    torch = torch_cuda
    rng = np.random.default_rng(9)
    buf = rng.uniform(-1, 1, (2, 24, 13, 16)).astype(np.float32)
    x = buf[:, :, :, ::-1][:, :, :, 1:15]          # width 14, reversed, one column skipped
    wt = rng.normal(0, 0.1, (32, 24, 3, 3)).astype(np.float32)
    dev = to_dev(buf, torch).reshape(-1)
    n, c, h, w = 2, 24, 13, 16
    xv = kx.TensorView(dev, (n, c, h, 14), (c * h * w, h * w, w, -1), w - 2)
    _check(kx, torch, np.ascontiguousarray(x), wt, dict(stride=(1, 1), padding=(1, 1), dilation=(1, 1), groups=1),
           x_dev=xv)
    assert tc.last_kernel == "conv_tc_3xtf32_128x128"


@pytest.mark.parametrize("co,width", [(40, 12), (256, 13), (256, 12)])
def test_conv_tc_nonfinite_input_tiles(kx, torch_cuda, tc, co, width):
    """inf/NaN in the input: the affected tiles are recomputed with FMA, so
    the result keeps IEEE propagation (no NaN from inf * 0 in a cross term);
    256 output channels take the CTA-pair kernel (gathered at width 13,
    patch-staged at width 12)."""
    torch = torch_cuda
    rng = np.random.default_rng(4)
    x = rng.uniform(-1, 1, (2, 32, 12, width)).astype(np.float32)
    x[0, 3, 5, 5] = np.inf
    x[1, 7, 0, 0] = np.nan
    wt = np.abs(rng.normal(0, 0.1, (co, 32, 3, 3))).astype(np.float32)
    opts = kx.Conv2dOptions(padding=(1, 1))
    got = kx.conv2d(to_dev(x, torch), to_dev(wt, torch), opts).cpu().numpy()
    assert tc.last_kernel.startswith(expected_kernel(x.shape, wt.shape, dict(groups=1))), tc.last_kernel
    tc.set_f32_variant(1)
    ref = kx.conv2d(to_dev(x, torch), to_dev(wt, torch), opts).cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    fin = np.isfinite(ref)
    assert np.isinf(got).any() and np.isnan(got).any()
    assert (np.abs(got[fin] - ref[fin]) <= 1e-5 * (1 + np.abs(ref[fin]))).all()


def test_conv_tc_nonfinite_weight_in_padding(kx, torch_cuda, tc):
    """A NaN weight tap that only lands on padding leaves the output finite
    (the ordered fixup replaces the tensor-core result, as for the SIMT path)."""
    x = np.arange(2 * 16 * 8 * 8, dtype=np.float32).reshape(2, 16, 8, 8) / 97.0
    w = np.ones((24, 16, 3, 3), dtype=np.float32) / 16
    w[:, :, 0, 0] = np.nan
    opts = dict(stride=(7, 7), padding=(1, 1), dilation=(1, 1), groups=1)
    ref = oracle.conv2d_reference(oracle.View.of(x), oracle.View.of(w), **opts)
    got = kx.conv2d(to_dev(x, torch_cuda), to_dev(w, torch_cuda), kx.Conv2dOptions(**opts)).cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(got[~np.isnan(got)], ref[~np.isnan(ref)])


def test_conv_tc_declines_to_simt(kx, torch_cuda, tc):
    """More taps than the shared-memory tap table holds (cin 1024 x 3 x 3) or
    fewer than one k-tile: the SIMT implicit GEMM takes over, same bound."""
    torch = torch_cuda
    rng = np.random.default_rng(12)
    x = rng.uniform(-1, 1, (1, 1024, 6, 6)).astype(np.float32)
    w = rng.normal(0, 0.02, (8, 1024, 3, 3)).astype(np.float32)
    _check(kx, torch, x, w, dict(stride=(1, 1), padding=(1, 1), dilation=(1, 1), groups=1))
    assert tc.last_kernel.startswith("conv_igemm"), tc.last_kernel
    x = rng.uniform(-1, 1, (1, 3, 6, 6)).astype(np.float32)
    w = rng.normal(0, 0.3, (8, 3, 2, 2)).astype(np.float32)
    _check(kx, torch, x, w, dict(stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1))
    assert tc.last_kernel.startswith("conv_igemm"), tc.last_kernel


def test_conv_auto_uses_tensor_cores_for_large_convs(kx, torch_cuda):
    torch = torch_cuda
    h = kx.handle(0)
    h.set_f32_variant(0)
    rng = np.random.default_rng(21)
    x = rng.uniform(-1, 1, (16, 64, 28, 28)).astype(np.float32)   # 98 tiles of 128 x 128
    w = rng.normal(0, 0.06, (128, 64, 3, 3)).astype(np.float32)
    y = kx.conv2d(to_dev(x, torch), to_dev(w, torch), kx.Conv2dOptions(padding=(1, 1)))
    assert h.last_kernel == "conv_tc_3xtf32_128x128", h.last_kernel
    d2, ab = oracle.conv2d_dot2(oracle.View.of(x[:1]), oracle.View.of(w), padding=(1, 1))
    assert (np.abs(y[:1].cpu().numpy().astype(np.float64) - d2) <= 2e-6 * ab + 1e-30).all()


def test_conv_patch_nonfinite_weights_fall_back(kx, torch_cuda, tc):
    """An inf weight on the patch-staged path: its split raises the flag and
    every tile is recomputed with FMA, so inf/NaN follow IEEE as on the SIMT
    path, and finite outputs keep the bound."""
    torch = torch_cuda
    rng = np.random.default_rng(8)
    x = rng.uniform(-1, 1, (2, 16, 12, 12)).astype(np.float32)
    wt = rng.normal(0, 0.1, (256, 16, 3, 3)).astype(np.float32)
    wt[7, 3, 1, 1] = np.inf
    opts = kx.Conv2dOptions(padding=(1, 1))
    got = kx.conv2d(to_dev(x, torch), to_dev(wt, torch), opts).cpu().numpy()
    assert tc.last_kernel.startswith("conv_tc_3xtf32_patch_256x"), tc.last_kernel
    tc.set_f32_variant(1)
    ref = kx.conv2d(to_dev(x, torch), to_dev(wt, torch), opts).cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    assert np.isinf(got[:, 7]).any()
    fin = np.isfinite(ref)
    assert (np.abs(got[fin] - ref[fin]) <= 1e-5 * (1 + np.abs(ref[fin]))).all()


def test_conv_patch_repacked_weights(kx, torch_cuda, tc):
    """Weights through a view whose taps are not dense rows (every row padded
    to 4 columns) are repacked beside their lo parts."""
    torch = torch_cuda
    rng = np.random.default_rng(9)
    x = rng.uniform(-1, 1, (1, 24, 16, 16)).astype(np.float32)
    wbuf = rng.normal(0, 0.08, (256, 24, 3, 4)).astype(np.float32)
    wt = np.ascontiguousarray(wbuf[..., :3])
    dev = to_dev(wbuf, torch).reshape(-1)
    wv = kx.TensorView(dev, (256, 24, 3, 3), (24 * 12, 12, 4, 1), 0)
    got = kx.conv2d(to_dev(x, torch), wv, kx.Conv2dOptions(padding=(1, 1))).cpu().numpy().astype(np.float64)
    assert tc.last_kernel.startswith("conv_tc_3xtf32_patch_256x"), tc.last_kernel
    d2, ab = oracle.conv2d_dot2(oracle.View.of(x), oracle.View.of(wt), padding=(1, 1))
    assert (np.abs(got - d2) <= 2e-6 * ab + 1e-30).all()
