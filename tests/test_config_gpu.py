"""Execution contexts made from configuration drive the device products.

A context's [cuda] settings (kernel family, ordered mode, reserved scratch)
apply to the products its CudaExecutor runs and to calls made under
``kx.using(handle)``, and leave the process's default handle alone; an
ordered context gives matmul_reference's bits (linalg.rs:57-64, 236-316)
through the executor, as [cpu] ordered_matmul does on the CPU
(config.rs:133-137, execution.rs:76-84).
"""
import numpy as np
import pytest

import kernix_b200 as kx
import oracle
from kernix_b200.config import Config, ConfigExecutionError, Context, CudaConfig, settings

pytestmark = pytest.mark.gpu


def test_context_settings_reach_the_handle(torch_cuda):
    ctx = Context.new(Config.from_toml("[cuda]\nf32_variant='ffma'\nf64_variant='dfma'\nworkspace_mib=64"))
    h = ctx.cuda().h
    s = settings(h)
    assert (s["device"], s["f32_variant"], s["f64_variant"], s["ordered_matmul"]) == (0, "ffma", "dfma", False)
    assert s["workspace_bytes"] >= 64 << 20
    torch = torch_cuda
    a = torch.rand(2048, 256, device="cuda")        # 128 tiles of 128 x 256: the automatic
    b = torch.rand(256, 2048, device="cuda")        # choice takes the tensor cores
    y = ctx.cuda().matmul(a, b)
    assert h.last_kernel.startswith("simt")
    kx.matmul(a, b)                                  # default handle: automatic choice
    assert kx.handle(0).last_kernel.startswith("tc_")
    ref = a.double() @ b.double()
    assert float((y.double() - ref).abs().max()) <= 1e-5 * float(ref.abs().max())


def test_ordered_context_is_bitwise_matmul_reference(torch_cuda):
    ctx = Context.new(Config.from_toml("[cpu]\nordered_matmul=true"))
    rs = np.random.default_rng(5)
    a = rs.uniform(-1, 1, (37, 300)).astype(np.float32)
    b = rs.uniform(-1, 1, (300, 29)).astype(np.float32)
    want = oracle.matmul_reference(oracle.View.of(a), oracle.View.of(b))
    ex = ctx.cuda()
    got = ex.download(ex.matmul(ex.upload(a), ex.upload(b)))
    assert np.array_equal(got, want)
    out = torch_cuda.empty(37, 29, device="cuda")
    ex.matmul_into(ex.upload(a), ex.upload(b), out)
    assert np.array_equal(out.cpu().numpy(), want)
    with kx.using(ex.h):
        assert np.array_equal(kx.matmul(ex.upload(a), ex.upload(b)).cpu().numpy(), want)
    assert not kx.handle(0).ordered_matmul


def test_device_out_of_range_is_an_execution_error(torch_cuda):
    with pytest.raises(ConfigExecutionError) as e:
        Context.new(Config(cuda=CudaConfig(device=torch_cuda.cuda.device_count())))
    assert isinstance(e.value.error, kx.NoDevice)
