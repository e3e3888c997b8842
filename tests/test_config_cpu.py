"""Configuration and execution context on the host (no device work).

Restates kernix/tests/config_tests.rs:4-43 for the mirror of
kernix/src/config.rs, extended to the [cuda] table, and checks that
kx_context_create validates every [cuda] key before it looks for a device.
"""
import ctypes as C
import os
import tempfile
from pathlib import Path

import pytest

import kernix_b200 as kx
from kernix_b200 import _abi
from kernix_b200.config import (Config, ConfigError, ConfigExecutionError, ConfigIoError, ConfigParseError,
                                Context, CpuConfig, CudaConfig)

HAVE_GPU = False
try:
    import torch
    HAVE_GPU = torch.cuda.is_available()
except Exception:  # pragma: no cover
    pass


def test_empty_input_and_missing_optional_file_use_defaults():
    assert Config.from_toml("") == Config()
    path = Path(tempfile.gettempdir()) / f"kernix-absent-{os.getpid()}" / "kernix.toml"
    assert Config.load_optional(path) == Config()
    assert Context().cpu().threads == 1                 # no device, no file touched


def test_shipped_example_file_is_the_defaults():
    """The example file states exactly what Context() uses (kernix.toml:1-2)."""
    here = Path(kx.__file__).parent / "kernix.toml"
    assert Config.load_optional(here) == Config()


@pytest.mark.parametrize("text", [
    "[cpu]\nthread=4", "[gpu]\nthreads=2", "[cpu]\nthreads=-1", "nonsense",
    "[cuda]\nvariant='ffma'", "[cuda]\nf32_variant='tf32'", "[cuda]\nf64_variant='3xtf32'", "[cuda]\ndevice=-1",
    "[cuda]\ndevice=true", "[cuda]\nordered_matmul=1", "[cuda]\nworkspace_mib=1.5", "cuda=3", "[cpu]\nthreads='2'",
    "[cpu]\nthreads=1\n[cpu]\nthreads=2",
])
def test_typos_wrong_types_and_negative_counts_are_parse_errors(text):
    with pytest.raises(ConfigParseError):
        Config.from_toml(text)


def test_zero_threads_is_an_execution_error_naming_the_key():
    with pytest.raises(ConfigExecutionError) as e:
        Config.from_toml("[cpu]\nthreads=0")
    assert isinstance(e.value.error, kx.InvalidParameter)
    assert e.value.error.parameter == "cpu.threads must be positive"
    assert isinstance(e.value, ConfigError)


def test_filesystem_errors_are_not_silently_defaulted(tmp_path):
    with pytest.raises(ConfigIoError) as e:
        Config.load_optional(tempfile.gettempdir())     # a directory
    assert e.value.path == Path(tempfile.gettempdir())
    bad = tmp_path / "bad.toml"
    bad.write_bytes(b"[cpu]\nthreads = 1 # \xff\xfe\n")
    with pytest.raises(ConfigIoError):
        Config.load_optional(bad)                       # not UTF-8
    plain = tmp_path / "plain"
    plain.write_text("")
    with pytest.raises(ConfigIoError):
        Config.load_optional(plain / "kernix.toml")     # a path through a file is not "missing"


def test_valid_explicit_settings():
    config = Config.from_toml("[cpu]\nthreads=1")
    assert config == Config(cpu=CpuConfig(threads=1))
    cfg = Config.from_toml("[cuda]\ndevice=3\nf32_variant='3xtf32-1sm'\nf64_variant='dmma'\nworkspace_mib=64")
    assert cfg.cuda == CudaConfig(device=3, f32_variant="3xtf32-1sm", f64_variant="dmma", workspace_mib=64)
    c = cfg.cuda_c()
    assert (c.device, c.f32_variant, c.f64_variant, c.ordered_matmul, c.workspace_bytes) == (3, 3, 2, 0, 64 << 20)


def test_device_ordered_mode_follows_cpu_unless_set():
    assert Config.from_toml("[cpu]\nordered_matmul=true").cuda_c().ordered_matmul == 1
    assert Config.from_toml("[cpu]\nordered_matmul=true\n[cuda]\nordered_matmul=false").cuda_c().ordered_matmul == 0
    assert Config.from_toml("[cuda]\nordered_matmul=true").cuda_c().ordered_matmul == 1
    assert Config().cuda_c().ordered_matmul == 0


def test_counts_the_abi_cannot_hold_are_rejected():
    with pytest.raises(kx.InvalidParameter):
        Config(cuda=CudaConfig(device=1 << 31)).cuda_c()
    with pytest.raises(kx.InvalidParameter):
        Config(cuda=CudaConfig(workspace_mib=1 << 44)).cuda_c()


def _create(**fields):
    c = _abi.KxCudaConfig()
    _abi.lib.kx_cuda_config_default(C.byref(c))
    for k, v in fields.items():
        setattr(c, k, v)
    ptr, err = C.c_void_p(), _abi.KxError()
    rc = _abi.lib.kx_context_create(C.byref(c), C.byref(ptr), C.byref(err))
    if rc == _abi.KX_OK:
        _abi.lib.kx_destroy(ptr)
    return rc, err.parameter.decode()


def test_context_create_checks_each_key_before_the_device():
    assert _create(device=-1) == (_abi.KX_E_PARAM, "cuda.device must be non-negative")
    assert _create(f32_variant=4) == (_abi.KX_E_PARAM, "cuda.f32_variant is not a kernel family")
    assert _create(f32_variant=-1) == (_abi.KX_E_PARAM, "cuda.f32_variant is not a kernel family")
    assert _create(f64_variant=3) == (_abi.KX_E_PARAM, "cuda.f64_variant is not a kernel family")
    assert _create(ordered_matmul=2) == (_abi.KX_E_PARAM, "cuda.ordered_matmul must be 0 or 1")
    rc, _ = _create()
    assert rc == (_abi.KX_OK if HAVE_GPU else _abi.KX_E_NO_DEVICE)
    ptr = C.c_void_p()
    assert _abi.lib.kx_context_create(None, C.byref(ptr), None) == _abi.KX_E_PARAM


@pytest.mark.skipif(HAVE_GPU, reason="checks the host without a device")
def test_context_new_without_a_device_is_an_execution_error():
    with pytest.raises(ConfigExecutionError) as e:
        Context.new(Config())
    assert isinstance(e.value.error, kx.NoDevice)
