"""Configuration and execution context: Kernix's ``config`` module with a
``[cuda]`` table beside ``[cpu]``.

Mirrors kernix/src/config.rs: ``Config.from_toml`` (:84-95) parses strict
TOML (unknown tables and keys, wrong types and negative counts are parse
errors; ``cpu.threads = 0`` is an execution error naming the key),
``Config.load_optional`` (:98-125) treats only a missing file as "use the
defaults" and keeps every other filesystem failure with its path, and
``Context.new`` (:133-137) validates the settings by building the executors
they ask for.  The CUDA executor comes from ``kx_context_create``, which checks
each ``[cuda]`` key before it touches a device.

``[cuda]`` keys (all optional)::

    device = 0                  # CUDA ordinal
    f32_variant = "auto"        # auto | ffma | 3xtf32 | 3xtf32-1sm
    f64_variant = "auto"        # auto | dfma | dmma
    ordered_matmul = false      # absent: follows [cpu] ordered_matmul
    workspace_mib = 0           # device scratch reserved when the context is made

The ``[cpu]`` table keeps the reference's meaning (threads, ordered_matmul) for
the caller's own CPU executor; this package computes on the device only.
"""
from __future__ import annotations

import ctypes as C
import errno
import os
import stat
import tomllib
from dataclasses import dataclass, field
from pathlib import Path

from . import _abi
from ._abi import InvalidParameter, KxCudaConfig, KxError, OpsError, raise_for

F32_VARIANTS = {"auto": 0, "ffma": 1, "3xtf32": 2, "3xtf32-1sm": 3}
F64_VARIANTS = {"auto": 0, "dfma": 1, "dmma": 2}


class ConfigError(Exception):
    """ConfigError (config.rs:43-57): Parse, Io or Execution."""


class ConfigParseError(ConfigError):
    """ConfigError::Parse: invalid TOML syntax or schema (unknown keys included)."""


class ConfigIoError(ConfigError):
    """ConfigError::Io: reading an explicitly requested file failed."""

    def __init__(self, path, source: Exception):
        super().__init__(f"cannot read Kernix configuration {path}: {source}")
        self.path = Path(path)
        self.source = source


class ConfigExecutionError(ConfigError):
    """ConfigError::Execution: the settings cannot be fulfilled (wraps an OpsError)."""

    def __init__(self, error: OpsError):
        super().__init__(f"cannot create Kernix execution context: {error}")
        self.error = error


ConfigError.Parse = ConfigParseError
ConfigError.Io = ConfigIoError
ConfigError.Execution = ConfigExecutionError


@dataclass(frozen=True)
class CpuConfig:
    """CpuConfig (config.rs:28-40)."""

    threads: int = 1
    ordered_matmul: bool = False


@dataclass(frozen=True)
class CudaConfig:
    """The [cuda] table (kx_cuda_config)."""

    device: int = 0
    f32_variant: str = "auto"
    f64_variant: str = "auto"
    ordered_matmul: bool | None = None
    workspace_mib: int = 0


def _count(table: str, key: str, value) -> int:
    # serde's usize: a TOML integer (not a boolean), not negative
    if isinstance(value, bool) or not isinstance(value, int) or value < 0:
        raise ConfigParseError(f"invalid Kernix configuration: {table}.{key}: expected a non-negative integer, "
                               f"found {value!r}")
    return value


def _flag(table: str, key: str, value) -> bool:
    if not isinstance(value, bool):
        raise ConfigParseError(f"invalid Kernix configuration: {table}.{key}: expected a boolean, found {value!r}")
    return value


def _name(table: str, key: str, value, names: dict) -> str:
    if not isinstance(value, str) or value not in names:
        raise ConfigParseError(f"invalid Kernix configuration: {table}.{key}: expected one of "
                               f"{', '.join(names)}, found {value!r}")
    return value


_SCHEMA = {
    "cpu": (CpuConfig, {"threads": _count, "ordered_matmul": _flag}),
    "cuda": (CudaConfig, {"device": _count, "ordered_matmul": _flag, "workspace_mib": _count,
                          "f32_variant": lambda t, k, v: _name(t, k, v, F32_VARIANTS),
                          "f64_variant": lambda t, k, v: _name(t, k, v, F64_VARIANTS)}),
}


@dataclass(frozen=True)
class Config:
    """Config (config.rs:19-24) plus the [cuda] table."""

    cpu: CpuConfig = field(default_factory=CpuConfig)
    cuda: CudaConfig = field(default_factory=CudaConfig)

    @staticmethod
    def from_toml(text: str) -> "Config":
        """Strict parse (config.rs:84-95): empty input gives the defaults."""
        try:
            doc = tomllib.loads(text)
        except tomllib.TOMLDecodeError as e:
            raise ConfigParseError(f"invalid Kernix configuration: {e}") from e
        tables = {}
        for name, value in doc.items():
            if name not in _SCHEMA:
                raise ConfigParseError(f"invalid Kernix configuration: unknown field `{name}`, expected one of "
                                       f"{', '.join(_SCHEMA)}")
            cls, keys = _SCHEMA[name]
            if not isinstance(value, dict):
                raise ConfigParseError(f"invalid Kernix configuration: `{name}` must be a table")
            kw = {}
            for key, v in value.items():
                if key not in keys:
                    raise ConfigParseError(f"invalid Kernix configuration: unknown field `{key}` in [{name}], "
                                           f"expected one of {', '.join(keys)}")
                kw[key] = keys[key](name, key, v)
            tables[name] = cls(**kw)
        config = Config(**tables)
        if config.cpu.threads == 0:
            raise ConfigExecutionError(InvalidParameter("Config::from_toml: cpu.threads must be positive",
                                                        operation="Config::from_toml",
                                                        parameter="cpu.threads must be positive"))
        return config

    @staticmethod
    def load_optional(path) -> "Config":
        """Read an explicitly chosen optional file (config.rs:98-125): only a
        missing file selects the defaults; other failures keep the path."""
        try:
            meta = os.stat(path)
        except FileNotFoundError:
            return Config()
        except OSError as e:
            raise ConfigIoError(path, e) from e
        if not stat.S_ISREG(meta.st_mode):
            raise ConfigIoError(path, OSError(errno.EINVAL, "configuration path is not a regular file"))
        try:
            text = Path(path).read_bytes().decode("utf-8")
        except (OSError, UnicodeDecodeError) as e:
            raise ConfigIoError(path, e) from e
        return Config.from_toml(text)

    def cuda_c(self) -> KxCudaConfig:
        """The [cuda] table as the C ABI's kx_cuda_config; an absent
        ordered_matmul follows [cpu] ordered_matmul."""
        cu = self.cuda
        if cu.device > 0x7FFFFFFF:
            raise InvalidParameter("Context::new: cuda.device out of range", operation="Context::new",
                                   parameter="cuda.device out of range")
        if cu.workspace_mib >= 1 << 44:
            raise InvalidParameter("Context::new: cuda.workspace_mib out of range", operation="Context::new",
                                   parameter="cuda.workspace_mib out of range")
        c = KxCudaConfig()
        _abi.lib.kx_cuda_config_default(C.byref(c))
        c.device = cu.device
        c.f32_variant = F32_VARIANTS[cu.f32_variant]
        c.f64_variant = F64_VARIANTS[cu.f64_variant]
        ordered = self.cpu.ordered_matmul if cu.ordered_matmul is None else cu.ordered_matmul
        c.ordered_matmul = int(ordered)
        c.workspace_bytes = cu.workspace_mib << 20
        return c


def create_handle(config: Config):
    """A library handle with the [cuda] settings (kx_context_create)."""
    from . import Handle
    c = config.cuda_c()             # InvalidParameter for counts the C struct cannot hold
    ptr = C.c_void_p()
    err = KxError()
    raise_for(_abi.lib.kx_context_create(C.byref(c), C.byref(ptr), C.byref(err)), err)
    return Handle.adopt(ptr, config.cuda.device)


class Context:
    """An application-owned execution context (config.rs:127-150).

    ``Context.new(config)`` validates the settings by creating the CUDA
    executor at once (errors are ConfigExecutionError wrapping the OpsError);
    ``Context()`` holds the defaults, which are valid by construction, and
    creates its executor on first use (it reads no file either way)."""

    def __init__(self, config: Config | None = None, _executor=None):
        self._config = config if config is not None else Config()
        self._cuda = _executor

    @staticmethod
    def new(config: Config) -> "Context":
        from . import CudaExecutor
        try:
            h = create_handle(config)
        except OpsError as e:
            raise ConfigExecutionError(e) from e
        return Context(config, CudaExecutor(config.cuda.device, _handle=h))

    @staticmethod
    def from_file(path) -> "Context":
        """Load optional TOML from a caller-chosen path, then validate (config.rs:139-142)."""
        return Context.new(Config.load_optional(path))

    def config(self) -> Config:
        return self._config

    def cpu(self) -> CpuConfig:
        """The [cpu] settings, carried for the caller's CPU executor."""
        return self._config.cpu

    def cuda(self):
        """This context's CudaExecutor (a MatmulDevice on the configured GPU)."""
        if self._cuda is None:
            from . import CudaExecutor
            self._cuda = CudaExecutor(self._config.cuda.device, _handle=create_handle(self._config))
        return self._cuda


def settings(h) -> dict:
    """The settings a handle runs with (kx_handle_config), by [cuda] key."""
    c = KxCudaConfig()
    rc = _abi.lib.kx_handle_config(h.ptr, C.byref(c))
    raise_for(rc, None)
    f32 = {v: k for k, v in F32_VARIANTS.items()}
    f64 = {v: k for k, v in F64_VARIANTS.items()}
    return {"device": c.device, "f32_variant": f32[c.f32_variant], "f64_variant": f64[c.f64_variant],
            "ordered_matmul": bool(c.ordered_matmul), "workspace_bytes": int(c.workspace_bytes)}


__all__ = [
    "Config", "CpuConfig", "CudaConfig", "Context", "ConfigError", "ConfigParseError", "ConfigIoError",
    "ConfigExecutionError", "F32_VARIANTS", "F64_VARIANTS", "create_handle", "settings",
]
