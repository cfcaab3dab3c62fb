"""LaunchError mirror (crates/beacon-cuda/src/error.rs:4-40).

Each C-ABI status code maps onto one variant; messages follow the reference's
Display strings (error.rs:19-40).
"""
from __future__ import annotations

from . import _lib


class LaunchError(Exception):
    """Base of every error a launch can return (error.rs:4)."""

    code = -1


class Unimplemented(LaunchError):
    code = _lib.ERR_UNIMPLEMENTED


class InvalidLaunchConfig(LaunchError):
    code = _lib.ERR_INVALID_LAUNCH_CONFIG


class ModuleLoad(LaunchError):
    code = _lib.ERR_MODULE_LOAD


class FunctionNotFound(LaunchError):
    code = _lib.ERR_FUNCTION_NOT_FOUND


class Cuda(LaunchError):
    code = _lib.ERR_CUDA


class Cublas(LaunchError):
    code = _lib.ERR_CUBLAS


class OutOfMemory(LaunchError):
    code = _lib.ERR_OUT_OF_MEMORY


class ShapeMismatch(LaunchError):
    code = _lib.ERR_SHAPE_MISMATCH


_BY_CODE = {c.code: c for c in (Unimplemented, InvalidLaunchConfig, ModuleLoad, FunctionNotFound, Cuda, Cublas,
                                OutOfMemory, ShapeMismatch)}


def check(rc: int) -> None:
    """Raise the LaunchError variant for a non-zero beacon_status."""
    if rc == _lib.OK:
        return
    cls = _BY_CODE.get(rc, LaunchError)
    raise cls(_lib.last_error())
