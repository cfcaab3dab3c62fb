"""ctypes binding of libbeacon_cuda.so (include/beacon_cuda.h).

The library is built in-tree (``beacon_b200/lib/libbeacon_cuda.so``) by
``beacon_b200/csrc/Makefile``.  Loading fails loudly when it is missing: there
is no CPU fallback behind any entry point.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libbeacon_cuda.so")
CSRC = os.path.join(_HERE, "csrc")

# beacon_status: LaunchError variants (crates/beacon-cuda/src/error.rs:4-13)
OK = 0
ERR_UNIMPLEMENTED = 1
ERR_INVALID_LAUNCH_CONFIG = 2
ERR_MODULE_LOAD = 3
ERR_FUNCTION_NOT_FOUND = 4
ERR_CUDA = 5
ERR_CUBLAS = 6
ERR_OUT_OF_MEMORY = 7
ERR_SHAPE_MISMATCH = 8

# beacon_dtype (crates/beacon-core/src/dtype.rs:1-7)
F32, F16, BF16, FP8E4M3 = 0, 1, 2, 3

# Every symbol include/beacon_cuda.h declares.
EXPORTS = (
    "beacon_version", "beacon_last_error", "beacon_device_status", "beacon_launch_count",
    "beacon_diag_wait_timeout", "beacon_diag_exp2_poly",
    "beacon_profile_enable", "beacon_profile_read",
    "beacon_matmul_plan", "beacon_matmul_fwd", "beacon_matmul_bwd", "beacon_linear_fwd", "beacon_linear_bwd",
    "beacon_matmul_fp8w_fwd", "beacon_linear_fp8w_fwd", "beacon_linear_fp8w_fwd_devscale",
    "beacon_quantize_fp8e4m3",
    "beacon_attention_adjoint_fwd", "beacon_attention_adjoint_bwd", "beacon_attention_bwd_workspace_size",
    "beacon_attention_gqa_fwd", "beacon_attention_gqa_bwd", "beacon_attention_bwd_with_out",
    "beacon_rmsnorm_adjoint_fwd", "beacon_rmsnorm_adjoint_bwd", "beacon_rmsnorm_adjoint_bwd_noalloc",
    "beacon_rmsnorm_fold_weight", "beacon_rmsnorm_linear_fwd",
    "beacon_layernorm_adjoint_fwd", "beacon_layernorm_adjoint_bwd",
    "beacon_swiglu_adjoint_fwd", "beacon_swiglu_adjoint_bwd", "beacon_swiglu_workspace_size",
    "beacon_llama_block_fwd", "beacon_llama_block_workspace_size", "beacon_llama_block_fwd_folded",
    "beacon_residual_add_fwd", "beacon_residual_add_bwd", "beacon_cast",
    "beacon_embedding_lookup_fwd", "beacon_embedding_lookup_bwd", "beacon_dropout_fwd", "beacon_dropout_bwd",
    "beacon_arena_create", "beacon_arena_destroy", "beacon_arena_base", "beacon_arena_size", "beacon_launch",
    "beacon_workspace_create",
)

_lib = None

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t
_fp = ctypes.POINTER(ctypes.c_float)


class KernelArgC(ctypes.Structure):
    """beacon_kernel_arg (KernelArg, crates/beacon-cuda/src/launcher.rs:21-26)."""

    _fields_ = [("offset", ctypes.c_uint64), ("len_bytes", ctypes.c_uint64), ("access", ctypes.c_int32)]


def build(force: bool = False) -> str:
    """Compile libbeacon_cuda.so in place with nvcc for sm_100a."""
    cmd = ["make", "-s", "-C", CSRC]
    if force:
        cmd.insert(1, "-B")
    subprocess.run(cmd, check=True)
    return LIB_PATH


def _sig(L, name, res, args):
    f = getattr(L, name)
    f.restype = res
    f.argtypes = args


def lib():
    """Load the library (raises OSError when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"libbeacon_cuda.so not built at {LIB_PATH}; run beacon_b200._lib.build()")
    L = ctypes.CDLL(LIB_PATH)
    _sig(L, "beacon_version", _int, [])
    _sig(L, "beacon_last_error", _int, [ctypes.c_char_p, _sz])
    _sig(L, "beacon_device_status", _int, [_int, ctypes.POINTER(ctypes.c_uint)])
    _sig(L, "beacon_launch_count", ctypes.c_uint64, [])
    _sig(L, "beacon_diag_wait_timeout", _int, [ctypes.c_uint64, _vp, _vp])
    _sig(L, "beacon_diag_exp2_poly", _int, [_vp, _vp, _i64, _vp])
    _sig(L, "beacon_profile_enable", None, [_int])
    _sig(L, "beacon_profile_read", _int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_double),
                                          ctypes.POINTER(ctypes.c_uint64)])
    _sig(L, "beacon_matmul_plan", _int, [_i64, _i64, _i64, ctypes.POINTER(ctypes.c_int32)])
    _sig(L, "beacon_matmul_fwd", _int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp])
    _sig(L, "beacon_matmul_bwd", _int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp])
    _sig(L, "beacon_linear_fwd", _int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp])
    _sig(L, "beacon_linear_bwd", _int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp])
    _sig(L, "beacon_matmul_fp8w_fwd", _int, [_vp, _vp, _vp, ctypes.c_float, _i64, _i64, _i64, _vp])
    _sig(L, "beacon_linear_fp8w_fwd", _int, [_vp, _vp, _vp, ctypes.c_float, _vp, _i64, _i64, _i64, _vp])
    _sig(L, "beacon_linear_fp8w_fwd_devscale", _int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp])
    _sig(L, "beacon_quantize_fp8e4m3", _int, [_vp, _vp, _vp, _vp, _i64, _vp])
    _sig(L, "beacon_attention_adjoint_fwd", _int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int, _vp])
    _sig(L, "beacon_attention_adjoint_bwd", _int,
         [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int, _vp, _sz, _vp])
    _sig(L, "beacon_attention_bwd_workspace_size", _sz, [_i64, _i64, _i64, _i64, _int])
    _sig(L, "beacon_attention_gqa_fwd", _int,
         [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _int, _int, _vp])
    _sig(L, "beacon_attention_gqa_bwd", _int,
         [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _int, _int, _vp, _sz, _vp])
    _sig(L, "beacon_attention_bwd_with_out", _int,
         [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _int, _int, _vp, _sz, _vp])
    _sig(L, "beacon_rmsnorm_adjoint_fwd", _int, [_vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_float, _int, _vp])
    _sig(L, "beacon_rmsnorm_adjoint_bwd", _int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _int, _vp, _sz, _vp])
    _sig(L, "beacon_rmsnorm_adjoint_bwd_noalloc", _int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _int, _vp])
    _sig(L, "beacon_rmsnorm_fold_weight", _int, [_vp, _vp, _vp, _i64, _i64, _int, _vp])
    _sig(L, "beacon_rmsnorm_linear_fwd", _int,
         [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, ctypes.c_float, _int, _vp])
    _sig(L, "beacon_layernorm_adjoint_fwd", _int,
         [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_float, _int, _vp])
    _sig(L, "beacon_layernorm_adjoint_bwd", _int,
         [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _int, _vp, _sz, _vp])
    _sig(L, "beacon_swiglu_adjoint_fwd", _int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _sz, _vp])
    _sig(L, "beacon_swiglu_adjoint_bwd", _int,
         [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _sz, _vp])
    _sig(L, "beacon_swiglu_workspace_size", _sz, [_i64, _i64, _i64, _int, _int])
    _sig(L, "beacon_llama_block_fwd", _int, [_vp] * 9 + [_i64] * 7 + [ctypes.c_float, _int, _vp, _sz, _vp])
    _sig(L, "beacon_llama_block_workspace_size", _sz, [_i64] * 7 + [_int])
    _sig(L, "beacon_llama_block_fwd_folded", _int, [_vp] * 7 + [_i64] * 7 + [ctypes.c_float, _int, _vp, _sz, _vp])
    _sig(L, "beacon_residual_add_fwd", _int, [_vp, _vp, _vp, _i64, _int, _vp])
    _sig(L, "beacon_residual_add_bwd", _int, [_vp, _vp, _vp, _i64, _int, _vp])
    _sig(L, "beacon_cast", _int, [_vp, _vp, _i64, _int, _vp])
    _sig(L, "beacon_embedding_lookup_fwd", _int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp])
    _sig(L, "beacon_embedding_lookup_bwd", _int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp])
    _sig(L, "beacon_dropout_fwd", _int, [_vp, _vp, _vp, _i64, ctypes.c_float, ctypes.c_uint64, _int, _vp])
    _sig(L, "beacon_dropout_bwd", _int, [_vp, _vp, _vp, _i64, _int, _vp])
    _sig(L, "beacon_arena_create", _vp, [_int, ctypes.c_uint64])
    _sig(L, "beacon_arena_destroy", None, [_vp])
    _sig(L, "beacon_arena_base", _vp, [_vp])
    _sig(L, "beacon_arena_size", ctypes.c_uint64, [_vp])
    _sig(L, "beacon_workspace_create", _int, [_vp, ctypes.c_uint64])
    _sig(L, "beacon_launch", _int, [_vp, ctypes.c_char_p, ctypes.POINTER(KernelArgC), _sz,
                                    ctypes.POINTER(ctypes.c_int64), _sz, _vp])
    _lib = L
    return L


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().beacon_last_error(buf, 512)
    return buf.value.decode(errors="replace")
