"""The C-ABI library without a GPU: it loads, exports every symbol the header
declares, and its host-side checks (dtype, shapes, arena extents, kernel-ID
dispatch) answer with the right LaunchError variant before touching a device."""
import ctypes
import os
import re

import pytest

from beacon_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "beacon_cuda.h")


def header_symbols():
    text = open(HEADER).read()
    # function declarations: "<type> [*]beacon_name(" at the start of a line
    return sorted(set(re.findall(r"^[a-z_0-9]+\*?\s+\*?(beacon_[a-z0-9_]+)\s*\(", text, re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    declared = header_symbols()
    assert len(declared) >= 25
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing
    assert sorted(_lib.EXPORTS) == declared


def test_version_and_workspace_sizes():
    L = _lib.lib()
    assert L.beacon_version() == 100
    ws = L.beacon_attention_bwd_workspace_size(8, 32, 4096, 128, _lib.BF16)
    rows = 8 * 32 * 4096
    # Dt and lse2 (fp32) per query row; neither the recomputed O nor dQ needs a buffer
    assert ws >= rows * 4 * 2
    assert ws < rows * 4 * 2 + 4096
    assert L.beacon_attention_bwd_workspace_size(0, 32, 4096, 128, _lib.BF16) == 0
    assert L.beacon_swiglu_workspace_size(8192, 4096, 14336, _lib.BF16, 0) >= 8192 * 14336 * 2


def test_host_side_errors_map_to_launch_error_variants():
    L = _lib.lib()
    rc = L.beacon_matmul_fwd(None, None, None, 8, 8, 8, _lib.F16, None)
    assert rc == _lib.ERR_UNIMPLEMENTED
    assert "dtype" in _lib.last_error()
    assert L.beacon_cast(None, None, 16, 9, None) == _lib.ERR_INVALID_LAUNCH_CONFIG
    assert L.beacon_residual_add_fwd(None, None, None, -1, _lib.BF16, None) == _lib.ERR_INVALID_LAUNCH_CONFIG
    assert L.beacon_launch(None, b"matmul_fwd", None, 0, None, 0, None) == _lib.ERR_INVALID_LAUNCH_CONFIG


class _FakeArena(ctypes.Structure):
    # layout of struct beacon_arena (beacon_b200/csrc/abi_arena.inc)
    _fields_ = [("device", ctypes.c_int), ("base", ctypes.c_void_p), ("bytes", ctypes.c_uint64)]


def _launch(kernel, args, scalars):
    L = _lib.lib()
    buf = ctypes.create_string_buffer(4096)
    arena = _FakeArena(0, ctypes.cast(buf, ctypes.c_void_p), 4096)
    arr = (_lib.KernelArgC * len(args))(*[_lib.KernelArgC(o, n, 0) for o, n in args])
    sc = (ctypes.c_int64 * max(len(scalars), 1))(*scalars)
    return L.beacon_launch(ctypes.byref(arena), kernel, arr, len(args), sc, len(scalars), None)


def test_arena_dispatch_host_checks():
    # IDs outside the hot path answer Unimplemented with their name, like runtime.rs:41
    # dropout_fwd needs p and the seed among its scalars
    assert _launch(b"dropout_fwd", [(0, 16)] * 3, [4]) == _lib.ERR_INVALID_LAUNCH_CONFIG
    assert "dropout_fwd" in _lib.last_error()
    # embedding: the indices (u32) must cover the tokens
    assert _launch_access(b"embedding_lookup_fwd", [(0, 64, 1), (64, 64, 0), (128, 8, 0)], [4, 8, _lib.BF16]) == \
        _lib.ERR_SHAPE_MISMATCH
    assert _launch(b"no_such_kernel", [(0, 16)], []) == _lib.ERR_FUNCTION_NOT_FOUND
    # an argument reaching past the arena
    assert _launch(b"matmul_fwd", [(4000, 512), (0, 128), (0, 128)], [8, 4, 8, _lib.BF16]) == \
        _lib.ERR_INVALID_LAUNCH_CONFIG
    # extents too small for the stated shapes
    assert _launch(b"matmul_fwd", [(0, 64), (0, 64), (0, 64)], [8, 8, 8, _lib.BF16]) == _lib.ERR_SHAPE_MISMATCH
    assert "expected argument 0 of matmul_fwd" in _lib.last_error()
    # attention scalars must describe the tensors
    assert _launch(b"attention_adjoint_fwd", [(0, 8)] * 5, [1, 1, 4, 0, 1, _lib.BF16]) == \
        _lib.ERR_INVALID_LAUNCH_CONFIG
    # layernorm: bad scalars, then an argument smaller than the stated rows x dim
    assert _launch(b"layernorm_adjoint_fwd", [(0, 16)] * 6, [4]) == _lib.ERR_INVALID_LAUNCH_CONFIG
    assert _launch(b"layernorm_adjoint_bwd", [(0, 64)] * 8, [4, 16, _lib.BF16]) == _lib.ERR_SHAPE_MISMATCH
    assert "layernorm_adjoint_bwd" in _lib.last_error()


# Every entry point validates its pointers before it asks for a device: each case below
# passes one required pointer as NULL (the rest point at a 16-byte aligned host buffer,
# never dereferenced) and must be answered with InvalidLaunchConfig.  Without a GPU,
# an entry that reached the device first would answer Cuda or ModuleLoad instead.
_BUF = ctypes.create_string_buffer(1 << 16)
_H = (ctypes.addressof(_BUF) + 255) & ~255  # 256-byte aligned host address


def _null_cases():
    b, f = _lib.BF16, _lib.F32
    h = _H
    return [
        # name, args with None at the position of each required pointer to try, positions
        ("beacon_matmul_fwd", [h, h, h, 8, 8, 8, b, None], [0, 1, 2]),
        ("beacon_matmul_bwd", [h, h, h, h, h, 8, 8, 8, b, None], [2, 3, 4]),
        ("beacon_linear_fwd", [h, h, h, None, 8, 8, 8, b, None], [0, 1, 2]),
        ("beacon_linear_bwd", [None, None, h, h, h, h, 8, 8, 8, b, None], [3]),
        ("beacon_matmul_fp8w_fwd", [h, h, h, 1.0, 8, 8, 8, None], [0, 1, 2]),
        ("beacon_attention_adjoint_fwd", [h, h, h, h, h, 1, 2, 128, 64, 1, b, None], [0, 1, 2, 3, 4]),
        ("beacon_attention_adjoint_bwd",
         [h, h, h, h, h, h, h, h, 1, 2, 128, 64, 1, b, None, 0, None], [0, 1, 2, 3, 4, 5, 6, 7]),
        ("beacon_attention_gqa_fwd", [h, h, h, h, h, 1, 4, 2, 128, 64, 1, b, None], [0, 1, 2, 3, 4]),
        ("beacon_rmsnorm_adjoint_fwd", [h, h, h, h, 4, 64, 1e-5, b, None], [0, 1, 2, 3]),
        ("beacon_rmsnorm_adjoint_bwd", [h, h, h, h, h, h, 4, 64, f, None, 0, None], [0, 2, 3, 4, 5]),
        ("beacon_rmsnorm_adjoint_bwd_noalloc", [h, h, h, h, h, h, 4, 64, b, None], [0, 2, 3, 4, 5]),
        ("beacon_layernorm_adjoint_fwd", [h, h, h, h, h, h, 4, 64, 1e-5, b, None], [0, 1, 2, 3, 4, 5]),
        ("beacon_layernorm_adjoint_bwd", [h, h, h, h, h, h, h, h, 4, 64, b, None, 0, None], [0, 3, 4, 5, 6, 7]),
        ("beacon_swiglu_adjoint_fwd", [h, h, h, h, h, 8, 16, 32, b, None, 0, None], [0, 1, 2, 3, 4]),
        ("beacon_swiglu_adjoint_bwd", [h, h, h, h, h, h, h, h, h, 8, 16, 32, b, None, 0, None], [4, 5, 6, 7, 8]),
        ("beacon_llama_block_fwd",
         [h] * 9 + [1, 128, 128, 2, 1, 64, 256, 1e-5, b, None, 0, None], list(range(9))),
        ("beacon_residual_add_fwd", [h, h, h, 64, b, None], [0, 1, 2]),
        ("beacon_residual_add_bwd", [h, h, h, 64, b, None], [2]),
        ("beacon_cast", [h, h, 64, 2, None], [0, 1]),
    ]


@pytest.mark.parametrize("name,args,positions", _null_cases(), ids=lambda v: v if isinstance(v, str) else "")
def test_null_pointers_rejected_before_any_device_call(name, args, positions):
    L = _lib.lib()
    fn = getattr(L, name)
    for pos in positions:
        a = list(args)
        a[pos] = None
        rc = fn(*a)
        assert rc == _lib.ERR_INVALID_LAUNCH_CONFIG, (name, pos, rc, _lib.last_error())
        assert "null pointer" in _lib.last_error(), (name, pos, _lib.last_error())


def _launch_access(kernel, args, scalars):
    """beacon_launch over a host-memory stand-in arena; args are (offset, len, access)."""
    L = _lib.lib()
    buf = ctypes.create_string_buffer(4096)
    arena = _FakeArena(0, ctypes.cast(buf, ctypes.c_void_p), 4096)
    arr = (_lib.KernelArgC * len(args))(*[_lib.KernelArgC(o, n, acc) for o, n, acc in args])
    sc = (ctypes.c_int64 * max(len(scalars), 1))(*scalars)
    return L.beacon_launch(ctypes.byref(arena), kernel, arr, len(args), sc, len(scalars), None)


def test_arena_dispatch_checks_access_modes():
    """A kernel never writes through an argument declared Read (launcher.rs:14-19); the
    check runs on the host before any device call."""
    R, W, RW = 0, 1, 2
    mm = [8, 4, 8, _lib.BF16]  # out 128 B, lhs 64 B, rhs 64 B
    rc = _launch_access(b"matmul_fwd", [(0, 128, R), (128, 64, R), (256, 64, R)], mm)
    assert rc == _lib.ERR_INVALID_LAUNCH_CONFIG and "declared Read" in _lib.last_error()
    rc = _launch_access(b"matmul_fwd", [(0, 128, 7), (128, 64, R), (256, 64, R)], mm)
    assert rc == _lib.ERR_INVALID_LAUNCH_CONFIG and "access 7" in _lib.last_error()
    # attention backward writes dq, dk, dv (arguments 0-2)
    at = [1, 1, 16, 16, 1, _lib.BF16]
    q = 16 * 16 * 2
    args = [(0, q, W), (q, q, RW), (2 * q, q, R)] + [(3 * q, q, R)] * 4 + [(3 * q, 64, R)]
    rc = _launch_access(b"attention_adjoint_bwd", args, at)
    assert rc == _lib.ERR_INVALID_LAUNCH_CONFIG and "argument 2" in _lib.last_error()
    # with Write / ReadWrite outputs the host checks pass and the call goes on to the
    # device (none in this container: the answer is then a CUDA-side error).  The stand-in
    # arena is host memory, so this step runs only where no GPU could receive the launch.
    import torch
    if not torch.cuda.is_available():
        rc = _launch_access(b"matmul_fwd", [(0, 128, W), (128, 64, R), (256, 64, RW)], mm)
        assert rc not in (_lib.OK, _lib.ERR_INVALID_LAUNCH_CONFIG, _lib.ERR_SHAPE_MISMATCH), _lib.last_error()


def test_matmul_plan_rejects_null_output_and_bad_shapes_before_any_device_call():
    L = _lib.lib()
    assert L.beacon_matmul_plan(64, 64, 64, None) == _lib.ERR_INVALID_LAUNCH_CONFIG
    out = (ctypes.c_int32 * 5)()
    assert L.beacon_matmul_plan(0, 64, 64, out) == _lib.ERR_INVALID_LAUNCH_CONFIG
    assert "bad shape" in _lib.last_error()
