"""Host-side mirror of beacon-cuda's launch layer (crates/beacon-cuda/src/).

KernelId / Access / KernelArg  launcher.rs:5-52
Dim3 / LaunchParams.validate   launch.rs:4-98
kernel IDs and grid helpers    attention.rs:5-18, matmul.rs:5-15, norm.rs:5-17, mlp.rs:5-9,
                               elementwise.rs:5-44
typed traits                   AttentionLaunch, MatmulLaunch, RmsNormLaunch, SwigluLaunch,
                               ElementwiseLaunch (same method names, parameter order and
                               argument lists as the reference)
Launcher                       runtime.rs:6-48: validates the launch parameters, then forwards
                               to beacon_launch() of the C ABI over one device arena.

The one deliberate difference: the reference's typed methods drop their shapes
(`let _ = (m, k, n)`, matmul.rs:27) before KernelLauncher::launch, so a real
launcher could not size the work.  Here `launch` takes those shapes as a
trailing `scalars` tuple; the typed methods' own parameter lists are unchanged.
"""
from __future__ import annotations

import ctypes
import struct
from abc import ABC, abstractmethod
from dataclasses import dataclass, field
from enum import Enum

from . import _lib
from .errors import InvalidLaunchConfig, check

# --------------------------------------------------------------------------- launcher.rs


@dataclass(frozen=True)
class KernelId:
    name_: str

    def name(self) -> str:
        return self.name_


class Access(Enum):
    READ = 0
    WRITE = 1
    READ_WRITE = 2


@dataclass(frozen=True)
class KernelArg:
    """A byte range of the launcher's arena (launcher.rs:21-52)."""

    offset: int
    len_bytes: int
    access: Access

    @staticmethod
    def read(offset, len_bytes):
        return KernelArg(offset, len_bytes, Access.READ)

    @staticmethod
    def write(offset, len_bytes):
        return KernelArg(offset, len_bytes, Access.WRITE)

    @staticmethod
    def read_write(offset, len_bytes):
        return KernelArg(offset, len_bytes, Access.READ_WRITE)


# --------------------------------------------------------------------------- launch.rs

MAX_THREADS_PER_BLOCK = 1024
MAX_DYNAMIC_SMEM_BYTES = 227 * 1024


@dataclass(frozen=True)
class Dim3:
    x: int
    y: int = 1
    z: int = 1

    @staticmethod
    def of(v) -> "Dim3":
        if isinstance(v, Dim3):
            return v
        if isinstance(v, int):
            return Dim3(v, 1, 1)
        v = tuple(v)
        return Dim3(*(v + (1,) * (3 - len(v))))

    def total(self) -> int:
        return self.x * self.y * self.z


@dataclass
class LaunchParams:
    grid: Dim3
    block: Dim3
    shared_mem_bytes: int = 0
    stream: int = 0  # StreamHandle(u64); 0 = default stream (device.rs:6-42)

    @staticmethod
    def new(grid, block) -> "LaunchParams":
        return LaunchParams(Dim3.of(grid), Dim3.of(block))

    def with_shared_mem(self, nbytes: int) -> "LaunchParams":
        self.shared_mem_bytes = nbytes
        return self

    def on_stream(self, stream: int) -> "LaunchParams":
        self.stream = stream
        return self

    def total_threads(self) -> int:
        return self.grid.total() * self.block.total()

    def validate(self) -> None:
        """launch.rs:78-97"""
        if self.grid.total() == 0 or self.block.total() == 0:
            raise InvalidLaunchConfig("grid and block dimensions must be nonzero")
        bt = self.block.total()
        if bt > MAX_THREADS_PER_BLOCK:
            raise InvalidLaunchConfig(f"block has {bt} threads, max is {MAX_THREADS_PER_BLOCK}")
        if self.shared_mem_bytes > MAX_DYNAMIC_SMEM_BYTES:
            raise InvalidLaunchConfig(f"dynamic shared memory {self.shared_mem_bytes} bytes exceeds "
                                      f"max {MAX_DYNAMIC_SMEM_BYTES}")


# --------------------------------------------------------------------------- kernel IDs + grids

class kid:
    # attention.rs:14-18
    ATTENTION_FWD = KernelId("attention_adjoint_fwd")
    ATTENTION_BWD = KernelId("attention_adjoint_bwd")
    # matmul.rs:5-11
    MATMUL_FWD = KernelId("matmul_fwd")
    MATMUL_BWD = KernelId("matmul_bwd")
    LINEAR_FWD = KernelId("linear_fwd")
    LINEAR_BWD = KernelId("linear_bwd")
    # norm.rs:11-17
    RMSNORM_FWD = KernelId("rmsnorm_adjoint_fwd")
    RMSNORM_BWD = KernelId("rmsnorm_adjoint_bwd")
    LAYERNORM_FWD = KernelId("layernorm_adjoint_fwd")
    LAYERNORM_BWD = KernelId("layernorm_adjoint_bwd")
    # mlp.rs:5-9
    SWIGLU_FWD = KernelId("swiglu_adjoint_fwd")
    SWIGLU_BWD = KernelId("swiglu_adjoint_bwd")
    # elementwise.rs:13-25
    RESIDUAL_ADD_FWD = KernelId("residual_add_fwd")
    RESIDUAL_ADD_BWD = KernelId("residual_add_bwd")
    EMBEDDING_FWD = KernelId("embedding_lookup_fwd")
    EMBEDDING_BWD = KernelId("embedding_lookup_bwd")
    DROPOUT_FWD = KernelId("dropout_fwd")
    DROPOUT_BWD = KernelId("dropout_bwd")
    CAST_F32_TO_FP8E4M3 = KernelId("cast_f32_to_fp8e4m3")
    CAST_FP8E4M3_TO_F32 = KernelId("cast_fp8e4m3_to_f32")
    CAST_F32_TO_BF16 = KernelId("cast_f32_to_bf16")
    CAST_BF16_TO_F32 = KernelId("cast_bf16_to_f32")


ATTN_Q_TILE = 64
ATTN_BLOCK = 128
NORM_BLOCK = 256
ELEMENTWISE_BLOCK = 256


def attention_grid(batch, heads, seqlen) -> LaunchParams:
    """attention.rs:8-12"""
    q_blocks = max((seqlen + ATTN_Q_TILE - 1) // ATTN_Q_TILE, 1)
    return LaunchParams.new((max(batch * heads, 1), q_blocks), ATTN_BLOCK)


def cublas_params() -> LaunchParams:
    """matmul.rs:13-15"""
    return LaunchParams.new(1, 1)


def rowwise(rows) -> LaunchParams:
    """norm.rs:7-9"""
    return LaunchParams.new(max(rows, 1), NORM_BLOCK)


def elementwise_grid(n) -> LaunchParams:
    """elementwise.rs:7-11"""
    return LaunchParams.new(max((n + ELEMENTWISE_BLOCK - 1) // ELEMENTWISE_BLOCK, 1), ELEMENTWISE_BLOCK)


class CastKind(Enum):
    """elementwise.rs:27-44"""

    F32_TO_F8E4M3 = 0
    F8E4M3_TO_F32 = 1
    F32_TO_BF16 = 2
    BF16_TO_F32 = 3

    def kernel(self) -> KernelId:
        return {0: kid.CAST_F32_TO_FP8E4M3, 1: kid.CAST_FP8E4M3_TO_F32, 2: kid.CAST_F32_TO_BF16,
                3: kid.CAST_BF16_TO_F32}[self.value]


BF16 = _lib.BF16
F32 = _lib.F32


# --------------------------------------------------------------------------- traits

class KernelLauncher(ABC):
    """launcher.rs:54-63"""

    @abstractmethod
    def device(self) -> int: ...

    @abstractmethod
    def launch(self, kernel: KernelId, params: LaunchParams, args, scalars=()) -> None: ...


class MatmulLaunch:
    """matmul.rs:17-81"""

    def matmul_fwd(self, out, lhs, rhs, m, k, n, dtype=BF16):
        self.launch(kid.MATMUL_FWD, cublas_params(), [out, lhs, rhs], (m, k, n, dtype))

    def matmul_bwd(self, dlhs, drhs, dout, lhs, rhs, m, k, n, dtype=BF16):
        self.launch(kid.MATMUL_BWD, cublas_params(), [dlhs, drhs, dout, lhs, rhs], (m, k, n, dtype))

    def linear_fwd(self, out, x, weight, bias, m, k, n, dtype=BF16):
        self.launch(kid.LINEAR_FWD, cublas_params(), [out, x, weight, bias], (m, k, n, dtype))

    def linear_bwd(self, dx, dweight, dbias, dout, x, weight, m, k, n, dtype=BF16):
        self.launch(kid.LINEAR_BWD, cublas_params(), [dx, dweight, dbias, dout, x, weight], (m, k, n, dtype))


class AttentionLaunch:
    """attention.rs:20-67"""

    def attention_fwd(self, out, q, k, v, lse, batch, heads, seqlen, head_dim, causal, dtype=BF16):
        self.launch(kid.ATTENTION_FWD, attention_grid(batch, heads, seqlen), [out, q, k, v, lse],
                    (batch, heads, seqlen, head_dim, int(causal), dtype))

    def attention_bwd(self, dq, dk, dv, dout, q, k, v, lse, batch, heads, seqlen, head_dim, causal, dtype=BF16):
        self.launch(kid.ATTENTION_BWD, attention_grid(batch, heads, seqlen), [dq, dk, dv, dout, q, k, v, lse],
                    (batch, heads, seqlen, head_dim, int(causal), dtype))


class RmsNormLaunch:
    """norm.rs:19-53"""

    def rmsnorm_fwd(self, out, x, weight, rms, tokens, dim, dtype=BF16):
        self.launch(kid.RMSNORM_FWD, rowwise(tokens), [out, x, weight, rms], (tokens, dim, dtype))

    def rmsnorm_bwd(self, dx, dweight, dy, x, rms, weight, tokens, dim, dtype=BF16):
        self.launch(kid.RMSNORM_BWD, rowwise(tokens), [dx, dweight, dy, x, rms, weight], (tokens, dim, dtype))


class LayerNormLaunch:
    """norm.rs:55-95"""

    def layernorm_fwd(self, out, x, weight, bias, mean, invstd, tokens, dim, dtype=BF16):
        self.launch(kid.LAYERNORM_FWD, rowwise(tokens), [out, x, weight, bias, mean, invstd], (tokens, dim, dtype))

    def layernorm_bwd(self, dx, dweight, dbias, dy, x, mean, invstd, weight, tokens, dim, dtype=BF16):
        self.launch(kid.LAYERNORM_BWD, rowwise(tokens), [dx, dweight, dbias, dy, x, mean, invstd, weight],
                    (tokens, dim, dtype))


class SwigluLaunch:
    """mlp.rs:11-55"""

    def swiglu_fwd(self, out, x, gate_proj, up_proj, down_proj, tokens, d_model, d_ff, dtype=BF16):
        self.launch(kid.SWIGLU_FWD, elementwise_grid(tokens * d_ff), [out, x, gate_proj, up_proj, down_proj],
                    (tokens, d_model, d_ff, dtype))

    def swiglu_bwd(self, dx, dgate_proj, dup_proj, ddown_proj, dy, x, gate_proj, up_proj, down_proj, tokens,
                   d_model, d_ff, dtype=BF16):
        self.launch(kid.SWIGLU_BWD, elementwise_grid(tokens * d_ff),
                    [dx, dgate_proj, dup_proj, ddown_proj, dy, x, gate_proj, up_proj, down_proj],
                    (tokens, d_model, d_ff, dtype))


class ElementwiseLaunch:
    """elementwise.rs:46-131"""

    def residual_add(self, out, a, b, n, dtype=BF16):
        self.launch(kid.RESIDUAL_ADD_FWD, elementwise_grid(n), [out, a, b], (n, dtype))

    def residual_add_backward(self, d_a, d_b, d_out, n, dtype=BF16):
        self.launch(kid.RESIDUAL_ADD_BWD, elementwise_grid(n), [d_a, d_b, d_out], (n, dtype))

    def embedding_lookup(self, out, table, indices, tokens, dim, dtype=BF16):
        self.launch(kid.EMBEDDING_FWD, elementwise_grid(tokens * dim), [out, table, indices], (tokens, dim, dtype))

    def embedding_backward(self, d_table, d_out, indices, tokens, dim, dtype=BF16):
        self.launch(kid.EMBEDDING_BWD, elementwise_grid(tokens * dim), [d_table, d_out, indices],
                    (tokens, dim, dtype))

    def dropout_forward(self, out, inp, mask, n, p, seed, dtype=BF16):
        p_bits = struct.unpack("<I", struct.pack("<f", float(p)))[0]
        self.launch(kid.DROPOUT_FWD, elementwise_grid(n), [out, inp, mask], (n, p_bits, seed, dtype))

    def dropout_backward(self, d_in, d_out, mask, n, dtype=BF16):
        self.launch(kid.DROPOUT_BWD, elementwise_grid(n), [d_in, d_out, mask], (n, dtype))

    def cast(self, dst, src, n, kind: CastKind):
        self.launch(kind.kernel(), elementwise_grid(n), [dst, src], (n,))


class AllLaunch(MatmulLaunch, AttentionLaunch, RmsNormLaunch, LayerNormLaunch, SwigluLaunch, ElementwiseLaunch):
    """Every typed trait, as the reference blanket-implements them on any KernelLauncher."""


# --------------------------------------------------------------------------- implementers

class Recorder(KernelLauncher, AllLaunch):
    """Fake launcher that records (kernel name, #args) (crates/beacon-cuda/src/testutil.rs:7-33)."""

    def __init__(self):
        self._calls = []

    def device(self) -> int:
        return 0

    def launch(self, kernel, params, args, scalars=()):
        params.validate()
        self._calls.append((kernel.name(), len(args)))

    def calls(self):
        return list(self._calls)


@dataclass
class Launcher(KernelLauncher, AllLaunch):
    """runtime.rs:6-48 over a device arena of `arena_bytes` (libbeacon_cuda.so)."""

    ordinal: int = 0
    arena_bytes: int = 1 << 20
    workspace_bytes: int = 0
    _arena: int = field(default=0, init=False, repr=False)

    def __post_init__(self):
        L = _lib.lib()
        self._arena = L.beacon_arena_create(self.ordinal, self.arena_bytes)
        if not self._arena:
            raise MemoryError(_lib.last_error())
        if self.workspace_bytes:
            self.reserve_workspace(self.workspace_bytes)

    @staticmethod
    def on_device(ordinal: int, arena_bytes: int = 1 << 20, workspace_bytes: int = 0) -> "Launcher":
        return Launcher(ordinal, arena_bytes, workspace_bytes)

    def reserve_workspace(self, nbytes: int) -> None:
        """The launcher's scratch, made once (kernels launched through it never allocate)."""
        check(_lib.lib().beacon_workspace_create(self._arena, int(nbytes)))
        self.workspace_bytes = int(nbytes)

    def device(self) -> int:
        return self.ordinal

    def base_ptr(self) -> int:
        return int(_lib.lib().beacon_arena_base(self._arena) or 0)

    def launch(self, kernel, params, args, scalars=()):
        params.validate()
        arr = (_lib.KernelArgC * len(args))(*[_lib.KernelArgC(a.offset, a.len_bytes, a.access.value) for a in args])
        sc = (ctypes.c_int64 * max(len(scalars), 1))(*[int(s) for s in scalars])
        check(_lib.lib().beacon_launch(self._arena, kernel.name().encode(), arr, len(args), sc, len(scalars),
                                       ctypes.c_void_p(params.stream)))

    def close(self):
        if self._arena:
            _lib.lib().beacon_arena_destroy(self._arena)
            self._arena = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
