"""The drop-in boundary end to end on the GPU: tensors placed in one device arena, kernels
launched through the reference's trait methods (beacon_b200.launcher.Launcher ->
beacon_launch, crates/beacon-cuda/src/runtime.rs:31-47) with byte-offset KernelArgs
(launcher.rs:21-52), results checked against the oracle.  The launcher reserves its
workspace once; the launches themselves allocate nothing."""
import numpy as np
import pytest

import oracle as O
from helpers import BF16_TOL, as_bf16, normal, rel_err, uniform

pytestmark = pytest.mark.gpu


class _ArenaView:
    """A uint8 torch view of the arena's device memory (by __cuda_array_interface__)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


class _Bump:
    """256-byte aligned regions of the arena, like crates/beacon-core/src/arena.rs:7."""

    def __init__(self):
        self.off = 0

    def take(self, nbytes):
        o = self.off
        self.off = (o + nbytes + 255) & ~255
        return o


def _setup(arena_bytes, ws_bytes):
    import torch
    from beacon_b200.launcher import Launcher
    la = Launcher.on_device(0, arena_bytes, ws_bytes)
    view = torch.as_tensor(_ArenaView(la.base_ptr(), arena_bytes), device="cuda")
    return la, view


def _put(view, off, arr, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(arr)).to(dtype).cuda().contiguous().view(torch.uint8).flatten()
    view[off:off + t.numel()].copy_(t)
    return t.numel()


def _get(view, off, shape, dtype):
    import torch
    n = int(np.prod(shape)) * torch.empty(0, dtype=dtype).element_size()
    return view[off:off + n].clone().view(dtype).reshape(shape).float().cpu().numpy()


def test_attention_and_matmul_through_the_arena_launcher():
    import torch
    from beacon_b200 import _lib
    from beacon_b200.launcher import KernelArg
    B, H, S, D = 1, 4, 256, 128
    ws = int(_lib.lib().beacon_attention_bwd_workspace_size(B, H, S, D, _lib.BF16))
    la, view = _setup(64 << 20, ws)
    bump = _Bump()
    nq = B * H * S * D
    q = as_bf16(normal((B, H, S, D), 91))
    k = as_bf16(normal((B, H, S, D), 91, offset=nq))
    v = as_bf16(normal((B, H, S, D), 91, offset=2 * nq))
    do = as_bf16(normal((B, H, S, D), 91, offset=3 * nq))
    tb = nq * 2
    o_q, o_k, o_v, o_do = (bump.take(tb) for _ in range(4))
    o_out, o_dq, o_dk, o_dv = (bump.take(tb) for _ in range(4))
    o_lse = bump.take(B * H * S * 4)
    for off, a in ((o_q, q), (o_k, k), (o_v, v), (o_do, do)):
        _put(view, off, a, torch.bfloat16)
    m, kk, n = 256, 512, 384
    a_m = as_bf16(uniform((m, kk), 92))
    b_m = as_bf16(uniform((kk, n), 93))
    o_a, o_b, o_c = bump.take(m * kk * 2), bump.take(kk * n * 2), bump.take(m * n * 2)
    _put(view, o_a, a_m, torch.bfloat16)
    _put(view, o_b, b_m, torch.bfloat16)
    torch.cuda.synchronize()

    R, W = KernelArg.read, KernelArg.write

    def step():
        la.attention_fwd(W(o_out, tb), R(o_q, tb), R(o_k, tb), R(o_v, tb), W(o_lse, B * H * S * 4), B, H, S, D,
                         True)
        la.attention_bwd(W(o_dq, tb), W(o_dk, tb), W(o_dv, tb), R(o_do, tb), R(o_q, tb), R(o_k, tb), R(o_v, tb),
                         R(o_lse, B * H * S * 4), B, H, S, D, True)
        la.matmul_fwd(W(o_c, m * n * 2), R(o_a, m * kk * 2), R(o_b, kk * n * 2), m, kk, n)

    # The first launch of a kernel in a process loads the library's module onto the device
    # (CUDA's lazy loading), which takes device memory once; the second pass is measured.
    step()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    step()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0  # the launches took their scratch from the launcher's workspace

    ro, rl = O.attention_fwd(q, k, v)
    rq, rk, rv = O.attention_bwd(do, q, k, v, rl)
    assert rel_err(_get(view, o_out, (B, H, S, D), torch.bfloat16), ro) <= BF16_TOL
    assert rel_err(_get(view, o_lse, (B, H, S), torch.float32), rl) <= 1e-3
    for off, r in ((o_dq, rq), (o_dk, rk), (o_dv, rv)):
        assert rel_err(_get(view, off, (B, H, S, D), torch.bfloat16), r) <= BF16_TOL
    assert rel_err(_get(view, o_c, (m, n), torch.bfloat16), O.matmul_fwd(a_m, b_m)) <= BF16_TOL
    la.close()


def test_arena_launch_without_workspace_fails_instead_of_allocating():
    """No workspace reserved: the attention backward answers OutOfMemory (requested /
    available) and nothing is allocated or launched."""
    import torch
    from beacon_b200.errors import LaunchError
    from beacon_b200.launcher import KernelArg
    B, H, S, D = 1, 2, 128, 64
    la, view = _setup(8 << 20, 0)
    tb = B * H * S * D * 2
    R, W = KernelArg.read, KernelArg.write
    n0 = __import__("beacon_b200.ops", fromlist=["launch_count"]).launch_count()
    with pytest.raises(LaunchError) as err:
        la.attention_bwd(W(0, tb), W(tb, tb), W(2 * tb, tb), R(3 * tb, tb), R(4 * tb, tb), R(5 * tb, tb),
                         R(6 * tb, tb), R(7 * tb, B * H * S * 4), B, H, S, D, True)
    assert "arena workspace" in str(err.value)
    from beacon_b200 import ops
    assert ops.launch_count() == n0
    torch.cuda.synchronize()
    la.close()
