"""beacon_rmsnorm_adjoint_bwd_noalloc: the RMSNorm backward for callers that cannot
allocate device memory (arena-only launchers, paths that cannot take a first-call
cudaMalloc).  It keeps its dweight partial sums in a fixed array inside the library
instead of a workspace, and must give the same dx and dweight as the allocating
entry point.  This file is named to be collected last, and passes both alone in a
fresh process and after the other GPU tests."""
import ctypes

import pytest

from helpers import BF16_TOL, F32_TOL, as_bf16, normal, rel_err, to_dev, to_np

pytestmark = pytest.mark.gpu


def _call(name, dt_code, dx, dw, dy, x, rms, w, T, dim):
    import torch
    from beacon_b200 import _lib
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    L = _lib.lib()
    if name == "noalloc":
        return L.beacon_rmsnorm_adjoint_bwd_noalloc(p(dx), p(dw), p(dy), p(x), p(rms), p(w), T, dim, dt_code, stream)
    return L.beacon_rmsnorm_adjoint_bwd(p(dx), p(dw), p(dy), p(x), p(rms), p(w), T, dim, dt_code, None, 0, stream)


@pytest.mark.parametrize("T,dim,dt", [(4096, 4096, "bf16"), (333, 1000, "f32")])
def test_noalloc_matches_allocating_entry_point_twice(T, dim, dt):
    import torch
    from beacon_b200 import _lib, ops
    tdt, code, tol = ((torch.bfloat16, _lib.BF16, BF16_TOL) if dt == "bf16" else (torch.float32, _lib.F32, F32_TOL))
    r = as_bf16 if dt == "bf16" else (lambda a: a)
    x, g = to_dev(r(normal((T, dim), 41)), tdt), to_dev(r(normal((dim,), 42)), tdt)
    _, rms = ops.rmsnorm_fwd(x, g)
    for call in range(2):  # two calls in a row: the shared array must not carry state over
        dy = to_dev(r(normal((T, dim), 43 + call)), tdt)
        dx_ref, dw_ref = torch.empty_like(x), torch.empty_like(g)
        dx_na, dw_na = torch.full_like(x, float("nan")), torch.full_like(g, float("nan"))
        assert _call("ref", code, dx_ref, dw_ref, dy, x, rms, g, T, dim) == 0, _lib.last_error()
        assert _call("noalloc", code, dx_na, dw_na, dy, x, rms, g, T, dim) == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert rel_err(to_np(dx_na), to_np(dx_ref)) <= tol
        assert rel_err(to_np(dw_na), to_np(dw_ref)) <= tol
    assert ops.device_status(0)[0] == 0


def test_noalloc_rejects_dim_beyond_its_fixed_scratch():
    import torch
    from beacon_b200 import _lib
    x = torch.empty(2, 8, dtype=torch.float32, device="cuda")
    rc = _lib.lib().beacon_rmsnorm_adjoint_bwd_noalloc(None, None, None, None, None, None, 2, (1 << 20) + 1,
                                                       _lib.F32, None)
    assert rc == _lib.ERR_INVALID_LAUNCH_CONFIG
    assert "exceeds the fixed scratch" in _lib.last_error()
    del x
