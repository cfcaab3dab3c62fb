"""RMSNorm (norm.rs:19-51), LayerNorm (norm.rs:55-95), SwiGLU MLP (mlp.rs:12-52), residual add and casts
(elementwise.rs) through the C ABI against the CPU oracle."""
import numpy as np
import pytest

import oracle as O
from helpers import BF16_TOL, F32_TOL, as_bf16, normal, rel_err, to_dev, to_np

pytestmark = pytest.mark.gpu


def _ops():
    from beacon_b200 import ops
    return ops


# bf16 rows that are whole multiples of 256 up to 4096 take the warp-per-row forward: one
# warp per row up to 2048 (17 x 256, 300 x 768, 1000 x 2048: more rows than the grid's row
# slots), two warps per row above (64 x 4096, 513 x 3072); 70 x 2304 (nine 256-column
# chunks, odd) and the rest take the CTA-per-row kernels.  The backward of bf16 rows of
# 256 x (1-4) x (1, 2 or 4 warps) columns runs one to four warps per row: 17 x 256, 40 x 512,
# 300 x 768 and 129 x 1024 one warp; 7 x 1536 and 1000 x 2048 two; 513 x 3072, 64 x 4096
# and 3 x 4096 (fewer rows than one CTA's row slots on the second CTA) four.
@pytest.mark.parametrize("T,dim,dt", [(64, 4096, "bf16"), (8, 14336, "bf16"), (33, 1000, "f32"), (16, 256, "f32"),
                                      (5, 100, "bf16"), (64, 4096, "f32"), (17, 256, "bf16"), (300, 768, "bf16"),
                                      (1000, 2048, "bf16"), (513, 3072, "bf16"), (70, 2304, "bf16"),
                                      (40, 512, "bf16"), (129, 1024, "bf16"), (7, 1536, "bf16"), (3, 4096, "bf16")])
def test_rmsnorm(T, dim, dt):
    import torch
    ops = _ops()
    tdt = torch.bfloat16 if dt == "bf16" else torch.float32
    tol = BF16_TOL if dt == "bf16" else F32_TOL
    r = as_bf16 if dt == "bf16" else (lambda a: a)
    x, g, dy = r(normal((T, dim), 3)), r(normal((dim,), 4)), r(normal((T, dim), 5))
    y, rms = ops.rmsnorm_fwd(to_dev(x, tdt), to_dev(g, tdt))
    ry, rr = O.rmsnorm_fwd(x, g)
    assert rel_err(to_np(y), ry) <= tol
    assert rel_err(to_np(rms), rr) <= 1e-5
    dx, dg = ops.rmsnorm_bwd(to_dev(dy, tdt), to_dev(x, tdt), rms, to_dev(g, tdt))
    rdx, rdg = O.rmsnorm_bwd(dy, x, rr, g)
    assert rel_err(to_np(dx), rdx) <= tol
    assert rel_err(to_np(dg), rdg) <= tol


# dweight not wanted (null): dx alone, on the warp-per-row backward (4096) and the row kernel
# (2304)
@pytest.mark.parametrize("T,dim", [(100, 4096), (70, 2304)])
def test_rmsnorm_bwd_dx_only(T, dim):
    import ctypes
    import torch
    from beacon_b200 import _lib
    from beacon_b200.errors import check
    ops = _ops()
    x, g, dy = (as_bf16(normal(s, 30 + i)) for i, s in enumerate([(T, dim), (dim,), (T, dim)]))
    t = lambda a: to_dev(a, torch.bfloat16)
    xt, gt, dyt = t(x), t(g), t(dy)
    _, rms = ops.rmsnorm_fwd(xt, gt)
    rdx, _ = O.rmsnorm_bwd(dy, x, to_np(rms), g)
    dx = torch.empty(T, dim, dtype=torch.bfloat16, device="cuda")
    p = lambda a: ctypes.c_void_p(a.data_ptr())
    check(_lib.lib().beacon_rmsnorm_adjoint_bwd(p(dx), None, p(dyt), p(xt), p(rms), p(gt), T, dim, _lib.BF16, None, 0,
                                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert rel_err(to_np(dx), rdx) <= BF16_TOL


# The forward of bf16 rows that are whole multiples of 256 up to 4096 (and not an odd count
# of chunks above 8) runs one or two warps per row: (2000, 768), (1000, 256), (64, 4096),
# (513, 3072); (70, 2304) and the rest take the CTA-per-row kernels.
# (2000, 768): more rows than CTAs, so each CTA's dweight / dbias partials cover several rows;
# widths up to 8192 (bf16) / 4096 (f32) take the register-resident backward, (8, 14336) the
# one with partials in global memory; (5, 100) and (7, 20) reach the any-dim forward and the
# scalar backward loop; 40 x 512, 129 x 1024, 7 x 1536, 300 x 2048 and 3 x 4096 (fewer rows
# than CTAs) cover the register-resident backward's one- and two-vector widths.
@pytest.mark.parametrize("T,dim,dt", [(64, 4096, "bf16"), (8, 14336, "bf16"), (2000, 768, "bf16"), (40, 6144, "bf16"),
                                      (33, 1000, "f32"), (16, 256, "f32"), (5, 100, "bf16"), (7, 20, "f32"),
                                      (64, 4096, "f32"), (513, 3072, "bf16"), (70, 2304, "bf16"), (1000, 256, "bf16"),
                                      (40, 512, "bf16"), (129, 1024, "bf16"), (7, 1536, "bf16"), (300, 2048, "bf16"),
                                      (3, 4096, "bf16")])
def test_layernorm(T, dim, dt):
    import torch
    ops = _ops()
    tdt = torch.bfloat16 if dt == "bf16" else torch.float32
    tol = BF16_TOL if dt == "bf16" else F32_TOL
    r = as_bf16 if dt == "bf16" else (lambda a: a)
    x, g, b, dy = r(normal((T, dim), 6)), r(normal((dim,), 7)), r(normal((dim,), 8)), r(normal((T, dim), 9))
    y, mu, inv = ops.layernorm_fwd(to_dev(x, tdt), to_dev(g, tdt), to_dev(b, tdt))
    ry, rmu, rinv = O.layernorm_fwd(x, g, b)
    assert rel_err(to_np(y), ry) <= tol
    assert rel_err(to_np(mu), rmu) <= 1e-5 and rel_err(to_np(inv), rinv) <= 1e-5
    dx, dg, db = ops.layernorm_bwd(to_dev(dy, tdt), to_dev(x, tdt), mu, inv, to_dev(g, tdt))
    rdx, rdg, rdb = O.layernorm_bwd(dy, x, rmu, rinv, g)
    assert rel_err(to_np(dx), rdx) <= tol
    assert rel_err(to_np(dg), rdg) <= tol
    assert rel_err(to_np(db), rdb) <= tol


@pytest.mark.parametrize("skip", ["dweight", "dbias", "both"])
def test_layernorm_bwd_one_parameter_gradient(skip):
    """dweight or dbias alone (the other NULL): the column-sum kernel writes only the one asked
    for; both NULL: dx alone."""
    import ctypes
    import torch
    from beacon_b200 import _lib
    from beacon_b200.errors import check
    ops = _ops()
    T, dim = 300, 2048
    x, g, b, dy = (as_bf16(normal(s, 20 + i)) for i, s in enumerate([(T, dim), (dim,), (dim,), (T, dim)]))
    t = lambda a: to_dev(a, torch.bfloat16)
    _, mu, inv = ops.layernorm_fwd(t(x), t(g), t(b))
    rdx, rdg, rdb = O.layernorm_bwd(dy, x, to_np(mu), to_np(inv), g)
    dx = torch.empty(T, dim, dtype=torch.bfloat16, device="cuda")
    dw = torch.full((dim,), float("nan"), dtype=torch.bfloat16, device="cuda")
    db = torch.full((dim,), float("nan"), dtype=torch.bfloat16, device="cuda")
    p = lambda a: None if a is None else ctypes.c_void_p(a.data_ptr())
    dyt, xt, gt = t(dy), t(x), t(g)
    check(_lib.lib().beacon_layernorm_adjoint_bwd(p(dx), None if skip in ("dweight", "both") else p(dw),
                                                  None if skip in ("dbias", "both") else p(db), p(dyt), p(xt), p(mu),
                                                  p(inv), p(gt), T, dim, _lib.BF16, None, 0,
                                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert rel_err(to_np(dx), rdx) <= BF16_TOL
    if skip == "both":
        assert torch.isnan(dw.float()).all() and torch.isnan(db.float()).all()
    elif skip == "dweight":
        assert torch.isnan(dw.float()).all() and rel_err(to_np(db), rdb) <= BF16_TOL
    else:
        assert torch.isnan(db.float()).all() and rel_err(to_np(dw), rdg) <= BF16_TOL


def test_layernorm_edges():
    import torch
    ops = _ops()
    dev = "cuda"
    # constant rows: zero variance, so out = bias up to float32 rounding
    x = torch.full((4, 512), 2.5, dtype=torch.float32, device=dev)
    g = torch.randn(512, device=dev)
    b = torch.randn(512, device=dev)
    y, mu, inv = ops.layernorm_fwd(x, g, b)
    assert torch.allclose(y, b.expand_as(y), atol=1e-6)
    assert torch.allclose(mu, torch.full_like(mu, 2.5))
    # no rows: the parameter gradients are empty sums
    x0 = torch.empty((0, 64), dtype=torch.bfloat16, device=dev)
    g0 = torch.ones(64, dtype=torch.bfloat16, device=dev)
    y0, mu0, inv0 = ops.layernorm_fwd(x0, g0, g0)
    assert y0.shape == (0, 64)
    dx0, dg0, db0 = ops.layernorm_bwd(x0, x0, mu0, inv0, g0)
    torch.cuda.synchronize()
    assert dx0.shape == (0, 64) and not dg0.float().any() and not db0.float().any()


# bf16 backward: F % 64 == 0 takes the fused five-GEMM path (K = 2F dx GEMM, N = 2F weight
# gradient GEMM); (64, 64, 96) the N-split but two dx GEMMs; (100, 128, 200) two GEMMs for each
@pytest.mark.parametrize("T,dm,F,dt", [(128, 256, 512, "bf16"), (200, 128, 320, "bf16"), (64, 64, 96, "f32"),
                                      (64, 64, 96, "bf16"), (100, 128, 200, "bf16")])
def test_swiglu(T, dm, F, dt):
    import torch
    ops = _ops()
    tdt = torch.bfloat16 if dt == "bf16" else torch.float32
    tol = BF16_TOL if dt == "bf16" else F32_TOL
    r = as_bf16 if dt == "bf16" else (lambda a: a)
    x = r(normal((T, dm), 3))
    wg, wu = r(normal((dm, F), 31, std=0.05)), r(normal((dm, F), 32, std=0.05))
    wd, dy = r(normal((F, dm), 33, std=0.05)), r(normal((T, dm), 34))
    dev = lambda a: to_dev(a, tdt)
    out = ops.swiglu_fwd(dev(x), dev(wg), dev(wu), dev(wd))
    assert rel_err(to_np(out), O.swiglu_fwd(x, wg, wu, wd)) <= tol
    grads = ops.swiglu_bwd(dev(dy), dev(x), dev(wg), dev(wu), dev(wd))
    refs = O.swiglu_bwd(dy, x, wg, wu, wd)
    for g, rf in zip(grads, refs):
        assert rel_err(to_np(g), rf) <= tol


def test_residual_add_bitexact():
    import torch
    ops = _ops()
    a, b = normal((1000003,), 1), normal((1000003,), 2)
    out = ops.residual_add(to_dev(a, torch.float32), to_dev(b, torch.float32))
    assert np.array_equal(to_np(out), a + b)
    da, db = ops.residual_add_bwd(to_dev(a, torch.float32))
    assert np.array_equal(to_np(da), a) and np.array_equal(to_np(db), a)
    ab, bb = as_bf16(a), as_bf16(b)
    outb = ops.residual_add(to_dev(ab, torch.bfloat16), to_dev(bb, torch.bfloat16))
    assert np.array_equal(to_np(outb), O.round_bf16(ab + bb))


def test_casts_bitexact():
    import torch
    ops = _ops()
    x = np.concatenate([normal((200000,), 9, std=50.0), normal((50000,), 10, std=0.01),
                        np.array([0.0, -0.0, 448.0, 464.0, -1e9, 1e9, np.nan, np.inf, -np.inf, 2.0 ** -9,
                                  2.0 ** -10, 3 * 2.0 ** -11, 1.0 + 2.0 ** -4, 255.99998], np.float32)]).astype(np.float32)
    f8 = ops.cast(to_dev(x, torch.float32), ops.CAST_F32_TO_FP8E4M3)
    assert np.array_equal(f8.cpu().numpy(), O.to_fp8_bits(x))
    back = ops.cast(f8, ops.CAST_FP8E4M3_TO_F32).cpu().numpy()
    ref_back = O.from_fp8_bits(O.to_fp8_bits(x))
    assert np.array_equal(np.isnan(back), np.isnan(ref_back))
    assert np.array_equal(back[~np.isnan(back)], ref_back[~np.isnan(ref_back)])
    b16 = ops.cast(to_dev(x, torch.float32), ops.CAST_F32_TO_BF16)
    assert np.array_equal(b16.view(torch.int16).cpu().numpy().view(np.uint16), O.to_bf16_bits(x))
    f32 = ops.cast(b16, ops.CAST_BF16_TO_F32).cpu().numpy()
    assert np.array_equal(f32.view(np.uint32), O.from_bf16_bits(O.to_bf16_bits(x)).view(np.uint32))


def test_no_device_fault_recorded():
    ops = _ops()
    code, site, count = ops.device_status(0)
    assert (code, count) == (0, 0)


@pytest.mark.parametrize("m,k,n,dt,bias", [(256, 512, 384, "bf16", False), (200, 136, 328, "bf16", True),
                                           (4096, 4096, 1024, "bf16", False), (64, 96, 48, "f32", True),
                                           (33, 40, 24, "bf16", True)])
def test_rmsnorm_folded_into_linear(m, k, n, dt, bias):
    """rmsnorm_fwd then linear_fwd (norm.rs:20-31, matmul.rs:46-58) as one statistics pass
    and one GEMM on raw x with the gain folded into W and 1/rms applied in the epilogue."""
    import torch
    ops = _ops()
    tdt = torch.bfloat16 if dt == "bf16" else torch.float32
    tol = BF16_TOL if dt == "bf16" else F32_TOL
    r = as_bf16 if dt == "bf16" else (lambda a: a)
    x, g = r(normal((m, k), 61)), r(1.0 + 0.1 * normal((k,), 62))
    w, b = r(normal((k, n), 63, std=0.05)), (r(normal((n,), 64)) if bias else None)
    dev = lambda a: None if a is None else to_dev(a, tdt)
    wf = ops.rmsnorm_fold_weight(dev(g), dev(w))
    assert rel_err(to_np(wf), r(g[:, None] * w)) <= (F32_TOL if dt == "f32" else 0.0)
    out, rms = ops.rmsnorm_linear_fwd(dev(x), wf, dev(b))
    y, rr = O.rmsnorm_fwd(x, g)
    ref = O.linear_fwd(r(y), w, b)
    assert rel_err(to_np(rms), rr) <= 1e-5
    assert rel_err(to_np(out), ref) <= tol
