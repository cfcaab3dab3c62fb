"""GEMM family parity (matmul.rs:18-78) through the C ABI against the CPU oracle."""
import numpy as np
import pytest

import oracle as O
from helpers import BF16_TOL, F32_TOL, as_bf16, rel_err, to_dev, to_np, uniform, normal

pytestmark = pytest.mark.gpu


def _ops():
    from beacon_b200 import ops
    return ops


@pytest.mark.parametrize("m,k,n", [
    (128, 64, 256),      # one tile
    (256, 512, 512),     # several K tiles, 2 N tiles
    (1024, 1024, 1024),
    (200, 136, 328),     # M / N / K tails on the TMA path
    (33, 47, 29),        # row strides not 16-byte multiples: exact SIMT path
    (1, 8, 8),
])
def test_matmul_fwd_bf16(m, k, n):
    import torch
    ops = _ops()
    a = as_bf16(uniform((m, k), 1))
    b = as_bf16(uniform((k, n), 1, offset=m * k))
    out = ops.matmul_fwd(to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16))
    ref = O.matmul_fwd(a, b)
    assert rel_err(to_np(out), ref) <= BF16_TOL


@pytest.mark.parametrize("m,k,n", [(128, 64, 96), (37, 51, 29)])
def test_matmul_fwd_f32(m, k, n):
    import torch
    ops = _ops()
    a = uniform((m, k), 3)
    b = uniform((k, n), 4)
    out = ops.matmul_fwd(to_dev(a, torch.float32), to_dev(b, torch.float32))
    assert rel_err(to_np(out), O.matmul_fwd(a, b)) <= F32_TOL


def test_matmul_4096_sampled_rows():
    """The 4096^3 workload: full GPU product, oracle on a sample of 64 rows."""
    import torch
    ops = _ops()
    m = k = n = 4096
    a = as_bf16(uniform((m, k), 1))
    b = as_bf16(uniform((k, n), 1, offset=m * k))
    out = to_np(ops.matmul_fwd(to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16)))
    rows = np.random.default_rng(0).choice(m, 64, replace=False)
    ref = O.matmul_fwd(np.ascontiguousarray(a[rows]), b)
    assert rel_err(out[rows], ref) <= BF16_TOL
    assert np.isfinite(out).all()


@pytest.mark.parametrize("m,k,n", [(256, 192, 320), (128, 64, 64), (72, 40, 24)])
def test_matmul_bwd_bf16(m, k, n):
    import torch
    ops = _ops()
    a = as_bf16(uniform((m, k), 5))
    b = as_bf16(uniform((k, n), 6))
    dy = as_bf16(uniform((m, n), 7))
    dl, dr = ops.matmul_bwd(to_dev(dy, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16))
    rl, rr = O.matmul_bwd(dy, a, b)
    assert rel_err(to_np(dl), rl) <= BF16_TOL
    assert rel_err(to_np(dr), rr) <= BF16_TOL


def test_matmul_bwd_f32():
    import torch
    ops = _ops()
    a, b, dy = uniform((64, 48), 8), uniform((48, 80), 9), uniform((64, 80), 10)
    dl, dr = ops.matmul_bwd(to_dev(dy, torch.float32), to_dev(a, torch.float32), to_dev(b, torch.float32))
    rl, rr = O.matmul_bwd(dy, a, b)
    assert rel_err(to_np(dl), rl) <= F32_TOL
    assert rel_err(to_np(dr), rr) <= F32_TOL


@pytest.mark.parametrize("dtype_name", ["bf16", "f32"])
def test_linear_fwd_bwd(dtype_name):
    import torch
    ops = _ops()
    dt = torch.bfloat16 if dtype_name == "bf16" else torch.float32
    tol = BF16_TOL if dtype_name == "bf16" else F32_TOL
    r = as_bf16 if dtype_name == "bf16" else (lambda x: x)
    m, k, n = 256, 128, 192
    x, w, bias, dy = r(normal((m, k), 11)), r(normal((k, n), 12, std=0.1)), r(normal((n,), 13)), r(normal((m, n), 14))
    out = ops.linear_fwd(to_dev(x, dt), to_dev(w, dt), to_dev(bias, dt))
    assert rel_err(to_np(out), O.linear_fwd(x, w, bias)) <= tol
    dx, dw, db = ops.linear_bwd(to_dev(dy, dt), to_dev(x, dt), to_dev(w, dt))
    rx, rw, rb = O.linear_bwd(dy, x, w)
    assert rel_err(to_np(dx), rx) <= tol
    assert rel_err(to_np(dw), rw) <= tol
    assert rel_err(to_np(db), rb) <= tol


def test_empty_reduction_gives_zeros():
    import torch
    ops = _ops()
    a = torch.empty(64, 0, dtype=torch.bfloat16, device="cuda")
    b = torch.empty(0, 64, dtype=torch.bfloat16, device="cuda")
    out = ops.matmul_fwd(a, b)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0


def test_no_device_fault_recorded():
    ops = _ops()
    code, site, count = ops.device_status(0)
    assert (code, count) == (0, 0)


# n % 16 == 0 with aligned rows: decoded inside the GEMM pipeline (k_gemm_fp8w_tc2);
# (72, 200, 200): n % 16 != 0, decoded to a bf16 copy first
@pytest.mark.parametrize("m,k,n,scale,with_bias", [(256, 512, 384, 1.0, False), (4096, 4096, 4096, 0.03125, True),
                                                   (100, 64, 48, 2.5, True), (300, 136, 336, 1.0, False),
                                                   (72, 200, 200, 0.5, True)])
def test_fp8_weight_gemm(m, k, n, scale, with_bias):
    """fp8 e4m3 weights (reference codec) dequantised in the GEMM path; bf16 activations."""
    import torch
    ops = _ops()
    a = as_bf16(normal((m, k), 21))
    w = normal((k, n), 22, std=20.0)
    w8 = O.to_fp8_bits(w)
    wdec = O.from_fp8_bits(w8)
    bias = as_bf16(normal((n,), 23)) if with_bias else None
    out = ops.matmul_fp8w_fwd(to_dev(a, torch.bfloat16), torch.from_numpy(w8).cuda(), scale,
                              None if bias is None else to_dev(bias, torch.bfloat16))
    if m > 1024:
        rows = np.random.default_rng(1).choice(m, 64, replace=False)
        ref = O.linear_fwd(np.ascontiguousarray(a[rows]), (wdec * scale).astype(np.float32), bias)
        got = to_np(out)[rows]
    else:
        ref = O.linear_fwd(a, (wdec * scale).astype(np.float32), bias)
        got = to_np(out)
    assert rel_err(got, ref) <= BF16_TOL


def test_fp8_dtype_through_matmul_fwd_entry():
    """dtype = Fp8E4M3 on the reference's matmul_fwd signature: rhs fp8, scale 1."""
    import ctypes
    import torch
    from beacon_b200 import _lib
    a = as_bf16(normal((128, 256), 24))
    w8 = O.to_fp8_bits(normal((256, 128), 25, std=4.0))
    A, W = to_dev(a, torch.bfloat16), torch.from_numpy(w8).cuda()
    out = torch.empty(128, 128, dtype=torch.bfloat16, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = _lib.lib().beacon_matmul_fwd(p(out), p(A), p(W), 128, 256, 128, _lib.FP8E4M3,
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _lib.last_error()
    assert rel_err(to_np(out), O.matmul_fwd(a, O.from_fp8_bits(w8))) <= BF16_TOL


def test_fp8_in_gemm_decode_of_every_code_is_exact():
    """All 256 e4m3 codes through the in-pipeline decoder: column j of the weight holds code
    j at row j % 64 and zeros elsewhere, the activations are the identity, so out[i, j] is
    exactly the decoded code at i == j % 64 (0 elsewhere), or NaN down the whole column of a
    NaN code.  Compared with the reference codec (crates/beacon-core/src/dtype.rs:138-161)."""
    import torch
    ops = _ops()
    k, n = 64, 256
    w8 = np.zeros((k, n), dtype=np.uint8)
    codes = np.arange(256, dtype=np.uint8)
    w8[np.arange(n) % k, np.arange(n)] = codes
    eye = np.eye(k, dtype=np.float32)
    out = to_np(ops.matmul_fp8w_fwd(to_dev(eye, torch.bfloat16), torch.from_numpy(w8).cuda(), 1.0))
    dec = O.from_fp8_bits(codes)
    ref = np.zeros((k, n), dtype=np.float32)
    ref[np.arange(n) % k, np.arange(n)] = dec
    ref[:, np.isnan(dec)] = np.nan
    assert np.array_equal(out, ref, equal_nan=True)


def test_fp8_quantizer_is_bit_exact_and_feeds_the_gemm():
    """fp32 master -> fp8 weights (amax, scale = amax / 448, encode of x * 448 / amax)
    against the oracle bit for bit, then the device-scale GEMM on those weights against the
    oracle and against the host-scale GEMM (same bits)."""
    import torch
    ops = _ops()
    k, n, m = 1024, 768, 256
    w = normal((k, n), 26, std=0.3)
    w[3, 5] = 7.25  # the tensor's maximum
    q, scale, amax = ops.quantize_fp8e4m3(torch.from_numpy(w).cuda())
    rq, rscale, ramax = O.quantize_fp8e4m3(w)
    assert np.array_equal(q.cpu().numpy(), rq)
    assert float(scale.item()) == float(rscale) and float(amax.item()) == float(ramax)
    a = as_bf16(normal((m, k), 27))
    ad = to_dev(a, torch.bfloat16)
    out = ops.linear_fp8w_fwd_devscale(ad, q, scale)
    ref = O.matmul_fwd(a, (O.from_fp8_bits(rq) * rscale).astype(np.float32))
    assert rel_err(to_np(out), ref) <= BF16_TOL
    assert rel_err(to_np(out), O.matmul_fwd(a, w)) <= 0.1  # the quantisation error itself stays small
    host = ops.matmul_fp8w_fwd(ad, q, float(scale.item()))
    assert torch.equal(out, host)
    # all zeros: scale 1, codes 0
    q0, s0, a0 = ops.quantize_fp8e4m3(torch.zeros(64, device="cuda"))
    assert not q0.any() and float(s0.item()) == 1.0 and float(a0.item()) == 0.0


def test_matmul_plan_reports_the_tile_shapes():
    """beacon_matmul_plan reports the shape the GEMM entries pick: 256x256 SM-pair tiles for
    4096^3, 256x128 pair tiles for the 8-way column shard 4096 x 512, 1-SM 128-row tiles when
    M = 128 would leave half of a pair's rows empty."""
    from beacon_b200 import ops
    big = ops.matmul_plan(4096, 4096, 4096)
    assert (big["tile_m"], big["tile_n"], big["sms_per_tile"], big["tiles"]) == (256, 256, 2, 256)
    shard = ops.matmul_plan(4096, 4096, 512)
    assert (shard["tile_m"], shard["tile_n"], shard["sms_per_tile"], shard["tiles"]) == (256, 128, 2, 64)
    small = ops.matmul_plan(128, 4096, 4096)
    assert small["tile_m"] == 128 and small["sms_per_tile"] == 1
    assert 0.0 < shard["wave_efficiency"] <= 1.0
