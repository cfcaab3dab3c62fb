"""Causal attention parity (attention.rs:21-64) through the C ABI against the CPU oracle."""
import numpy as np
import pytest

import oracle as O
from helpers import BF16_TOL, F32_TOL, as_bf16, normal, rel_err, to_dev, to_np

pytestmark = pytest.mark.gpu


def _ops():
    from beacon_b200 import ops
    return ops


def _qkv(B, Hq, Hkv, S, D, seed, bf16=True):
    r = as_bf16 if bf16 else (lambda x: x)
    nq, nk = B * Hq * S * D, B * Hkv * S * D
    q = r(normal((B, Hq, S, D), seed))
    k = r(normal((B, Hkv, S, D), seed, offset=nq))
    v = r(normal((B, Hkv, S, D), seed, offset=nq + nk))
    do = r(normal((B, Hq, S, D), seed, offset=nq + 2 * nk))
    return q, k, v, do


def test_config1_f32_forward():
    """f32 causal SDPA B=1 H=4 S=128 D=64, seed 0, at 1e-5."""
    import torch
    ops = _ops()
    q, k, v, _ = _qkv(1, 4, 4, 128, 64, 0, bf16=False)
    out, lse = ops.attention_fwd(to_dev(q, torch.float32), to_dev(k, torch.float32), to_dev(v, torch.float32))
    ro, rl = O.attention_fwd(q, k, v)
    assert rel_err(to_np(out), ro) <= F32_TOL
    assert rel_err(to_np(lse), rl) <= F32_TOL


@pytest.mark.parametrize("B,H,S,D,causal", [
    (1, 4, 128, 64, True),
    (2, 4, 256, 128, True),
    (1, 2, 384, 128, True),
    (1, 2, 200, 128, True),   # S tail: keys >= S masked, rows >= S not stored
    (1, 2, 256, 128, False),
    (1, 1, 1, 64, True),
    (1, 2, 130, 64, False),
])
def test_forward_bf16(B, H, S, D, causal):
    import torch
    ops = _ops()
    q, k, v, _ = _qkv(B, H, H, S, D, 2)
    out, lse = ops.attention_fwd(to_dev(q, torch.bfloat16), to_dev(k, torch.bfloat16), to_dev(v, torch.bfloat16),
                                 causal=causal)
    ro, rl = O.attention_fwd(q, k, v, causal=causal)
    assert rel_err(to_np(out), ro) <= BF16_TOL
    assert rel_err(to_np(lse), rl) <= 1e-3


def test_forward_gqa_bf16():
    import torch
    ops = _ops()
    q, k, v, _ = _qkv(1, 8, 2, 256, 128, 4)
    out, lse = ops.attention_fwd(to_dev(q, torch.bfloat16), to_dev(k, torch.bfloat16), to_dev(v, torch.bfloat16))
    ro, rl = O.attention_fwd(q, k, v)
    assert rel_err(to_np(out), ro) <= BF16_TOL
    assert rel_err(to_np(lse), rl) <= 1e-3


def test_forward_config3_sampled_heads():
    """B=8 H=32 S=4096 D=128 (the fwd+bwd benchmark shape): oracle on 2 sampled heads."""
    import torch
    ops = _ops()
    B, H, S, D = 8, 32, 4096, 128
    q, k, v, _ = _qkv(B, H, H, S, D, 2)
    out, lse = ops.attention_fwd(to_dev(q, torch.bfloat16), to_dev(k, torch.bfloat16), to_dev(v, torch.bfloat16))
    heads = [0, 8 * 32 - 1]
    ro, rl = O.attention_fwd_heads(q, k, v, heads)
    out_np, lse_np = to_np(out).reshape(B * H, S, D), to_np(lse).reshape(B * H, S)
    for hh in heads:
        assert rel_err(out_np[hh], ro.reshape(B * H, S, D)[hh]) <= BF16_TOL
        assert rel_err(lse_np[hh], rl.reshape(B * H, S)[hh]) <= 1e-3
    assert np.isfinite(out_np).all()


@pytest.mark.parametrize("B,H,Hkv,S,D", [(1, 2, 2, 256, 64), (1, 2, 2, 256, 128), (1, 4, 2, 200, 128)])
def test_backward_bf16(B, H, Hkv, S, D):
    import torch
    ops = _ops()
    q, k, v, do = _qkv(B, H, Hkv, S, D, 5)
    _, rl = O.attention_fwd(q, k, v)
    dq, dk, dv = ops.attention_bwd(to_dev(do, torch.bfloat16), to_dev(q, torch.bfloat16), to_dev(k, torch.bfloat16),
                                   to_dev(v, torch.bfloat16), to_dev(rl, torch.float32))
    rq, rk, rv = O.attention_bwd(do, q, k, v, rl)
    assert rel_err(to_np(dq), rq) <= BF16_TOL
    assert rel_err(to_np(dk), rk) <= BF16_TOL
    assert rel_err(to_np(dv), rv) <= BF16_TOL


@pytest.mark.parametrize("B,H,Hkv,S,causal", [(1, 2, 2, 640, True), (2, 4, 1, 130, True), (1, 2, 2, 384, False),
                                               (1, 2, 2, 136, False)])
def test_backward_tile_edges_bf16(B, H, Hkv, S, causal):
    """An odd number of key tiles, S a tile plus a few rows, a single KV head for four query
    heads, non-causal attention with a ragged last tile."""
    import torch
    ops = _ops()
    q, k, v, do = _qkv(B, H, Hkv, S, 128, 11)
    t = lambda a: to_dev(a, torch.bfloat16)
    _, rl = O.attention_fwd(q, k, v, causal=causal)
    g = ops.attention_bwd(t(do), t(q), t(k), t(v), to_dev(rl, torch.float32), causal=causal)
    refs = O.attention_bwd(do, q, k, v, rl, causal=causal)
    for a, r in zip(g, refs):
        assert rel_err(to_np(a), r) <= BF16_TOL


def test_backward_f32():
    import torch
    ops = _ops()
    q, k, v, do = _qkv(1, 4, 4, 128, 64, 0, bf16=False)
    _, rl = O.attention_fwd(q, k, v)
    t = lambda a: to_dev(a, torch.float32)
    dq, dk, dv = ops.attention_bwd(t(do), t(q), t(k), t(v), t(rl))
    rq, rk, rv = O.attention_bwd(do, q, k, v, rl)
    assert rel_err(to_np(dq), rq) <= F32_TOL
    assert rel_err(to_np(dk), rk) <= F32_TOL
    assert rel_err(to_np(dv), rv) <= F32_TOL


def test_no_device_fault_recorded():
    ops = _ops()
    code, site, count = ops.device_status(0)
    assert (code, count) == (0, 0)


def test_backward_with_out_matches_drop_in():
    """beacon_attention_bwd_with_out (O given) and the drop-in backward (O recomputed in
    tensor memory) agree.  They differ only in rowsum(dO * O): from the bf16 output in one,
    from the fp32 accumulator in the other."""
    import torch
    ops = _ops()
    q, k, v, do = _qkv(1, 4, 4, 384, 128, 6)
    t = lambda a: to_dev(a, torch.bfloat16)
    out, lse = ops.attention_fwd(t(q), t(k), t(v))
    g1 = ops.attention_bwd(t(do), t(q), t(k), t(v), lse)
    g2 = ops.attention_bwd(t(do), t(q), t(k), t(v), lse, out=out)
    for a, b in zip(g1, g2):  # about one bf16 rounding step apart
        assert rel_err(to_np(a), to_np(b)) <= 1e-2
    _, rl = O.attention_fwd(q, k, v)
    refs = O.attention_bwd(do, q, k, v, rl)
    for g in (g1, g2):
        for a, r in zip(g, refs):
            assert rel_err(to_np(a), r) <= BF16_TOL


@pytest.mark.parametrize("causal", [True, False])
def test_backward_long_sampled_head(causal):
    """S=2048 backward (16 query tiles per key tile) against the oracle on one head."""
    import torch
    ops = _ops()
    q, k, v, do = _qkv(1, 2, 2, 2048, 128, 7)
    t = lambda a: to_dev(a, torch.bfloat16)
    _, lse = ops.attention_fwd(t(q), t(k), t(v), causal=causal)
    dq, dk, dv = ops.attention_bwd(t(do), t(q), t(k), t(v), lse, causal=causal)
    sl = slice(1, 2)
    qs, ks, vs, dos = (np.ascontiguousarray(a[:, sl]) for a in (q, k, v, do))
    _, rl = O.attention_fwd(qs, ks, vs, causal=causal)
    rq, rk, rv = O.attention_bwd(dos, qs, ks, vs, rl, causal=causal)
    assert rel_err(to_np(dq)[:, sl], rq) <= BF16_TOL
    assert rel_err(to_np(dk)[:, sl], rk) <= BF16_TOL
    assert rel_err(to_np(dv)[:, sl], rv) <= BF16_TOL


def test_backward_gqa_group4_bf16():
    import torch
    ops = _ops()
    q, k, v, do = _qkv(2, 8, 2, 256, 64, 8)
    t = lambda a: to_dev(a, torch.bfloat16)
    _, rl = O.attention_fwd(q, k, v)
    g = ops.attention_bwd(t(do), t(q), t(k), t(v), to_dev(rl, torch.float32))
    refs = O.attention_bwd(do, q, k, v, rl)
    for a, r in zip(g, refs):
        assert rel_err(to_np(a), r) <= BF16_TOL


def test_outputs_only_16_byte_aligned():
    """Outputs that are 16- but not 32-byte aligned (views 8 bf16 into a buffer) take the
    16-byte store path and give the same bits as aligned outputs."""
    import torch
    from beacon_b200 import _lib
    from beacon_b200.errors import check
    ops = _ops()
    B, H, S, D = 1, 2, 256, 128
    q, k, v, do = _qkv(B, H, H, S, D, 9)
    t = lambda a: to_dev(a, torch.bfloat16)
    q, k, v, do = t(q), t(k), t(v), t(do)
    n = B * H * S * D

    def view16(like):
        buf = torch.empty(n + 16, dtype=torch.bfloat16, device=like.device)
        out = buf[8:8 + n].view_as(like)
        assert out.data_ptr() % 32 == 16
        return out

    ref_out, lse = ops.attention_fwd(q, k, v)
    out = view16(q)
    ops.attention_fwd(q, k, v, out=out)
    assert torch.equal(out, ref_out)

    rq, rk, rv = ops.attention_bwd(do, q, k, v, lse)
    dq, dk, dv = view16(q), view16(k), view16(v)
    L = _lib.lib()
    rc = L.beacon_attention_adjoint_bwd(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), do.data_ptr(), q.data_ptr(),
                                        k.data_ptr(), v.data_ptr(), lse.data_ptr(), B, H, S, D, 1, _lib.BF16, None, 0,
                                        torch.cuda.current_stream().cuda_stream)
    check(rc)
    torch.cuda.synchronize()
    assert torch.equal(dq, rq) and torch.equal(dk, rk) and torch.equal(dv, rv)


def test_work_counter_slots_rotate_and_reset():
    """The persistent forward and dQ kernels draw their work items from per-launch counter
    slots in device memory (64 per device, reset by each launch's last CTA).  150 forward +
    backward calls in a row wrap the slots twice, and two streams running at once take
    different slots: every call must give the same outputs as the first."""
    import torch
    ops = _ops()
    B, H, S, D = 1, 3, 640, 128  # 3 heads x 3 query-tile pairs: fewer items than SMs, and more
    q, k, v, do = _qkv(B, H, H, S, D, 12)
    t = lambda a: to_dev(a, torch.bfloat16)
    q, k, v, do = t(q), t(k), t(v), t(do)
    out0, lse0 = ops.attention_fwd(q, k, v)
    dq0, dk0, dv0 = ops.attention_bwd(do, q, k, v, lse0)
    for _ in range(150):
        out, lse = ops.attention_fwd(q, k, v)
    dq, dk, dv = ops.attention_bwd(do, q, k, v, lse)
    torch.cuda.synchronize()
    assert torch.equal(out, out0) and torch.equal(lse, lse0)
    assert torch.equal(dq, dq0) and torch.equal(dk, dk0) and torch.equal(dv, dv0)
    # two streams at once, a larger problem on each (more items than SMs)
    q2, k2, v2, do2 = (t(a) for a in _qkv(2, 16, 16, 1024, 128, 13))
    ref2 = ops.attention_fwd(q2, k2, v2)
    refg = ops.attention_bwd(do2, q2, k2, v2, ref2[1])
    torch.cuda.synchronize()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    ws_bytes = ops.attention_bwd_workspace_bytes(2, 16, 1024, 128)
    wss = [torch.empty(ws_bytes, dtype=torch.uint8, device="cuda") for _ in range(2)]  # one per stream
    res = []
    for s, ws in zip((s1, s2), wss):
        with torch.cuda.stream(s):
            o, l = ops.attention_fwd(q2, k2, v2)
            res.append((o, l, ops.attention_bwd(do2, q2, k2, v2, l, workspace=ws)))
    torch.cuda.synchronize()
    for o, l, g in res:
        assert torch.equal(o, ref2[0]) and torch.equal(l, ref2[1])
        for a, b in zip(g, refg):
            assert torch.equal(a, b)
    assert ops.device_status(0)[0] == 0


@pytest.mark.parametrize("B,H,Hkv,S,D,causal", [
    (2, 96, 96, 256, 128, True),    # 192 heads: more items than SMs in all three kernels, 1-2 tiles each
    (2, 96, 48, 384, 64, True),     # GQA groups of 2 at head_dim 64, ragged causal items
    (1, 160, 160, 200, 128, False),  # one tile per item, a tail inside it
])
def test_persistent_kernels_many_short_items(B, H, Hkv, S, D, causal):
    """The persistent forward, dK/dV and dQ kernels with more (and much shorter) work items
    than SMs: the item rings wrap many times and consecutive items overlap.  Every head is
    checked against the oracle."""
    import torch
    ops = _ops()
    q, k, v, do = _qkv(B, H, Hkv, S, D, 14)
    t = lambda a: to_dev(a, torch.bfloat16)
    out, lse = ops.attention_fwd(t(q), t(k), t(v), causal=causal)
    dq, dk, dv = ops.attention_bwd(t(do), t(q), t(k), t(v), lse, causal=causal)
    ro, rl = O.attention_fwd(q, k, v, causal=causal)
    assert rel_err(to_np(out), ro) <= BF16_TOL
    assert rel_err(to_np(lse), rl) <= 1e-3
    for a, r in zip((dq, dk, dv), O.attention_bwd(do, q, k, v, rl, causal=causal)):
        assert rel_err(to_np(a), r) <= BF16_TOL
    assert ops.device_status(0)[0] == 0
