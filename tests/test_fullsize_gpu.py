"""Parity at the benchmarked sizes, through the drop-in C entry points.

The benchmark's workloads run on the GPU at full size; the oracle checks them on
sampled units (whole heads, or query rows of a head, or rows of one sequence):
  - causal attention forward + backward, B=8 H=32 S=4096 D=128 (the fwd+bwd headline),
    attention_adjoint_fwd then attention_adjoint_bwd (attention.rs:21-64), three heads;
  - long grouped-query causal forward, 64 query / 8 KV heads, S=32768 (query heads of
    two KV groups, rows that see all 256 key tiles among them);
  - the pre-norm block forward at batch 4 x seq 2048, d_model 4096, 32 x 128 heads,
    SwiGLU hidden 14336 (rows of one sequence).
"""
import numpy as np
import pytest

import oracle as O
from helpers import BF16_TOL, as_bf16, normal, rel_err, to_dev, to_np

pytestmark = pytest.mark.gpu


def _qkv(B, Hq, Hkv, S, D, seed, with_do=True):
    nq, nk = B * Hq * S * D, B * Hkv * S * D
    q = as_bf16(normal((B, Hq, S, D), seed))
    k = as_bf16(normal((B, Hkv, S, D), seed, offset=nq))
    v = as_bf16(normal((B, Hkv, S, D), seed, offset=nq + nk))
    do = as_bf16(normal((B, Hq, S, D), seed, offset=nq + 2 * nk)) if with_do else None
    return q, k, v, do


def test_attention_fwd_bwd_benchmark_shape_sampled_heads():
    """B=8 H=32 S=4096 D=128, seed 2: the drop-in forward then the drop-in backward (which
    recomputes O) on all 256 heads; out, lse, dq, dk, dv of heads 0, 97 and 255 against
    the oracle (whole heads: every query and key row)."""
    import torch
    from beacon_b200 import ops
    B, H, S, D = 8, 32, 4096, 128
    q, k, v, do = _qkv(B, H, H, S, D, 2)
    t = lambda a: to_dev(a, torch.bfloat16)
    qd, kd, vd, dod = t(q), t(k), t(v), t(do)
    out, lse = ops.attention_fwd(qd, kd, vd)
    dq, dk, dv = ops.attention_bwd(dod, qd, kd, vd, lse)
    torch.cuda.synchronize()
    flat = lambda a: a.reshape(B * H, S, D)
    for hh in (0, 97, B * H - 1):
        qh, kh, vh, doh = (np.ascontiguousarray(flat(a)[hh]) for a in (q, k, v, do))
        ro, rl = O.attention_fwd_rows(qh, kh, vh, np.arange(S))
        rq, rk, rv = O.attention_bwd_head(doh, qh, kh, vh, rl)
        assert rel_err(to_np(out.reshape(B * H, S, D)[hh]), ro) <= BF16_TOL, hh
        assert rel_err(to_np(lse.reshape(B * H, S)[hh]), rl) <= 1e-3, hh
        assert rel_err(to_np(dq.reshape(B * H, S, D)[hh]), rq) <= BF16_TOL, hh
        assert rel_err(to_np(dk.reshape(B * H, S, D)[hh]), rk) <= BF16_TOL, hh
        assert rel_err(to_np(dv.reshape(B * H, S, D)[hh]), rv) <= BF16_TOL, hh
    for g in (dq, dk, dv):
        assert bool(torch.isfinite(g.float()).all())
    assert ops.device_status(0)[0] == 0


def test_gqa_long_context_forward_sampled_rows():
    """B=1, 64 query heads, 8 KV heads, S=32768, D=128, seed 4: query heads 0 (KV group 0)
    and 63 (KV group 7); the last 256 query rows (each sees all 256 key tiles), 256 rows
    spread over the sequence and the first 8."""
    import torch
    from beacon_b200 import ops
    B, Hq, Hkv, S, D = 1, 64, 8, 32768, 128
    q, k, v, _ = _qkv(B, Hq, Hkv, S, D, 4, with_do=False)
    t = lambda a: to_dev(a, torch.bfloat16)
    out, lse = ops.attention_fwd(t(q), t(k), t(v))
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.arange(8), np.linspace(8, S - 257, 256).astype(np.int64),
                                     np.arange(S - 256, S)]))
    for h in (0, Hq - 1):
        g = h // (Hq // Hkv)
        ro, rl = O.attention_fwd_rows(q[0, h], np.ascontiguousarray(k[0, g]), np.ascontiguousarray(v[0, g]), rows)
        assert rel_err(to_np(out[0, h])[rows], ro) <= BF16_TOL, h
        assert rel_err(to_np(lse[0, h])[rows], rl) <= 1e-3, h
    assert bool(torch.isfinite(out.float()).all())
    assert ops.device_status(0)[0] == 0


def test_llama_block_benchmark_shape_sampled_rows():
    """Batch 4 x seq 2048, d_model 4096, 32 x 128 heads, SwiGLU 14336; weights N(0, 0.02)
    and x N(0, 1) from seed 3, norm gains 1.  Rows of sequence 2 (a batch offset that is
    not 0) against the sampled-row block oracle."""
    import torch
    from beacon_b200 import ops
    Bt, S, dm, H, D, F = 4, 2048, 4096, 32, 128, 14336
    T = Bt * S
    shapes = dict(w_qkv=(dm, 3 * H * D), w_o=(H * D, dm), w_gate=(dm, F), w_up=(dm, F), w_down=(F, dm))
    w, off = {}, 0
    for name, shp in shapes.items():
        w[name] = as_bf16(normal(shp, 3, std=0.02, offset=off))
        off += int(np.prod(shp))
    x = as_bf16(normal((T, dm), 3, offset=off))
    ones = np.ones(dm, dtype=np.float32)
    dev = {k_: to_dev(a, torch.bfloat16) for k_, a in w.items()}
    n1 = to_dev(ones, torch.bfloat16)
    out = ops.llama_block_fwd(to_dev(x, torch.bfloat16), n1, dev["w_qkv"], dev["w_o"], n1, dev["w_gate"],
                              dev["w_up"], dev["w_down"], Bt, S, H, H)
    torch.cuda.synchronize()
    got = to_np(out)
    assert np.isfinite(got).all()
    seq = 2
    rows = np.unique(np.concatenate([[0, 1, 127, 128, 1000, S - 1],
                                     np.random.default_rng(0).choice(S, 26, replace=False)]))
    xs = np.ascontiguousarray(x[seq * S:(seq + 1) * S])
    ref = O.llama_block_fwd_rows(xs, ones, w["w_qkv"], w["w_o"], ones, w["w_gate"], w["w_up"], w["w_down"], H, H,
                                 rows)
    g = got[seq * S + rows]
    assert rel_err(g, ref) <= BF16_TOL
    assert rel_err(g - xs[rows], ref - xs[rows]) <= BF16_TOL
    # the same block with both norms folded into the GEMMs after them
    wq, wg, wu = ops.llama_block_fold_weights(n1, dev["w_qkv"], n1, dev["w_gate"], dev["w_up"])
    folded = to_np(ops.llama_block_fwd_folded(to_dev(x, torch.bfloat16), wq, dev["w_o"], wg, wu, dev["w_down"], Bt,
                                              S, H, H))
    gf = folded[seq * S + rows]
    assert rel_err(gf, ref) <= BF16_TOL
    assert rel_err(gf - xs[rows], ref - xs[rows]) <= BF16_TOL
    assert ops.device_status(0)[0] == 0


def test_block_backward_shapes_sampled():
    """The backward operators at the block's shapes (tokens 8192, d_model 4096, SwiGLU hidden
    14336, QKV width 12288): swiglu_bwd (mlp.rs:31-52), linear_bwd (matmul.rs:60-78) and
    rmsnorm_bwd (norm.rs:33-50) on the GPU in full, the oracle on sampled rows of dx and
    sampled columns of the weight gradients (rmsnorm_bwd and dbias in full)."""
    import torch
    from beacon_b200 import ops
    T, dm, F, N = 8192, 4096, 14336, 12288
    t = lambda a: to_dev(a, torch.bfloat16)
    rng = np.random.default_rng(1)
    rows = np.sort(rng.choice(T, 16, replace=False))
    # SwiGLU MLP backward
    x, dy = as_bf16(normal((T, dm), 81)), as_bf16(normal((T, dm), 82))
    wg, wu = as_bf16(normal((dm, F), 83, std=0.02)), as_bf16(normal((dm, F), 84, std=0.02))
    wd = as_bf16(normal((F, dm), 85, std=0.02))
    dx, dwg, dwu, dwd = (to_np(a) for a in ops.swiglu_bwd(t(dy), t(x), t(wg), t(wu), t(wd)))
    cols = np.sort(rng.choice(F, 16, replace=False))
    rdx, rdwg, rdwu, rdwd = O.swiglu_bwd_sampled(dy, x, wg, wu, wd, rows, cols)
    assert rel_err(dx[rows], rdx) <= BF16_TOL
    assert rel_err(dwg[:, cols], rdwg) <= BF16_TOL and rel_err(dwu[:, cols], rdwu) <= BF16_TOL
    assert rel_err(dwd[cols, :], rdwd) <= BF16_TOL
    del dx, dwg, dwu, dwd, wg, wu, wd
    # linear backward of the QKV projection
    w = as_bf16(normal((dm, N), 86, std=0.02))
    dout = as_bf16(normal((T, N), 87))
    ldx, ldw, ldb = (to_np(a) for a in ops.linear_bwd(t(dout), t(x), t(w)))
    lcols = np.sort(rng.choice(N, 16, replace=False))
    f64 = lambda a: np.asarray(a, dtype=np.float64)
    assert rel_err(ldx[rows], f64(dout[rows]) @ f64(w).T) <= BF16_TOL
    assert rel_err(ldw[:, lcols], f64(x).T @ f64(dout[:, lcols])) <= BF16_TOL
    assert rel_err(ldb, f64(dout).sum(axis=0)) <= BF16_TOL
    del ldx, ldw, ldb, dout, w
    # RMSNorm backward, in full
    g = as_bf16(1.0 + 0.1 * normal((dm,), 88))
    _, rms = ops.rmsnorm_fwd(t(x), t(g))
    rdx, rdg = O.rmsnorm_bwd(dy, x, to_np(rms), g)
    ndx, ndg = ops.rmsnorm_bwd(t(dy), t(x), rms, t(g))
    assert rel_err(to_np(ndx), rdx) <= BF16_TOL and rel_err(to_np(ndg), rdg) <= BF16_TOL
    assert ops.device_status(0)[0] == 0
