"""CPU oracle for the beacon hot path -- TEST INFRASTRUCTURE ONLY.

ctypes front end over ``libbeacon_oracle.so`` (built from ``beacon_oracle.c`` by
``oracle/Makefile``).  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package: it is the checker, never the thing measured or shipped.

Parity status: the dtype codecs restate crates/beacon-core/src/dtype.rs and are
pinned by that file's known-answer tests; the op results (attention, GEMM,
RMSNorm, SwiGLU) are parity unpinned by the reference, which has no numeric
implementation (crates/beacon-ops/src/lib.rs:1), and are cross-checked against
torch float64 instead.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libbeacon_oracle.so")
_lib = None

_f = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.c_int64


def build() -> str:
    """Compile the oracle library in place (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.bo_splitmix64.restype = ctypes.c_uint64
        L.bo_splitmix64.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.bo_fill_uniform.argtypes = [_f, ctypes.c_size_t, ctypes.c_float, ctypes.c_float,
                                      ctypes.c_uint64, ctypes.c_uint64]
        L.bo_fill_normal.argtypes = [_f, ctypes.c_size_t, ctypes.c_float, ctypes.c_float,
                                     ctypes.c_uint64, ctypes.c_uint64]
        L.bo_bf16_from_f32.restype = ctypes.c_uint16
        L.bo_bf16_from_f32.argtypes = [ctypes.c_float]
        L.bo_bf16_to_f32.restype = ctypes.c_float
        L.bo_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.bo_fp8e4m3_from_f32.restype = ctypes.c_uint8
        L.bo_fp8e4m3_from_f32.argtypes = [ctypes.c_float]
        L.bo_fp8e4m3_to_f32.restype = ctypes.c_float
        L.bo_fp8e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.bo_f32_to_bf16.argtypes = [ctypes.c_void_p, _f, ctypes.c_size_t]
        L.bo_bf16_to_f32_n.argtypes = [_f, ctypes.c_void_p, ctypes.c_size_t]
        L.bo_round_bf16_inplace.argtypes = [_f, ctypes.c_size_t]
        L.bo_f32_to_fp8e4m3.argtypes = [ctypes.c_void_p, _f, ctypes.c_size_t]
        L.bo_fp8e4m3_to_f32_n.argtypes = [_f, ctypes.c_void_p, ctypes.c_size_t]
        L.bo_matmul_fwd.argtypes = [_f, _f, _f, _i64, _i64, _i64]
        L.bo_matmul_bwd.argtypes = [_f, _f, _f, _f, _f, _i64, _i64, _i64]
        L.bo_linear_fwd.argtypes = [_f, _f, _f, _f, _i64, _i64, _i64]
        L.bo_linear_bwd.argtypes = [_f, _f, _f, _f, _f, _f, _i64, _i64, _i64]
        L.bo_attention_fwd.argtypes = [_f, _f, _f, _f, _f, _i64, _i64, _i64, _i64, _i64,
                                       ctypes.c_int, ctypes.c_float]
        L.bo_attention_fwd_heads.argtypes = [_f, _f, _f, _f, _f, _i64, _i64, _i64, _i64, _i64,
                                             ctypes.c_int, ctypes.c_float,
                                             ctypes.POINTER(ctypes.c_int64), _i64]
        L.bo_attention_bwd.argtypes = [_f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _i64,
                                       _i64, ctypes.c_int, ctypes.c_float]
        L.bo_attention_fwd_rows.argtypes = [_f, _f, _f, _f, _f, _i64, _i64, ctypes.c_int, ctypes.c_float,
                                            ctypes.POINTER(ctypes.c_int64), _i64]
        L.bo_attention_bwd_head.argtypes = [_f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64, ctypes.c_int,
                                            ctypes.c_float]
        L.bo_rmsnorm_fwd.argtypes = [_f, _f, _f, _f, _i64, _i64, ctypes.c_float]
        L.bo_rmsnorm_bwd.argtypes = [_f, _f, _f, _f, _f, _f, _i64, _i64]
        L.bo_layernorm_fwd.argtypes = [_f, _f, _f, _f, _f, _f, _i64, _i64, ctypes.c_float]
        L.bo_layernorm_bwd.argtypes = [_f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64]
        L.bo_swiglu_fwd.argtypes = [_f, _f, _f, _f, _f, _i64, _i64, _i64]
        L.bo_swiglu_bwd.argtypes = [_f, _f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64]
        L.bo_residual_add_fwd.argtypes = [_f, _f, _f, _i64]
        L.bo_residual_add_bwd.argtypes = [_f, _f, _f, _i64]
        L.bo_num_threads.restype = ctypes.c_int
        L.bo_set_num_threads.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_f)


def _empty(*shape) -> np.ndarray:
    return np.empty(shape, dtype=np.float32)


# ---- inputs -----------------------------------------------------------------

def normal(shape, seed: int, mean: float = 0.0, std: float = 1.0, offset: int = 0) -> np.ndarray:
    out = _empty(*shape)
    lib().bo_fill_normal(_p(out), out.size, mean, std, seed, offset)
    return out


def uniform(shape, seed: int, lo: float = -1.0, hi: float = 1.0, offset: int = 0) -> np.ndarray:
    out = _empty(*shape)
    lib().bo_fill_uniform(_p(out), out.size, lo, hi, seed, offset)
    return out


# ---- codecs -----------------------------------------------------------------

def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().bo_f32_to_bf16(out.ctypes.data, _p(x), x.size)
    return out


def from_bf16_bits(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = _empty(*h.shape)
    lib().bo_bf16_to_f32_n(_p(out), h.ctypes.data, h.size)
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    out = np.array(x, dtype=np.float32, copy=True, order="C")
    lib().bo_round_bf16_inplace(_p(out), out.size)
    return out


def to_fp8_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint8)
    lib().bo_f32_to_fp8e4m3(out.ctypes.data, _p(x), x.size)
    return out


def quantize_fp8e4m3(x: np.ndarray):
    """fp32 master -> fp8 e4m3 with one scale per tensor, in float32 arithmetic:
    amax = max |x| (NaN ignored), scale = amax / 448 (1 when amax is 0),
    q = F8E4M3::from_f32(x * (448 / amax)) (the encode of crates/beacon-core/src/dtype.rs:163-195).
    The reference names the step ("fp32 master -> fp8 weights", crates/beacon-train/Cargo.toml:7)
    but fixes no scale convention; this is the one the library implements.
    Returns (codes uint8, scale float32, amax float32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    finite = np.abs(x[~np.isnan(x)])
    a = np.float32(finite.max()) if finite.size else np.float32(0.0)
    inv = np.float32(448.0) / a if a > 0 else np.float32(1.0)
    scale = a / np.float32(448.0) if a > 0 else np.float32(1.0)
    return to_fp8_bits((x * inv).astype(np.float32)), np.float32(scale), np.float32(a)


def from_fp8_bits(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8)
    out = _empty(*b.shape)
    lib().bo_fp8e4m3_to_f32_n(_p(out), b.ctypes.data, b.size)
    return out


# ---- ops ----------------------------------------------------------------------

def matmul_fwd(lhs, rhs):
    M, K = lhs.shape
    N = rhs.shape[1]
    out = _empty(M, N)
    lib().bo_matmul_fwd(_p(out), _p(lhs), _p(rhs), M, K, N)
    return out


def matmul_bwd(dout, lhs, rhs):
    M, K = lhs.shape
    N = rhs.shape[1]
    dl, dr = _empty(M, K), _empty(K, N)
    lib().bo_matmul_bwd(_p(dl), _p(dr), _p(dout), _p(lhs), _p(rhs), M, K, N)
    return dl, dr


def linear_fwd(x, w, bias=None):
    M, K = x.shape
    N = w.shape[1]
    out = _empty(M, N)
    lib().bo_linear_fwd(_p(out), _p(x), _p(w), _p(bias), M, K, N)
    return out


def linear_bwd(dy, x, w):
    M, K = x.shape
    N = w.shape[1]
    dx, dw, db = _empty(M, K), _empty(K, N), _empty(N)
    lib().bo_linear_bwd(_p(dx), _p(dw), _p(db), _p(dy), _p(x), _p(w), M, K, N)
    return dx, dw, db


def attention_fwd(q, k, v, causal=True, scale=0.0):
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    out, lse = _empty(B, Hq, S, D), _empty(B, Hq, S)
    lib().bo_attention_fwd(_p(out), _p(lse), _p(q), _p(k), _p(v), B, Hq, Hkv, S, D, int(causal), scale)
    return out, lse


def attention_fwd_heads(q, k, v, heads, causal=True, scale=0.0):
    """Forward for the listed flat (b*Hq + h) query heads only; other rows stay NaN."""
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    out = np.full((B, Hq, S, D), np.nan, dtype=np.float32)
    lse = np.full((B, Hq, S), np.nan, dtype=np.float32)
    hs = np.ascontiguousarray(np.asarray(heads, dtype=np.int64))
    lib().bo_attention_fwd_heads(_p(out), _p(lse), _p(q), _p(k), _p(v), B, Hq, Hkv, S, D,
                                 int(causal), scale,
                                 hs.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), hs.size)
    return out, lse


def attention_fwd_rows(q, k, v, rows, causal=True, scale=0.0):
    """Forward of one head (q, k, v: [S, D]) for the listed query rows: (out [n, D], lse [n])."""
    S, D = q.shape
    rs = np.ascontiguousarray(np.asarray(rows, dtype=np.int64))
    out, lse = _empty(rs.size, D), _empty(rs.size)
    lib().bo_attention_fwd_rows(_p(out), _p(lse), _p(np.ascontiguousarray(q)), _p(np.ascontiguousarray(k)),
                                _p(np.ascontiguousarray(v)), S, D, int(causal), scale,
                                rs.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), rs.size)
    return out, lse


def attention_bwd_head(dout, q, k, v, lse, causal=True, scale=0.0):
    """Backward of one head ([S, D] each, lse [S]), rows spread over the threads: (dq, dk, dv)."""
    S, D = q.shape
    dq, dk, dv = _empty(S, D), _empty(S, D), _empty(S, D)
    c = np.ascontiguousarray
    lib().bo_attention_bwd_head(_p(dq), _p(dk), _p(dv), _p(c(dout)), _p(c(q)), _p(c(k)), _p(c(v)), _p(c(lse)),
                                S, D, int(causal), scale)
    return dq, dk, dv


def attention_bwd(dout, q, k, v, lse, causal=True, scale=0.0):
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    dq, dk, dv = _empty(B, Hq, S, D), _empty(B, Hkv, S, D), _empty(B, Hkv, S, D)
    lib().bo_attention_bwd(_p(dq), _p(dk), _p(dv), _p(dout), _p(q), _p(k), _p(v), _p(lse),
                           B, Hq, Hkv, S, D, int(causal), scale)
    return dq, dk, dv


def rmsnorm_fwd(x, g, eps=1e-5):
    T, dim = x.shape
    y, rms = _empty(T, dim), _empty(T)
    lib().bo_rmsnorm_fwd(_p(y), _p(rms), _p(x), _p(g), T, dim, eps)
    return y, rms


def rmsnorm_bwd(dy, x, rms, g):
    T, dim = x.shape
    dx, dg = _empty(T, dim), _empty(dim)
    lib().bo_rmsnorm_bwd(_p(dx), _p(dg), _p(dy), _p(x), _p(rms), _p(g), T, dim)
    return dx, dg


def layernorm_fwd(x, g, b, eps=1e-5):
    T, dim = x.shape
    y, mean, invstd = _empty(T, dim), _empty(T), _empty(T)
    lib().bo_layernorm_fwd(_p(y), _p(mean), _p(invstd), _p(x), _p(g), _p(b), T, dim, eps)
    return y, mean, invstd


def layernorm_bwd(dy, x, mean, invstd, g):
    T, dim = x.shape
    dx, dg, db = _empty(T, dim), _empty(dim), _empty(dim)
    lib().bo_layernorm_bwd(_p(dx), _p(dg), _p(db), _p(dy), _p(x), _p(mean), _p(invstd), _p(g), T, dim)
    return dx, dg, db


def swiglu_fwd(x, wg, wu, wd):
    T, dm = x.shape
    F = wg.shape[1]
    out = _empty(T, dm)
    lib().bo_swiglu_fwd(_p(out), _p(x), _p(wg), _p(wu), _p(wd), T, dm, F)
    return out


def swiglu_bwd(dy, x, wg, wu, wd):
    T, dm = x.shape
    F = wg.shape[1]
    dx, dwg, dwu, dwd = _empty(T, dm), _empty(dm, F), _empty(dm, F), _empty(F, dm)
    lib().bo_swiglu_bwd(_p(dx), _p(dwg), _p(dwu), _p(dwd), _p(dy), _p(x), _p(wg), _p(wu), _p(wd),
                        T, dm, F)
    return dx, dwg, dwu, dwd


def swiglu_bwd_sampled(dy, x, wg, wu, wd, rows, cols):
    """swiglu_bwd (crates/beacon-cuda/src/mlp.rs:31-52; adjoint
    crates/beacon-adjoint-table/src/lib.rs:100-107: x stored, gate and up recomputed) at
    sampled rows of dx and sampled hidden columns of the weight gradients, in float64:
        g = x Wg, u = x Wu, s = sigmoid(g), h = g s u, dh = dy Wd^T,
        dgate = dh u s (1 + g (1 - s)), dup = dh g s,
        dx = dgate Wg^T + dup Wu^T, dWg = x^T dgate, dWu = x^T dup, dWd = h^T dy.
    Each sampled quantity needs only its own rows / columns of the intermediates, so the
    block-sized backward (T = 8192, d_model = 4096, d_ff = 14336) is checked in seconds.
    Returns (dx[rows], dWg[:, cols], dWu[:, cols], dWd[cols, :])."""
    f = lambda a: np.asarray(a, dtype=np.float64)
    x64, dy64 = f(x), f(dy)
    rows, cols = np.asarray(rows), np.asarray(cols)

    def parts(xr, dyr, wg_, wu_, wd_t):
        g, u, dh = xr @ wg_, xr @ wu_, dyr @ wd_t
        s = 1.0 / (1.0 + np.exp(-g))
        return g, u, s, dh * u * s * (1.0 + g * (1.0 - s)), dh * g * s

    _, _, _, dgr, dur = parts(x64[rows], dy64[rows], f(wg), f(wu), f(wd).T)
    dx = dgr @ f(wg).T + dur @ f(wu).T
    g, u, s, dgc, duc = parts(x64, dy64, f(wg[:, cols]), f(wu[:, cols]), f(wd[cols, :]).T)
    return (dx.astype(np.float32), (x64.T @ dgc).astype(np.float32), (x64.T @ duc).astype(np.float32),
            ((g * s * u).T @ dy64).astype(np.float32))


def embedding_lookup_fwd(table, indices):
    """embedding_lookup (crates/beacon-cuda/src/elementwise.rs:67-80): out[t] = table[indices[t]];
    an index at or beyond the table gives a zero row (the library's rule for that case)."""
    idx = np.asarray(indices, dtype=np.int64)
    out = np.zeros((idx.size, table.shape[1]), dtype=np.float32)
    ok = idx < table.shape[0]
    out[ok] = table[idx[ok]]
    return out


def embedding_lookup_bwd(d_table, d_out, indices):
    """embedding_backward (elementwise.rs:82-95): d_table[indices[t]] += d_out[t] (float64 sums,
    indices beyond the table skipped).  Returns the updated copy of d_table."""
    idx = np.asarray(indices, dtype=np.int64)
    acc = np.asarray(d_table, dtype=np.float64).copy()
    ok = idx < acc.shape[0]
    np.add.at(acc, idx[ok], np.asarray(d_out, dtype=np.float64)[ok])
    return acc.astype(np.float32)


def _splitmix64(seed: int, i: np.ndarray) -> np.ndarray:
    """SplitMix64 at counters i (the same stream as bo_splitmix64), vectorised in uint64."""
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (i.astype(np.uint64) + np.uint64(1)) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def dropout_fwd(x, p, seed, bf16=False):
    """dropout_forward (elementwise.rs:97-108) with the library's mask rule: element i is kept
    when (splitmix64(seed, i) >> 40) / 2^24 >= p; mask = 1 / (1 - p) (float32, rounded to bf16
    for bf16 data) where kept, 0 where dropped; out = x * mask in float32 (rounded to bf16 for
    bf16 data).  Returns (out, mask)."""
    x = np.asarray(x, dtype=np.float32).ravel()
    u = (_splitmix64(seed, np.arange(x.size)) >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    p32 = np.float32(p)
    keep = (u >= p32) & (p32 < np.float32(1.0))
    scale = np.float32(1.0) / (np.float32(1.0) - p32) if p32 < 1 else np.float32(0.0)
    if bf16:
        scale = round_bf16(np.array([scale], dtype=np.float32))[0]
    mask = np.where(keep, scale, np.float32(0.0)).astype(np.float32)
    out = np.where(keep, x * scale, np.float32(0.0)).astype(np.float32)
    if bf16:
        out = round_bf16(out)
    return out, mask


def residual_add_fwd(a, b):
    out = _empty(*a.shape)
    lib().bo_residual_add_fwd(_p(out), _p(a), _p(b), a.size)
    return out


def llama_block_fwd(x, attn_norm, w_qkv, w_o, ffn_norm, w_gate, w_up, w_down, batch, seq, heads, kv_heads,
                    eps=1e-5, round_between=True):
    """Pre-norm Llama block composed from the operator restatements above, in the order a
    caller of the reference's ops would make: rmsnorm_fwd (crates/beacon-cuda/src/norm.rs:19-31),
    linear_fwd (crates/beacon-cuda/src/matmul.rs:46-58), attention_fwd
    (crates/beacon-cuda/src/attention.rs:21-40) on [B, H, S, D] tensors, residual_add
    (crates/beacon-cuda/src/elementwise.rs:47-55) and swiglu_fwd (crates/beacon-cuda/src/mlp.rs:12-29).
    With ``round_between`` every operator output is rounded to bf16, as bf16 operators
    would store it."""
    rnd = round_bf16 if round_between else (lambda a: a)
    T, dm = x.shape
    hd = w_o.shape[0] // heads
    xn, _ = rmsnorm_fwd(x, attn_norm, eps)
    qkv = rnd(matmul_fwd(rnd(xn), w_qkv))

    def heads_major(cols, nh):
        return np.ascontiguousarray(cols.reshape(batch, seq, nh, hd).transpose(0, 2, 1, 3))

    q = heads_major(qkv[:, :heads * hd], heads)
    k = heads_major(qkv[:, heads * hd:(heads + kv_heads) * hd], kv_heads)
    v = heads_major(qkv[:, (heads + kv_heads) * hd:], kv_heads)
    ao, _ = attention_fwd(q, k, v, causal=True)
    ao = rnd(np.ascontiguousarray(ao.transpose(0, 2, 1, 3)).reshape(T, heads * hd))
    h = rnd(residual_add_fwd(rnd(matmul_fwd(ao, w_o)), x)) if round_between else matmul_fwd(ao, w_o) + x
    hn, _ = rmsnorm_fwd(h, ffn_norm, eps)
    f = swiglu_fwd(rnd(hn), w_gate, w_up, w_down)
    return residual_add_fwd(rnd(f), h)


def llama_block_fwd_rows(x_seq, attn_norm, w_qkv, w_o, ffn_norm, w_gate, w_up, w_down, heads, kv_heads, rows,
                         eps=1e-5):
    """The pre-norm block of llama_block_fwd for ONE sequence (x_seq [S, dm]), evaluated
    only at the listed rows: the full-size check of the block (batch 4 x seq 2048,
    d_model 4096) in seconds.  Every row's keys and values are computed (attention needs
    them); queries, the output projection and the MLP only for `rows`.  The operators
    are the same restatements -- rmsnorm_fwd (crates/beacon-cuda/src/norm.rs:19-31),
    linear_fwd (crates/beacon-cuda/src/matmul.rs:46-58) as float64 matrix products,
    attention_fwd (crates/beacon-cuda/src/attention.rs:21-40) on the sampled rows,
    residual_add (crates/beacon-cuda/src/elementwise.rs:47-55) and swiglu_fwd
    (crates/beacon-cuda/src/mlp.rs:12-29) -- with every operator output rounded to bf16
    as bf16 operators store it.  Returns out[rows] [len(rows), dm]."""
    S, dm = x_seq.shape
    hd = w_o.shape[0] // heads
    rows = np.asarray(rows, dtype=np.int64)
    f64 = lambda a: np.asarray(a, dtype=np.float64)
    xn, _ = rmsnorm_fwd(np.ascontiguousarray(x_seq), attn_norm, eps)
    xn = f64(round_bf16(xn))
    nq, nkv = heads * hd, kv_heads * hd
    kv = round_bf16((xn @ f64(w_qkv[:, nq:nq + 2 * nkv])).astype(np.float32))
    q = round_bf16((xn[rows] @ f64(w_qkv[:, :nq])).astype(np.float32))
    ao = np.empty((rows.size, nq), dtype=np.float32)
    group = heads // kv_heads
    for h in range(heads):
        g = h // group
        kh = np.ascontiguousarray(kv[:, g * hd:(g + 1) * hd])
        vh = np.ascontiguousarray(kv[:, nkv + g * hd:nkv + (g + 1) * hd])
        # a query row stands alone: put row r of the sample at position rows[r] of a
        # copy of the head, so the causal limit is its own position
        qh = np.zeros((S, hd), dtype=np.float32)
        qh[rows] = q[:, h * hd:(h + 1) * hd]
        o, _ = attention_fwd_rows(qh, kh, vh, rows, causal=True)
        ao[:, h * hd:(h + 1) * hd] = o
    ao = f64(round_bf16(ao))
    hres = f64(round_bf16((ao @ f64(w_o) + f64(x_seq[rows])).astype(np.float32)))
    hn, _ = rmsnorm_fwd(np.ascontiguousarray(hres.astype(np.float32)), ffn_norm, eps)
    hn = f64(round_bf16(hn))
    gate, up = hn @ f64(w_gate), hn @ f64(w_up)
    act = f64(round_bf16((gate / (1.0 + np.exp(-gate)) * up).astype(np.float32)))
    return (act @ f64(w_down) + hres).astype(np.float32)


def num_threads() -> int:
    return int(lib().bo_num_threads())


def set_num_threads(n: int) -> None:
    lib().bo_set_num_threads(int(n))


def rel_err(x: np.ndarray, ref: np.ndarray) -> float:
    """Norm-wise relative error max|x - ref| / max|ref| (the tolerance measure of the tests)."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = float(np.max(np.abs(ref))) if ref.size else 0.0
    if denom == 0.0:
        return float(np.max(np.abs(x - ref))) if ref.size else 0.0
    return float(np.max(np.abs(x - ref)) / denom)
