"""Tensor-level front end over the C ABI (torch tensors for device memory and streams).

Every function checks its operands, calls one ``beacon_*`` entry point on the
current torch stream, and raises a :mod:`beacon_b200.errors` variant on failure.
Operands must be contiguous CUDA tensors: there is no CPU path.

Shapes follow the reference's launcher traits (crates/beacon-cuda/src/*.rs):
matrices are row-major ``[rows, cols]``, attention tensors ``[B, H, S, D]``.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .errors import InvalidLaunchConfig, check

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dtype(*ts) -> int:
    t0 = ts[0]
    if t0.dtype not in _DT:
        raise InvalidLaunchConfig(f"dtype {t0.dtype} not supported (float32, bfloat16)")
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise InvalidLaunchConfig("operands must be CUDA tensors (no CPU path)")
        if not t.is_contiguous():
            raise InvalidLaunchConfig("operands must be contiguous")
        if t.dtype != t0.dtype:
            raise InvalidLaunchConfig(f"mixed dtypes {t0.dtype} / {t.dtype}")
    return _DT[t0.dtype]


# ---------------------------------------------------------------- matmul / linear

def matmul_plan(m, k, n):
    """The bf16 GEMM's tile shape for [m, k] x [k, n] on the current device, with its wave
    efficiency: {tile_m, tile_n, tiles, sms_per_tile, sms, wave_efficiency}."""
    out = (ctypes.c_int32 * 5)()
    check(_lib.lib().beacon_matmul_plan(m, k, n, out))
    tile_m, tile_n, tiles, per, sms = (int(v) for v in out)
    slots = max(sms // per, 1)
    waves = -(-tiles // slots)
    return {"tile_m": tile_m, "tile_n": tile_n, "tiles": tiles, "sms_per_tile": per, "sms": sms,
            "wave_efficiency": tiles / (waves * slots)}


def matmul_fwd(lhs, rhs, out=None):
    """out[m,n] = lhs[m,k] . rhs[k,n]  (matmul.rs:18-29)."""
    m, k = lhs.shape
    k2, n = rhs.shape
    if k != k2:
        raise InvalidLaunchConfig(f"matmul_fwd: inner dims {k} vs {k2}")
    dt = _dtype(lhs, rhs)
    if out is None:
        out = torch.empty(m, n, dtype=lhs.dtype, device=lhs.device)
    check(_lib.lib().beacon_matmul_fwd(_p(out), _p(lhs), _p(rhs), m, k, n, dt, _stream()))
    return out


def matmul_bwd(dout, lhs, rhs, need_dlhs=True, need_drhs=True):
    """(dlhs, drhs) = (dout . rhs^T, lhs^T . dout)  (matmul.rs:31-44)."""
    m, k = lhs.shape
    n = rhs.shape[1]
    dt = _dtype(dout, lhs, rhs)
    dl = torch.empty(m, k, dtype=lhs.dtype, device=lhs.device) if need_dlhs else None
    dr = torch.empty(k, n, dtype=lhs.dtype, device=lhs.device) if need_drhs else None
    check(_lib.lib().beacon_matmul_bwd(_p(dl), _p(dr), _p(dout), _p(lhs), _p(rhs), m, k, n, dt, _stream()))
    return dl, dr


def linear_fwd(x, weight, bias=None, out=None):
    """out = x . weight + bias, weight [k, n]  (matmul.rs:46-58)."""
    m, k = x.shape
    n = weight.shape[1]
    dt = _dtype(x, weight, bias)
    if out is None:
        out = torch.empty(m, n, dtype=x.dtype, device=x.device)
    check(_lib.lib().beacon_linear_fwd(_p(out), _p(x), _p(weight), _p(bias), m, k, n, dt, _stream()))
    return out


def linear_bwd(dout, x, weight, need_dbias=True):
    """(dx, dweight, dbias)  (matmul.rs:60-78)."""
    m, k = x.shape
    n = weight.shape[1]
    dt = _dtype(dout, x, weight)
    dx = torch.empty_like(x)
    dw = torch.empty_like(weight)
    db = torch.empty(n, dtype=x.dtype, device=x.device) if need_dbias else None
    check(_lib.lib().beacon_linear_bwd(_p(dx), _p(dw), _p(db), _p(dout), _p(x), _p(weight), m, k, n, dt,
                                       _stream()))
    return dx, dw, db


def matmul_fp8w_fwd(lhs, rhs_fp8, scale=1.0, bias=None, out=None):
    """out = (lhs . decode_e4m3(rhs_fp8)) * scale (+ bias); lhs/bias/out bf16, rhs uint8 [k, n]."""
    m, k = lhs.shape
    k2, n = rhs_fp8.shape
    if k != k2 or rhs_fp8.dtype != torch.uint8 or lhs.dtype != torch.bfloat16:
        raise InvalidLaunchConfig("matmul_fp8w_fwd: lhs bf16 [m,k], rhs uint8 (fp8 e4m3) [k,n]")
    _dtype(lhs, bias)
    if not rhs_fp8.is_cuda or not rhs_fp8.is_contiguous():
        raise InvalidLaunchConfig("matmul_fp8w_fwd: rhs must be a contiguous CUDA tensor")
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=lhs.device)
    if bias is None:
        rc = _lib.lib().beacon_matmul_fp8w_fwd(_p(out), _p(lhs), _p(rhs_fp8), float(scale), m, k, n, _stream())
    else:
        rc = _lib.lib().beacon_linear_fp8w_fwd(_p(out), _p(lhs), _p(rhs_fp8), float(scale), _p(bias), m, k, n,
                                               _stream())
    check(rc)
    return out


def quantize_fp8e4m3(src):
    """fp32 master -> (fp8 e4m3 bytes, scale, amax): one scale per tensor, scale = amax / 448,
    q = F8E4M3::from_f32(src * 448 / amax) (crates/beacon-core/src/dtype.rs:163-195).
    scale and amax are one-element float32 device tensors."""
    if src.dtype != torch.float32 or not src.is_cuda or not src.is_contiguous():
        raise InvalidLaunchConfig("quantize_fp8e4m3: src must be a contiguous float32 CUDA tensor")
    q = torch.empty(src.shape, dtype=torch.uint8, device=src.device)
    scale = torch.empty(1, dtype=torch.float32, device=src.device)
    amax = torch.empty(1, dtype=torch.float32, device=src.device)
    check(_lib.lib().beacon_quantize_fp8e4m3(_p(q), _p(scale), _p(amax), _p(src), src.numel(), _stream()))
    return q, scale, amax


def linear_fp8w_fwd_devscale(x, weight_fp8, scale_dev, bias=None, out=None):
    """(x . decode(weight_fp8)) * scale_dev[0] (+ bias), the scale read on the device."""
    m, k = x.shape
    n = weight_fp8.shape[1]
    if weight_fp8.dtype != torch.uint8 or x.dtype != torch.bfloat16 or scale_dev.dtype != torch.float32:
        raise InvalidLaunchConfig("linear_fp8w_fwd_devscale: x bf16, weight uint8 (e4m3), scale float32")
    _dtype(x, bias)
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    check(_lib.lib().beacon_linear_fp8w_fwd_devscale(_p(out), _p(x), _p(weight_fp8), _p(scale_dev), _p(bias), m, k,
                                                     n, _stream()))
    return out


# ---------------------------------------------------------------- attention

def attention_fwd(q, k, v, causal=True, out=None, lse=None):
    """(out, lse) for q [B,Hq,S,D], k/v [B,Hkv,S,D]  (attention.rs:21-40; GQA when Hkv < Hq)."""
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    dt = _dtype(q, k, v)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty(B, Hq, S, dtype=torch.float32, device=q.device)
    L = _lib.lib()
    if Hkv == Hq:
        rc = L.beacon_attention_adjoint_fwd(_p(out), _p(q), _p(k), _p(v), _p(lse), B, Hq, S, D, int(causal), dt,
                                            _stream())
    else:
        rc = L.beacon_attention_gqa_fwd(_p(out), _p(q), _p(k), _p(v), _p(lse), B, Hq, Hkv, S, D, int(causal), dt,
                                        _stream())
    check(rc)
    return out, lse


def attention_bwd(dout, q, k, v, lse, causal=True, out=None, workspace=None):
    """(dq, dk, dv)  (attention.rs:42-64).  Passing the forward `out` skips its recompute."""
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    dt = _dtype(dout, q, k, v, out)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ws = _p(workspace)
    wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
    L = _lib.lib()
    if out is not None:
        rc = L.beacon_attention_bwd_with_out(_p(dq), _p(dk), _p(dv), _p(dout), _p(q), _p(k), _p(v), _p(out),
                                             _p(lse), B, Hq, Hkv, S, D, int(causal), dt, ws, wsb, _stream())
    elif Hkv == Hq:
        rc = L.beacon_attention_adjoint_bwd(_p(dq), _p(dk), _p(dv), _p(dout), _p(q), _p(k), _p(v), _p(lse), B, Hq,
                                            S, D, int(causal), dt, ws, wsb, _stream())
    else:
        rc = L.beacon_attention_gqa_bwd(_p(dq), _p(dk), _p(dv), _p(dout), _p(q), _p(k), _p(v), _p(lse), B, Hq,
                                        Hkv, S, D, int(causal), dt, ws, wsb, _stream())
    check(rc)
    return dq, dk, dv


def attention_bwd_workspace_bytes(B, Hq, S, D, dtype=torch.bfloat16) -> int:
    return int(_lib.lib().beacon_attention_bwd_workspace_size(B, Hq, S, D, _DT[dtype]))


# ---------------------------------------------------------------- RMSNorm

def rmsnorm_fwd(x, weight, eps=1e-5):
    """(out, rms) with rms[t] = sqrt(mean(x[t]^2) + eps)  (norm.rs:20-31)."""
    T, dim = x.shape
    dt = _dtype(x, weight)
    out = torch.empty_like(x)
    rms = torch.empty(T, dtype=torch.float32, device=x.device)
    check(_lib.lib().beacon_rmsnorm_adjoint_fwd(_p(out), _p(x), _p(weight), _p(rms), T, dim, eps, dt, _stream()))
    return out, rms


def rmsnorm_bwd(dy, x, rms, weight):
    """(dx, dweight)  (norm.rs:33-50)."""
    T, dim = x.shape
    dt = _dtype(dy, x, weight)
    dx = torch.empty_like(x)
    dw = torch.empty_like(weight)
    check(_lib.lib().beacon_rmsnorm_adjoint_bwd(_p(dx), _p(dw), _p(dy), _p(x), _p(rms), _p(weight), T, dim, dt,
                                                None, 0, _stream()))
    return dx, dw


def rmsnorm_fold_weight(gain, weight):
    """diag(gain) . weight: the RMSNorm gain folded into the rows of the weight that follows
    the norm (once per weight version)."""
    k, n = weight.shape
    dt = _dtype(weight, gain)
    out = torch.empty_like(weight)
    check(_lib.lib().beacon_rmsnorm_fold_weight(_p(out), _p(gain), _p(weight), k, n, dt, _stream()))
    return out


def rmsnorm_linear_fwd(x, weight_folded, bias=None, eps=1e-5, out=None):
    """(out, rms): rmsnorm(x, g) . W + bias with W folded as diag(g) . W
    (norm.rs:20-31 then matmul.rs:46-58 in one pass over x plus one GEMM)."""
    m, k = x.shape
    n = weight_folded.shape[1]
    dt = _dtype(x, weight_folded, bias)
    if out is None:
        out = torch.empty(m, n, dtype=x.dtype, device=x.device)
    rms = torch.empty(m, dtype=torch.float32, device=x.device)
    check(_lib.lib().beacon_rmsnorm_linear_fwd(_p(out), _p(rms), _p(x), _p(weight_folded), _p(bias), m, k, n, eps,
                                               dt, _stream()))
    return out, rms


# ---------------------------------------------------------------- LayerNorm

def layernorm_fwd(x, weight, bias, eps=1e-5):
    """(out, mean, invstd), biased variance  (norm.rs:56-73)."""
    T, dim = x.shape
    dt = _dtype(x, weight, bias)
    out = torch.empty_like(x)
    mean = torch.empty(T, dtype=torch.float32, device=x.device)
    invstd = torch.empty(T, dtype=torch.float32, device=x.device)
    check(_lib.lib().beacon_layernorm_adjoint_fwd(_p(out), _p(x), _p(weight), _p(bias), _p(mean), _p(invstd), T,
                                                  dim, eps, dt, _stream()))
    return out, mean, invstd


def layernorm_bwd(dy, x, mean, invstd, weight):
    """(dx, dweight, dbias)  (norm.rs:75-94)."""
    T, dim = x.shape
    dt = _dtype(dy, x, weight)
    dx = torch.empty_like(x)
    dw, db = torch.empty_like(weight), torch.empty_like(weight)
    check(_lib.lib().beacon_layernorm_adjoint_bwd(_p(dx), _p(dw), _p(db), _p(dy), _p(x), _p(mean), _p(invstd),
                                                  _p(weight), T, dim, dt, None, 0, _stream()))
    return dx, dw, db


# ---------------------------------------------------------------- SwiGLU MLP

def swiglu_fwd(x, gate_proj, up_proj, down_proj):
    """out = (silu(x Wg) * (x Wu)) Wd  (mlp.rs:12-29)."""
    T, dm = x.shape
    F = gate_proj.shape[1]
    dt = _dtype(x, gate_proj, up_proj, down_proj)
    out = torch.empty(T, dm, dtype=x.dtype, device=x.device)
    check(_lib.lib().beacon_swiglu_adjoint_fwd(_p(out), _p(x), _p(gate_proj), _p(up_proj), _p(down_proj), T, dm, F,
                                               dt, None, 0, _stream()))
    return out


def swiglu_bwd(dy, x, gate_proj, up_proj, down_proj):
    """(dx, dgate_proj, dup_proj, ddown_proj)  (mlp.rs:31-52)."""
    T, dm = x.shape
    F = gate_proj.shape[1]
    dt = _dtype(dy, x, gate_proj, up_proj, down_proj)
    dx = torch.empty_like(x)
    dg, du, dd = torch.empty_like(gate_proj), torch.empty_like(up_proj), torch.empty_like(down_proj)
    check(_lib.lib().beacon_swiglu_adjoint_bwd(_p(dx), _p(dg), _p(du), _p(dd), _p(dy), _p(x), _p(gate_proj),
                                               _p(up_proj), _p(down_proj), T, dm, F, dt, None, 0, _stream()))
    return dx, dg, du, dd


# ---------------------------------------------------------------- pre-norm block

def llama_block_workspace_bytes(batch, seq, d_model, heads, kv_heads, head_dim, d_ff) -> int:
    return int(_lib.lib().beacon_llama_block_workspace_size(batch, seq, d_model, heads, kv_heads, head_dim, d_ff,
                                                            _lib.BF16))


def llama_block_fwd(x, attn_norm, w_qkv, w_o, ffn_norm, w_gate, w_up, w_down, batch, seq, heads, kv_heads=None,
                    eps=1e-5, out=None, workspace=None):
    """One pre-norm block: h = x + attn(rmsnorm(x)) Wo; out = h + swiglu(rmsnorm(h)).

    x: [batch*seq, d_model] bf16; w_qkv: [d_model, (heads + 2*kv_heads)*head_dim]
    (query, key, value heads in that order); w_o: [heads*head_dim, d_model].
    """
    kv_heads = heads if kv_heads is None else kv_heads
    T, dm = x.shape
    hd = w_o.shape[0] // heads
    F = w_gate.shape[1]
    dt = _dtype(x, attn_norm, w_qkv, w_o, ffn_norm, w_gate, w_up, w_down)
    if out is None:
        out = torch.empty_like(x)
    ws, wsb = (None, 0) if workspace is None else (_p(workspace), workspace.numel() * workspace.element_size())
    check(_lib.lib().beacon_llama_block_fwd(_p(out), _p(x), _p(attn_norm), _p(w_qkv), _p(w_o), _p(ffn_norm),
                                            _p(w_gate), _p(w_up), _p(w_down), batch, seq, dm, heads, kv_heads, hd, F,
                                            eps, dt, ws, wsb, _stream()))
    return out


def llama_block_fold_weights(attn_norm, w_qkv, ffn_norm, w_gate, w_up):
    """(w_qkv_folded, w_gate_folded, w_up_folded) for llama_block_fwd_folded."""
    return (rmsnorm_fold_weight(attn_norm, w_qkv), rmsnorm_fold_weight(ffn_norm, w_gate),
            rmsnorm_fold_weight(ffn_norm, w_up))


def llama_block_fwd_folded(x, w_qkv_folded, w_o, w_gate_folded, w_up_folded, w_down, batch, seq, heads,
                           kv_heads=None, eps=1e-5, out=None, workspace=None):
    """llama_block_fwd with both RMSNorm gains folded into the weights that follow them
    (llama_block_fold_weights): the norms run as row statistics and GEMM row scales."""
    kv_heads = heads if kv_heads is None else kv_heads
    T, dm = x.shape
    hd = w_o.shape[0] // heads
    F = w_gate_folded.shape[1]
    dt = _dtype(x, w_qkv_folded, w_o, w_gate_folded, w_up_folded, w_down)
    if out is None:
        out = torch.empty_like(x)
    ws, wsb = (None, 0) if workspace is None else (_p(workspace), workspace.numel() * workspace.element_size())
    check(_lib.lib().beacon_llama_block_fwd_folded(_p(out), _p(x), _p(w_qkv_folded), _p(w_o), _p(w_gate_folded),
                                                   _p(w_up_folded), _p(w_down), batch, seq, dm, heads, kv_heads, hd,
                                                   F, eps, dt, ws, wsb, _stream()))
    return out


# ---------------------------------------------------------------- elementwise

def residual_add(a, b):
    """a + b  (elementwise.rs:47-55)."""
    dt = _dtype(a, b)
    out = torch.empty_like(a)
    check(_lib.lib().beacon_residual_add_fwd(_p(out), _p(a), _p(b), a.numel(), dt, _stream()))
    return out


def residual_add_bwd(dout):
    """(d_a, d_b) = (dout, dout)  (elementwise.rs:57-65)."""
    dt = _dtype(dout)
    da, db = torch.empty_like(dout), torch.empty_like(dout)
    check(_lib.lib().beacon_residual_add_bwd(_p(da), _p(db), _p(dout), dout.numel(), dt, _stream()))
    return da, db


def embedding_lookup(table, indices):
    """out[t] = table[indices[t]] (elementwise.rs:67-80); indices int32/uint32 on the device."""
    vocab, dim = table.shape
    dt = _dtype(table)
    if indices.dtype not in (torch.int32, torch.uint32) or not indices.is_cuda or not indices.is_contiguous():
        raise InvalidLaunchConfig("embedding_lookup: indices must be a contiguous 32-bit CUDA tensor")
    out = torch.empty(indices.numel(), dim, dtype=table.dtype, device=table.device)
    check(_lib.lib().beacon_embedding_lookup_fwd(_p(out), _p(table), _p(indices), indices.numel(), dim, vocab, dt,
                                                 _stream()))
    return out


def embedding_backward(d_table, d_out, indices):
    """d_table[indices[t]] += d_out[t] in place (elementwise.rs:82-95)."""
    vocab, dim = d_table.shape
    dt = _dtype(d_table, d_out)
    check(_lib.lib().beacon_embedding_lookup_bwd(_p(d_table), _p(d_out), _p(indices), indices.numel(), dim, vocab,
                                                 dt, _stream()))
    return d_table


def dropout_fwd(x, p, seed):
    """(out, mask) with mask = 1/(1-p) on kept elements, 0 on dropped (elementwise.rs:97-108)."""
    dt = _dtype(x)
    out, mask = torch.empty_like(x), torch.empty_like(x)
    check(_lib.lib().beacon_dropout_fwd(_p(out), _p(x), _p(mask), x.numel(), float(p), int(seed), dt, _stream()))
    return out, mask


def dropout_bwd(d_out, mask):
    """d_in = d_out * mask (elementwise.rs:110-118)."""
    dt = _dtype(d_out, mask)
    d_in = torch.empty_like(d_out)
    check(_lib.lib().beacon_dropout_bwd(_p(d_in), _p(d_out), _p(mask), d_out.numel(), dt, _stream()))
    return d_in


CAST_F32_TO_FP8E4M3, CAST_FP8E4M3_TO_F32, CAST_F32_TO_BF16, CAST_BF16_TO_F32 = 0, 1, 2, 3


def cast(src, kind: int):
    """CastKind conversions with the reference's rounding (elementwise.rs:120-128)."""
    if not src.is_cuda or not src.is_contiguous():
        raise InvalidLaunchConfig("cast: operand must be a contiguous CUDA tensor")
    out_dt = {0: torch.uint8, 1: torch.float32, 2: torch.bfloat16, 3: torch.float32}[kind]
    in_dt = {0: torch.float32, 1: torch.uint8, 2: torch.float32, 3: torch.bfloat16}[kind]
    if src.dtype != in_dt:
        raise InvalidLaunchConfig(f"cast kind {kind} expects {in_dt}, got {src.dtype}")
    out = torch.empty(src.shape, dtype=out_dt, device=src.device)
    check(_lib.lib().beacon_cast(_p(out), _p(src), src.numel(), kind, _stream()))
    return out


def device_status(device: int = 0):
    """(code, site, count) of device-side faults since the last call; raises Cuda on a fault."""
    arr = (ctypes.c_uint * 3)()
    rc = _lib.lib().beacon_device_status(device, arr)
    check(rc)
    return tuple(arr)


def launch_count() -> int:
    return int(_lib.lib().beacon_launch_count())


def profile_enable(on: bool = True) -> None:
    """Bracket the tensor-core kernels with CUDA events on their launch stream."""
    _lib.lib().beacon_profile_enable(int(on))


def profile_read(kernel: str):
    """(total milliseconds, launches) recorded for `kernel` since the last reset."""
    ms = ctypes.c_double()
    cnt = ctypes.c_uint64()
    check(_lib.lib().beacon_profile_read(kernel.encode(), ctypes.byref(ms), ctypes.byref(cnt)))
    return ms.value, int(cnt.value)


def profile_reset() -> None:
    check(_lib.lib().beacon_profile_read(None, None, None))
