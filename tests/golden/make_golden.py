"""Generates tests/golden/golden.npz: known answers for the oracle.

The op answers come from an independent float64 restatement in torch (autograd
for the gradients), on inputs drawn from the oracle's seeded SplitMix64 streams;
the codec tables come from a direct restatement of the fp8 e4m3 / bf16 formats
(crates/beacon-core/src/dtype.rs).  Run from the repository root:

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
import oracle as O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
f64 = lambda a: torch.tensor(a, dtype=torch.float64, requires_grad=True)


def attn_case(B, Hq, Hkv, S, D, seed, causal):
    nq, nk = B * Hq * S * D, B * Hkv * S * D
    q = O.normal((B, Hq, S, D), seed)
    k = O.normal((B, Hkv, S, D), seed, offset=nq)
    v = O.normal((B, Hkv, S, D), seed, offset=nq + nk)
    do = O.normal((B, Hq, S, D), seed, offset=nq + 2 * nk)
    tq, tk, tv = f64(q), f64(k), f64(v)
    g = Hq // Hkv
    kk, vv = tk.repeat_interleave(g, 1), tv.repeat_interleave(g, 1)
    s = (tq @ kk.transpose(-1, -2)) / np.sqrt(D)
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1), -float("inf"))
    o = torch.softmax(s, -1) @ vv
    lse = torch.logsumexp(s, -1)
    o.backward(torch.tensor(do, dtype=torch.float64))
    return {"o": o.detach().numpy(), "lse": lse.detach().numpy(), "dq": tq.grad.numpy(), "dk": tk.grad.numpy(),
            "dv": tv.grad.numpy()}


def fp8_decode(b):
    s = -1.0 if b & 0x80 else 1.0
    e, m = (b >> 3) & 0xF, b & 7
    if e == 0xF and m == 7:
        return np.nan
    if e == 0:
        return s * m * 2.0 ** -9
    return s * (1 + m / 8) * 2.0 ** (e - 7)


def main():
    G = {}
    # PRNG streams (first values)
    G["prng_normal_seed0"] = O.normal((16,), 0).astype(np.float64)
    G["prng_uniform_seed1"] = O.uniform((16,), 1).astype(np.float64)
    # attention: config-1 shape (f32 causal B=1 H=4 S=128 D=64, seed 0), GQA, non-causal
    for name, args in {"attn_cfg1": (1, 4, 4, 128, 64, 0, True), "attn_gqa": (1, 4, 2, 48, 16, 11, True),
                       "attn_full": (2, 2, 2, 40, 32, 12, False)}.items():
        for k, v in attn_case(*args).items():
            G[f"{name}_{k}"] = v
    # GEMM family
    a, b = O.uniform((48, 40), 1), O.uniform((40, 24), 2)
    bias, dy = O.normal((24,), 3), O.normal((48, 24), 4)
    ta, tb, tbias = f64(a), f64(b), f64(bias)
    y = ta @ tb + tbias
    y.backward(torch.tensor(dy, dtype=torch.float64))
    G["lin_y"], G["lin_dx"], G["lin_dw"], G["lin_db"] = (y.detach().numpy(), ta.grad.numpy(), tb.grad.numpy(),
                                                         tbias.grad.numpy())
    # RMSNorm
    x, w, dy = O.normal((8, 64), 5), O.normal((64,), 6), O.normal((8, 64), 7)
    tx, tw = f64(x), f64(w)
    r = torch.sqrt((tx * tx).mean(-1, keepdim=True) + 1e-5)
    y = tx * tw / r
    y.backward(torch.tensor(dy, dtype=torch.float64))
    G["rms_y"], G["rms_rms"], G["rms_dx"], G["rms_dw"] = (y.detach().numpy(), r.detach().numpy()[:, 0],
                                                          tx.grad.numpy(), tw.grad.numpy())
    # LayerNorm (biased variance, eps 1e-5)
    x, w, bb, dy = O.normal((8, 96), 13), O.normal((96,), 14), O.normal((96,), 15), O.normal((8, 96), 16)
    tx, tw, tb = f64(x), f64(w), f64(bb)
    mu = tx.mean(-1, keepdim=True)
    inv = 1.0 / torch.sqrt(((tx - mu) ** 2).mean(-1, keepdim=True) + 1e-5)
    y = (tx - mu) * inv * tw + tb
    y.backward(torch.tensor(dy, dtype=torch.float64))
    G["ln_y"], G["ln_mean"], G["ln_invstd"] = (y.detach().numpy(), mu.detach().numpy()[:, 0],
                                               inv.detach().numpy()[:, 0])
    G["ln_dx"], G["ln_dw"], G["ln_db"] = tx.grad.numpy(), tw.grad.numpy(), tb.grad.numpy()
    # SwiGLU MLP
    x = O.normal((16, 32), 8)
    wg, wu, wd = O.normal((32, 48), 9, std=0.2), O.normal((32, 48), 10, std=0.2), O.normal((48, 32), 11, std=0.2)
    dy = O.normal((16, 32), 12)
    T = [f64(t) for t in (x, wg, wu, wd)]
    y = (torch.nn.functional.silu(T[0] @ T[1]) * (T[0] @ T[2])) @ T[3]
    y.backward(torch.tensor(dy, dtype=torch.float64))
    G["swiglu_y"] = y.detach().numpy()
    for n, t in zip(("dx", "dwg", "dwu", "dwd"), T):
        G[f"swiglu_{n}"] = t.grad.numpy()
    # codecs
    G["fp8_decode_table"] = np.array([fp8_decode(i) for i in range(256)], dtype=np.float64)
    G["bf16_special_in"] = np.array([1.0, -2.5, 3.1415927, 1e6, -1e-6, 65504.0, 1.00390625, 1.01171875,
                                     np.inf, -np.inf, 3.4e38], dtype=np.float32)
    # round-to-nearest-even on the top 16 bits, computed with integer arithmetic here
    bits = G["bf16_special_in"].view(np.uint32).astype(np.uint64)
    G["bf16_special_out"] = (((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)
    # op answers are stored as float32 (their rounding, 6e-8 relative, is far below the 1e-6 check)
    for key in list(G):
        if G[key].dtype == np.float64 and not key.startswith(("fp8_", "prng_")):
            G[key] = G[key].astype(np.float32)
    np.savez_compressed(OUT, **G)
    print("wrote", OUT, os.path.getsize(OUT), "bytes,", len(G), "arrays")


if __name__ == "__main__":
    main()
