"""Small, self-contained launches of one hot-path kernel, for ncu captures and quick timing.

    python profile_cases.py attn_bwd --heads 32
    python profile_cases.py attn_fwd --heads 32
    python profile_cases.py gemm --m 4096 --n 4096 --k 4096
    python profile_cases.py layernorm_bwd --tokens 16384 --width 4096
    python profile_cases.py gemm_fp8 --m 4096 --n 4096 --k 4096
    python profile_cases.py swiglu_bwd --tokens 16384 --width 4096 --n 14336
    python profile_cases.py swiglu_fwd --tokens 4096 --width 4096 --n 14336
    python profile_cases.py residual_add | cast_f32_bf16 | dropout_fwd   (16384 x 4096 elements)
    python profile_cases.py block          (pre-norm block forward, batch 4 x seq 2048, d_model 4096)
    python profile_cases.py block_folded   (the same with both RMSNorms folded into the GEMMs)

Each case runs `--warmup` untimed launches and then `--iters` launches timed with
CUDA events, printing the per-launch time and TFLOP/s (algorithmic FLOPs: causal
attention forward 2*H*S^2*D, backward 2.5x that; GEMM 2*M*N*K).  The LayerNorm
and RMSNorm backward cases are HBM-bound and print GB/s of algorithmic bytes instead
(RMSNorm backward: x, dy in, dx out, 4 B of rms per row): the LayerNorm forward reads x
and writes out (2 * tokens * width * 2 B, bf16) plus 8 B of statistics per row; the
backward reads x and dy and writes dx (3 * tokens * width * 2 B) plus the statistics
read, timed over the whole call (row kernel and the two column sums).  The elementwise
cases count their operands once: residual add and dropout 3 x 2 B per element (two bf16
tensors in and one out, or one in and out plus the mask), the f32 -> bf16 cast 4 + 2 B.
Sizes default to
a case larger than the 126 MB L2 but a few hundred MB on the device, the size an
ncu capture of a single launch (-k <kernel> -s <warmup launches> -c 1) should use.
"""
from __future__ import annotations

import argparse
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["attn_fwd", "attn_bwd", "attn_bwd_recompute", "gemm", "gemm_fp8", "swiglu_bwd",
                                     "swiglu_fwd", "block", "block_folded", "residual_add", "cast_f32_bf16",
                                     "dropout_fwd",
                                     "layernorm_fwd", "layernorm_bwd", "rmsnorm_fwd", "rmsnorm_bwd"])
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--width", type=int, default=4096)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=0)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--dim", type=int, default=128)
    ap.add_argument("--non-causal", action="store_true", help="attention cases: every key for every query")
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args(argv)

    import torch

    from beacon_b200 import ops

    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    if a.case.startswith(("layernorm", "rmsnorm", "residual", "cast", "dropout")):
        return _hbm_case(a, torch, ops, dev)
    if a.case.startswith("attn"):
        H, S, D = a.heads, a.seq, a.dim
        Hkv = a.kv_heads or H
        q = torch.randn(1, H, S, D, device=dev).bfloat16()
        k = torch.randn(1, Hkv, S, D, device=dev).bfloat16()
        v = torch.randn(1, Hkv, S, D, device=dev).bfloat16()
        do = torch.randn(1, H, S, D, device=dev).bfloat16()
        c = not a.non_causal
        out, lse = ops.attention_fwd(q, k, v, causal=c)
        fwd = 2.0 * H * S * S * D * (1 if c else 2)
        if a.case == "attn_fwd":
            fn, flops, kname = (lambda: ops.attention_fwd(q, k, v, causal=c, out=out, lse=lse)), fwd, "k_attn_fwd_tc"
        elif a.case == "attn_bwd":
            fn, flops, kname = ((lambda: ops.attention_bwd(do, q, k, v, lse, causal=c, out=out)), 2.5 * fwd,
                                "k_attn_bwd_dkdv")
        else:
            fn, flops, kname = (lambda: ops.attention_bwd(do, q, k, v, lse, causal=c)), 2.5 * fwd, "k_attn_bwd_dkdv"
    elif a.case == "gemm_fp8":
        A = (torch.rand(a.m, a.k, device=dev) * 2 - 1).bfloat16()
        W8, scale, _ = ops.quantize_fp8e4m3(torch.randn(a.k, a.n, device=dev))
        C = torch.empty(a.m, a.n, device=dev, dtype=torch.bfloat16)
        fn = lambda: ops.linear_fp8w_fwd_devscale(A, W8, scale, out=C)
        flops, kname = 2.0 * a.m * a.n * a.k, "k_gemm_fp8w_tc2"
    elif a.case.startswith("block"):
        # pre-norm Llama block forward: batch 4 x seq 2048, d_model 4096, 32 x 128 heads, SwiGLU 14336
        Bb, Sb, dm, Hb, F = 4, 2048, 4096, 32, 14336
        T = Bb * Sb
        x = torch.randn(T, dm, device=dev).bfloat16()
        w = lambda r, c: (torch.randn(r, c, device=dev) * 0.02).bfloat16()
        n1, n2 = torch.ones(dm, device=dev).bfloat16(), torch.ones(dm, device=dev).bfloat16()
        wqkv, wo, wg, wu, wd = w(dm, 3 * dm), w(dm, dm), w(dm, F), w(dm, F), w(F, dm)
        out = torch.empty_like(x)
        ws = torch.empty(ops.llama_block_workspace_bytes(Bb, Sb, dm, Hb, Hb, 128, F), dtype=torch.uint8, device=dev)
        if a.case == "block":
            fn = lambda: ops.llama_block_fwd(x, n1, wqkv, wo, n2, wg, wu, wd, Bb, Sb, Hb, Hb, out=out, workspace=ws)
        else:
            wqkv_f, wg_f, wu_f = ops.llama_block_fold_weights(n1, wqkv, n2, wg, wu)
            fn = lambda: ops.llama_block_fwd_folded(x, wqkv_f, wo, wg_f, wu_f, wd, Bb, Sb, Hb, Hb, out=out,
                                                    workspace=ws)
        flops = (2.0 * T * dm * 3 * dm + 2.0 * T * dm * dm + 2.0 * T * dm * 2 * F + 2.0 * T * F * dm
                 + 2.0 * Bb * Hb * Sb * Sb * 128)
        kname = "k_gemm_bf16_tc"
    elif a.case == "swiglu_fwd":
        T, dm, F = a.tokens // 2, a.width, a.n
        x = torch.randn(T, dm, device=dev).bfloat16()
        wg, wu = ((torch.randn(dm, F, device=dev) * 0.02).bfloat16() for _ in range(2))
        wd = (torch.randn(F, dm, device=dev) * 0.02).bfloat16()
        fn = lambda: ops.swiglu_fwd(x, wg, wu, wd)  # gate/up GEMM with the SwiGLU epilogue, then down
        flops, kname = 6.0 * T * dm * F, "k_gemm_bf16_tc"
    elif a.case == "swiglu_bwd":
        T, dm, F = a.tokens // 2, a.width, a.n
        x = torch.randn(T, dm, device=dev).bfloat16()
        dy = torch.randn(T, dm, device=dev).bfloat16()
        wg, wu = ((torch.randn(dm, F, device=dev) * 0.02).bfloat16() for _ in range(2))
        wd = (torch.randn(F, dm, device=dev) * 0.02).bfloat16()
        fn = lambda: ops.swiglu_bwd(dy, x, wg, wu, wd)
        flops, kname = 12.0 * T * dm * F, "k_gemm_bf16_tc"  # dWd, dh, dWg, dWu, dx (recompute not counted)
    else:
        A = (torch.rand(a.m, a.k, device=dev) * 2 - 1).bfloat16()
        Bm = (torch.rand(a.k, a.n, device=dev) * 2 - 1).bfloat16()
        C = torch.empty(a.m, a.n, device=dev, dtype=torch.bfloat16)
        fn, flops, kname = (lambda: ops.matmul_fwd(A, Bm, out=C)), 2.0 * a.m * a.n * a.k, "k_gemm_bf16_tc"

    for _ in range(a.warmup):
        fn()
    torch.cuda.synchronize()
    ops.profile_reset()
    ops.profile_enable(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ops.profile_enable(False)
    ms, n = ops.profile_read(kname)
    kms = ms / max(n, 1)
    call_ms = e0.elapsed_time(e1) / a.iters
    if a.case.startswith(("swiglu", "block")):  # several launches per call: the whole call
        print(f"{a.case}: {call_ms:.4f} ms/call {flops / (call_ms * 1e-3) / 1e12:.1f} TFLOP/s algorithmic "
              f"({n // max(a.iters, 1)} GEMM launches per call, {kms:.4f} ms each on average)", flush=True)
    else:
        print(f"{a.case}: {kname} {kms:.4f} ms/launch {flops / (kms * 1e-3) / 1e12:.1f} TFLOP/s; "
              f"call {call_ms:.4f} ms", flush=True)
    if a.case.startswith("attn_bwd"):  # the dQ kernel of the same calls: 3 of the backward's 5 products
        qms, qn = ops.profile_read("k_attn_bwd_dq")
        qms /= max(qn, 1)
        print(f"{a.case}: k_attn_bwd_dq {qms:.4f} ms/launch {0.6 * flops / (qms * 1e-3) / 1e12:.1f} TFLOP/s executed",
              flush=True)
    ops.device_status(0)
    return 0


def _hbm_case(a, torch, ops, dev):
    T, W = a.tokens, a.width
    x = torch.randn(T, W, device=dev).bfloat16()
    dy = torch.randn(T, W, device=dev).bfloat16()
    g = torch.randn(W, device=dev).bfloat16()
    b = torch.randn(W, device=dev).bfloat16()
    out, mean, invstd = ops.layernorm_fwd(x, g, b)
    if a.case == "layernorm_fwd":
        fn, nbytes = (lambda: ops.layernorm_fwd(x, g, b)), 2.0 * T * W * 2 + 8.0 * T
    elif a.case == "rmsnorm_fwd":
        fn, nbytes = (lambda: ops.rmsnorm_fwd(x, g)), 2.0 * T * W * 2 + 4.0 * T
    elif a.case == "rmsnorm_bwd":
        _, rms = ops.rmsnorm_fwd(x, g)
        fn, nbytes = (lambda: ops.rmsnorm_bwd(dy, x, rms, g)), 3.0 * T * W * 2 + 4.0 * T
    elif a.case == "residual_add":  # a, b in, out: bf16
        fn, nbytes = (lambda: ops.residual_add(x, dy)), 3.0 * T * W * 2
    elif a.case == "cast_f32_bf16":  # f32 in, bf16 out with the reference's rounding
        xf = x.float()
        fn, nbytes = (lambda: ops.cast(xf, 2)), 6.0 * T * W
    elif a.case == "dropout_fwd":  # x in, out and the mask out: bf16
        fn, nbytes = (lambda: ops.dropout_fwd(x, 0.1, 7)), 3.0 * T * W * 2
    else:
        fn, nbytes = (lambda: ops.layernorm_bwd(dy, x, mean, invstd, g)), 3.0 * T * W * 2 + 8.0 * T
    for _ in range(a.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.iters
    print(f"{a.case}: tokens {T} width {W} {ms:.4f} ms/call {nbytes / (ms * 1e-3) / 1e9:.0f} GB/s algorithmic",
          flush=True)
    ops.device_status(0)
    return 0


if __name__ == "__main__":
    sys.exit(main())
