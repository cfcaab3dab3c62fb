"""Small, self-contained launches of one hot-path kernel, for ncu captures and quick timing.

    python -m beacon_b200.profile_cases attn_bwd --heads 32
    python -m beacon_b200.profile_cases attn_fwd --heads 32
    python -m beacon_b200.profile_cases gemm --m 4096 --n 4096 --k 4096

Each case runs `--warmup` untimed launches and then `--iters` launches timed with
CUDA events, printing the per-launch time and TFLOP/s (algorithmic FLOPs: causal
attention forward 2*H*S^2*D, backward 2.5x that; GEMM 2*M*N*K).  Sizes default to
a case larger than the 126 MB L2 but a few hundred MB on the device, the size an
ncu capture of a single launch (-k <kernel> -s <warmup launches> -c 1) should use.
"""
from __future__ import annotations

import argparse
import sys


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["attn_fwd", "attn_bwd", "attn_bwd_recompute", "gemm"])
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=0)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--dim", type=int, default=128)
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args(argv)

    import torch

    from . import ops

    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    if a.case.startswith("attn"):
        H, S, D = a.heads, a.seq, a.dim
        Hkv = a.kv_heads or H
        q = torch.randn(1, H, S, D, device=dev).bfloat16()
        k = torch.randn(1, Hkv, S, D, device=dev).bfloat16()
        v = torch.randn(1, Hkv, S, D, device=dev).bfloat16()
        do = torch.randn(1, H, S, D, device=dev).bfloat16()
        out, lse = ops.attention_fwd(q, k, v)
        fwd = 2.0 * H * S * S * D
        if a.case == "attn_fwd":
            fn, flops, kname = (lambda: ops.attention_fwd(q, k, v, out=out, lse=lse)), fwd, "k_attn_fwd_tc"
        elif a.case == "attn_bwd":
            fn, flops, kname = (lambda: ops.attention_bwd(do, q, k, v, lse, out=out)), 2.5 * fwd, "k_attn_bwd_dkdv"
        else:
            fn, flops, kname = (lambda: ops.attention_bwd(do, q, k, v, lse)), 2.5 * fwd, "k_attn_bwd_dkdv"
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
    print(f"{a.case}: {kname} {kms:.4f} ms/launch {flops / (kms * 1e-3) / 1e12:.1f} TFLOP/s; "
          f"call {e0.elapsed_time(e1) / a.iters:.4f} ms", flush=True)
    if a.case.startswith("attn_bwd"):  # the dQ kernel of the same calls: 3 of the backward's 5 products
        qms, qn = ops.profile_read("k_attn_bwd_dq")
        qms /= max(qn, 1)
        print(f"{a.case}: k_attn_bwd_dq {qms:.4f} ms/launch {0.6 * flops / (qms * 1e-3) / 1e12:.1f} TFLOP/s executed",
              flush=True)
    ops.device_status(0)
    return 0


if __name__ == "__main__":
    sys.exit(main())
