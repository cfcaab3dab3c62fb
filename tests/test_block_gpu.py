"""Pre-norm Llama block forward (beacon_llama_block_fwd) through the C ABI against the
oracle's composition of the reference operators it fuses: rmsnorm_fwd (norm.rs:19-31),
linear_fwd (matmul.rs:46-58), attention_fwd (attention.rs:21-40), residual_add
(elementwise.rs:47-55) and swiglu_fwd (mlp.rs:12-29)."""
import numpy as np
import pytest

import oracle as O
from helpers import BF16_TOL, as_bf16, normal, rel_err, to_dev, to_np

pytestmark = pytest.mark.gpu


def _weights(dm, Hq, Hkv, D, F, seed, std):
    r = as_bf16
    return dict(
        attn_norm=r(1.0 + 0.1 * normal((dm,), seed)),
        w_qkv=r(normal((dm, (Hq + 2 * Hkv) * D), seed + 1, std=std)),
        w_o=r(normal((Hq * D, dm), seed + 2, std=std)),
        ffn_norm=r(1.0 + 0.1 * normal((dm,), seed + 3)),
        w_gate=r(normal((dm, F), seed + 4, std=std)),
        w_up=r(normal((dm, F), seed + 5, std=std)),
        w_down=r(normal((F, dm), seed + 6, std=std)),
    )


@pytest.mark.parametrize("Bt,S,dm,Hq,Hkv,D,F", [
    (2, 200, 256, 4, 2, 64, 384),     # GQA, ragged sequence (not a multiple of 128)
    (1, 256, 256, 2, 2, 128, 512),    # head_dim 128, multi-head
    (1, 512, 1024, 8, 2, 128, 2816),  # the Llama proportions at small scale
])
def test_llama_block_fwd(Bt, S, dm, Hq, Hkv, D, F):
    import torch
    from beacon_b200 import ops
    w = _weights(dm, Hq, Hkv, D, F, 40, std=0.05)
    x = as_bf16(normal((Bt * S, dm), 3))
    ref = O.llama_block_fwd(x, w["attn_norm"], w["w_qkv"], w["w_o"], w["ffn_norm"], w["w_gate"], w["w_up"],
                            w["w_down"], Bt, S, Hq, Hkv)
    dev = {k: to_dev(v, torch.bfloat16) for k, v in w.items()}
    out = ops.llama_block_fwd(to_dev(x, torch.bfloat16), dev["attn_norm"], dev["w_qkv"], dev["w_o"],
                              dev["ffn_norm"], dev["w_gate"], dev["w_up"], dev["w_down"], Bt, S, Hq, Hkv)
    torch.cuda.synchronize()
    got = to_np(out)
    assert np.isfinite(got).all()
    assert rel_err(got, ref) <= BF16_TOL
    # the block's own contribution (out - x) is checked too, so that the residual
    # stream cannot hide an error in the attention or MLP branches
    assert rel_err(got - x, ref - x) <= BF16_TOL


def test_llama_block_fwd_caller_workspace_and_errors():
    import torch
    from beacon_b200 import errors, ops
    Bt, S, dm, Hq, Hkv, D, F = 1, 128, 128, 2, 1, 64, 256
    w = {k: to_dev(v, torch.bfloat16) for k, v in _weights(dm, Hq, Hkv, D, F, 50, std=0.05).items()}
    x = to_dev(as_bf16(normal((Bt * S, dm), 5)), torch.bfloat16)
    need = ops.llama_block_workspace_bytes(Bt, S, dm, Hq, Hkv, D, F)
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    a = ops.llama_block_fwd(x, w["attn_norm"], w["w_qkv"], w["w_o"], w["ffn_norm"], w["w_gate"], w["w_up"],
                            w["w_down"], Bt, S, Hq, Hkv, workspace=ws)
    b = ops.llama_block_fwd(x, w["attn_norm"], w["w_qkv"], w["w_o"], w["ffn_norm"], w["w_gate"], w["w_up"],
                            w["w_down"], Bt, S, Hq, Hkv)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    with pytest.raises(errors.LaunchError):
        ops.llama_block_fwd(x, w["attn_norm"], w["w_qkv"], w["w_o"], w["ffn_norm"], w["w_gate"], w["w_up"],
                            w["w_down"], Bt, S, Hq, Hkv, workspace=ws[: need // 2])


@pytest.mark.parametrize("Bt,S,dm,Hq,Hkv,D,F", [
    (2, 200, 256, 4, 2, 64, 384),
    (1, 512, 1024, 8, 2, 128, 2816),
])
def test_llama_block_fwd_folded(Bt, S, dm, Hq, Hkv, D, F):
    """The block with both RMSNorms folded into the GEMMs after them (gains folded into the
    weights, statistics as row scales, the second statistic summed in the output
    projection's epilogue) against the operator-by-operator oracle and the unfused block."""
    import torch
    from beacon_b200 import ops
    w = _weights(dm, Hq, Hkv, D, F, 40, std=0.05)
    x = as_bf16(normal((Bt * S, dm), 3))
    ref = O.llama_block_fwd(x, w["attn_norm"], w["w_qkv"], w["w_o"], w["ffn_norm"], w["w_gate"], w["w_up"],
                            w["w_down"], Bt, S, Hq, Hkv)
    dev = {k: to_dev(v, torch.bfloat16) for k, v in w.items()}
    xd = to_dev(x, torch.bfloat16)
    wq, wg, wu = ops.llama_block_fold_weights(dev["attn_norm"], dev["w_qkv"], dev["ffn_norm"], dev["w_gate"],
                                              dev["w_up"])
    out = ops.llama_block_fwd_folded(xd, wq, dev["w_o"], wg, wu, dev["w_down"], Bt, S, Hq, Hkv)
    unfused = ops.llama_block_fwd(xd, dev["attn_norm"], dev["w_qkv"], dev["w_o"], dev["ffn_norm"], dev["w_gate"],
                                  dev["w_up"], dev["w_down"], Bt, S, Hq, Hkv)
    torch.cuda.synchronize()
    got = to_np(out)
    assert np.isfinite(got).all()
    assert rel_err(got, ref) <= BF16_TOL
    assert rel_err(got - x, ref - x) <= BF16_TOL
    assert rel_err(got - x, to_np(unfused) - x) <= BF16_TOL
