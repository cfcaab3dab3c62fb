"""Embedding lookup and dropout (crates/beacon-cuda/src/elementwise.rs:67-118) through the
C ABI against the oracle: the lookup and its accumulating backward, an index beyond the
table (zero row, nothing read, a fault word recorded), and the counter-based dropout mask
bit for bit."""
import numpy as np
import pytest

import oracle as O
from helpers import BF16_TOL, F32_TOL, as_bf16, normal, rel_err, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("vocab,dim,tokens,dt", [(1000, 256, 4096, "bf16"), (50, 100, 333, "f32"),
                                                 (32000, 4096, 2048, "bf16")])
def test_embedding_lookup_and_backward(vocab, dim, tokens, dt):
    import torch
    from beacon_b200 import ops
    tdt = torch.bfloat16 if dt == "bf16" else torch.float32
    r = as_bf16 if dt == "bf16" else (lambda a: a)
    table = r(normal((vocab, dim), 51))
    idx = np.random.default_rng(5).integers(0, vocab, tokens).astype(np.int32)
    idx[:7] = idx[7]  # repeated rows: their gradients add up
    it = torch.from_numpy(idx).cuda()
    out = ops.embedding_lookup(to_dev(table, tdt), it)
    assert np.array_equal(to_np(out), O.embedding_lookup_fwd(table, idx))  # a copy: bit-exact
    d_out = r(normal((tokens, dim), 52))
    d_table0 = r(normal((vocab, dim), 53, std=0.1))
    dt_dev = to_dev(d_table0, tdt)
    ops.embedding_backward(dt_dev, to_dev(d_out, tdt), it)
    ref = O.embedding_lookup_bwd(d_table0, d_out, idx)
    tol = BF16_TOL if dt == "bf16" else F32_TOL
    assert rel_err(to_np(dt_dev), ref) <= tol
    assert ops.device_status(0)[0] == 0


def test_embedding_index_beyond_the_table():
    """Index 70 in a 64-row table: that output row is zeros, the other rows are looked up,
    and the fault word holds code 3; the backward skips the token."""
    import torch
    from beacon_b200 import _lib, ops
    from beacon_b200.errors import LaunchError
    ops.device_status(0)
    table = normal((64, 32), 54)
    idx = np.array([3, 70, 5, 63], dtype=np.int32)
    out = to_np(ops.embedding_lookup(to_dev(table, torch.float32), torch.from_numpy(idx).cuda()))
    assert np.array_equal(out, O.embedding_lookup_fwd(table, idx)) and not out[1].any()
    d = torch.zeros(64, 32, device="cuda")
    ops.embedding_backward(d, torch.ones(4, 32, device="cuda"), torch.from_numpy(idx).cuda())
    torch.cuda.synchronize()
    assert float(d.sum()) == 3 * 32.0
    with pytest.raises(LaunchError):
        ops.device_status(0)
    assert "fault code 3" in _lib.last_error()


@pytest.mark.parametrize("n,p,dt", [(1 << 20, 0.1, "bf16"), (1000003, 0.5, "f32"), (4096, 0.0, "bf16"),
                                    (4096, 1.0, "f32")])
def test_dropout_mask_is_bit_exact(n, p, dt):
    import torch
    from beacon_b200 import ops
    tdt = torch.bfloat16 if dt == "bf16" else torch.float32
    r = as_bf16 if dt == "bf16" else (lambda a: a)
    x = r(normal((n,), 55))
    out, mask = ops.dropout_fwd(to_dev(x, tdt), p, seed=1234)
    rout, rmask = O.dropout_fwd(x, p, 1234, bf16=(dt == "bf16"))
    assert np.array_equal(to_np(mask), rmask)
    assert np.array_equal(to_np(out), rout)
    dy = r(normal((n,), 56))
    d_in = ops.dropout_bwd(to_dev(dy, tdt), mask)
    ref = dy * rmask
    assert np.array_equal(to_np(d_in), as_bf16(ref) if dt == "bf16" else ref)


def test_dropout_scalar_path_for_unaligned_input():
    """An input that is not 16-byte aligned takes the one-element-per-thread kernels, with
    the same draw: masks and outputs bit-exact as on the vectorised path."""
    import torch
    from beacon_b200 import ops
    x = as_bf16(normal((5001,), 57))
    dev = to_dev(np.concatenate([np.zeros(1, dtype=np.float32), x]), torch.bfloat16)[1:]  # 2-byte offset
    assert dev.data_ptr() % 16 != 0
    out, mask = ops.dropout_fwd(dev, 0.3, seed=99)
    rout, rmask = O.dropout_fwd(x, 0.3, 99, bf16=True)
    assert np.array_equal(to_np(mask), rmask)
    assert np.array_equal(to_np(out), rout)
