"""Shared helpers for the parity tests: seeded inputs from the oracle's
SplitMix64 streams, bf16 rounding by the reference's rule, device transfer and
the norm-wise relative error the tolerances are stated in."""
from __future__ import annotations

import numpy as np

import oracle as O

BF16_TOL = 2e-2   # bf16 inputs, fp32 accumulation (gradients included)
F32_TOL = 1e-5    # float32 path


def normal(shape, seed, std=1.0, offset=0):
    return O.normal(shape, seed, std=std, offset=offset)


def uniform(shape, seed, lo=-1.0, hi=1.0, offset=0):
    return O.uniform(shape, seed, lo, hi, offset=offset)


def as_bf16(x):
    """Round a float32 array to bf16 values (reference rule), still float32."""
    return O.round_bf16(x)


def to_dev(x, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dtype)
    return t.cuda()


def to_np(t):
    return t.detach().float().cpu().numpy()


rel_err = O.rel_err
