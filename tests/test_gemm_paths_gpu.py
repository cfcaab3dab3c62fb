"""Every GEMM kernel shape -- 1-SM 128-row tiles, 2-SM (cta_group::2) 256x256 pair tiles and
256x128 pair tiles -- on every operand layout and epilogue, forced through BEACON_GEMM_PATH
in a child process so the shape heuristic cannot hide any of them."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CHILD = r'''
import sys
sys.path.insert(0, sys.argv[1])
import numpy as np, torch
import oracle as O
from helpers import as_bf16, uniform, normal, to_dev, to_np, rel_err, BF16_TOL
from beacon_b200 import ops
bf = torch.bfloat16
fails = []
def chk(name, got, ref):
    e = rel_err(to_np(got), ref)
    if not e <= BF16_TOL:
        fails.append((name, e))
for (m, k, n) in [(512, 256, 512), (300, 136, 520), (256, 64, 256)]:
    a = as_bf16(uniform((m, k), 1)); b = as_bf16(uniform((k, n), 2)); dy = as_bf16(uniform((m, n), 3))
    chk(f"fwd{m}", ops.matmul_fwd(to_dev(a, bf), to_dev(b, bf)), O.matmul_fwd(a, b))
    dl, dr = ops.matmul_bwd(to_dev(dy, bf), to_dev(a, bf), to_dev(b, bf))
    rl, rr = O.matmul_bwd(dy, a, b)
    chk(f"dlhs{m}", dl, rl); chk(f"drhs{m}", dr, rr)
    bias = as_bf16(normal((n,), 4))
    chk(f"linear{m}", ops.linear_fwd(to_dev(a, bf), to_dev(b, bf), to_dev(bias, bf)), O.linear_fwd(a, b, bias))
x = as_bf16(normal((384, 256), 5)); wg = as_bf16(normal((256, 384), 6, std=0.05)); wu = as_bf16(normal((256, 384), 7, std=0.05))
wd = as_bf16(normal((384, 256), 8, std=0.05))
chk("swiglu", ops.swiglu_fwd(*[to_dev(t, bf) for t in (x, wg, wu, wd)]), O.swiglu_fwd(x, wg, wu, wd))
ops.device_status(0)
print("FAILS", fails)
sys.exit(1 if fails else 0)
'''


@pytest.mark.parametrize("path", ["1sm", "2sm", "2sm128"])
def test_gemm_kernel_path(path):
    env = dict(os.environ, BEACON_GEMM_PATH=path, PYTHONPATH=HERE + os.pathsep + os.path.dirname(HERE))
    r = subprocess.run([sys.executable, "-c", CHILD, HERE], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
