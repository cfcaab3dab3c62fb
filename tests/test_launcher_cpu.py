"""The launch layer mirror: the reference's own unit tests for
crates/beacon-cuda (routing through a fake launcher, grids, LaunchParams
validation, the kernel-ID / adjoint-table consistency check) and
crates/beacon-adjoint-table, restated against beacon_b200.launcher."""
import pytest

from beacon_b200 import adjoint_table as T
from beacon_b200.errors import InvalidLaunchConfig
from beacon_b200.launcher import (Access, CastKind, Dim3, KernelArg, KernelId, LaunchParams, Recorder,
                                  MAX_DYNAMIC_SMEM_BYTES, MAX_THREADS_PER_BLOCK, attention_grid, elementwise_grid,
                                  kid)


def a():
    return KernelArg.read(0, 256)


def test_attention_grid_tiles_q():          # attention.rs:78-83
    g = attention_grid(4, 12, 512)
    assert (g.grid.x, g.grid.y) == (48, 8)


def test_attention_routes():                # attention.rs:85-95
    r = Recorder()
    r.attention_fwd(a(), a(), a(), a(), a(), 4, 12, 512, 64, True)
    r.attention_bwd(a(), a(), a(), a(), a(), a(), a(), a(), 4, 12, 512, 64, True)
    assert r.calls() == [("attention_adjoint_fwd", 5), ("attention_adjoint_bwd", 8)]


def test_matmul_and_linear_route():         # matmul.rs:92-108
    r = Recorder()
    r.matmul_fwd(a(), a(), a(), 2048, 768, 3072)
    r.matmul_bwd(a(), a(), a(), a(), a(), 2048, 768, 3072)
    r.linear_fwd(a(), a(), a(), a(), 2048, 768, 50257)
    r.linear_bwd(a(), a(), a(), a(), a(), a(), 2048, 768, 50257)
    assert r.calls() == [("matmul_fwd", 3), ("matmul_bwd", 5), ("linear_fwd", 4), ("linear_bwd", 6)]


def test_norm_routes():                     # norm.rs:108-128
    r = Recorder()
    r.rmsnorm_fwd(a(), a(), a(), a(), 512, 768)
    r.rmsnorm_bwd(a(), a(), a(), a(), a(), a(), 512, 768)
    r.layernorm_fwd(a(), a(), a(), a(), a(), a(), 512, 768)
    r.layernorm_bwd(a(), a(), a(), a(), a(), a(), a(), a(), 512, 768)
    assert r.calls() == [("rmsnorm_adjoint_fwd", 4), ("rmsnorm_adjoint_bwd", 6), ("layernorm_adjoint_fwd", 6),
                         ("layernorm_adjoint_bwd", 8)]


def test_swiglu_routes():                   # mlp.rs:66-76
    r = Recorder()
    r.swiglu_fwd(a(), a(), a(), a(), a(), 2048, 768, 3072)
    r.swiglu_bwd(a(), a(), a(), a(), a(), a(), a(), a(), a(), 2048, 768, 3072)
    assert r.calls() == [("swiglu_adjoint_fwd", 5), ("swiglu_adjoint_bwd", 9)]


def test_elementwise_families_route():      # elementwise.rs:178-204
    r = Recorder()
    r.residual_add(KernelArg.write(0, 256), a(), a(), 64)
    r.residual_add_backward(KernelArg.read_write(0, 256), KernelArg.read_write(256, 256), a(), 64)
    r.embedding_lookup(KernelArg.write(0, 256), a(), a(), 8, 32)
    r.embedding_backward(KernelArg.read_write(0, 256), a(), a(), 8, 32)
    r.dropout_forward(KernelArg.write(0, 256), a(), KernelArg.write(256, 256), 64, 0.0, 7)
    r.dropout_backward(KernelArg.write(0, 256), a(), a(), 64)
    r.cast(KernelArg.write(0, 256), a(), 64, CastKind.F32_TO_F8E4M3)
    assert r.calls() == [("residual_add_fwd", 3), ("residual_add_bwd", 3), ("embedding_lookup_fwd", 3),
                         ("embedding_lookup_bwd", 3), ("dropout_fwd", 3), ("dropout_bwd", 3),
                         ("cast_f32_to_fp8e4m3", 2)]


def test_grid_is_nonzero_even_for_zero_elements():
    assert elementwise_grid(0).grid.total() >= 1
    assert elementwise_grid(513).grid.x == 3


def test_cast_kind_maps_to_kernels():
    assert CastKind.F32_TO_F8E4M3.kernel() == kid.CAST_F32_TO_FP8E4M3
    assert CastKind.BF16_TO_F32.kernel() == kid.CAST_BF16_TO_F32


def test_kernel_arg_access_modes():         # launcher.rs:100-104
    assert KernelArg.read(0, 16).access == Access.READ
    assert KernelArg.write(16, 32).access == Access.WRITE
    assert KernelArg.read_write(48, 8).access == Access.READ_WRITE
    assert KernelId("rmsnorm_adjoint_fwd").name() == "rmsnorm_adjoint_fwd"


def test_launch_params():                   # launch.rs:100-148
    assert Dim3.of(8) == Dim3(8, 1, 1)
    assert Dim3.of((4, 4)) == Dim3(4, 4, 1)
    assert Dim3(2, 3, 4).total() == 24
    p = LaunchParams.new(128, 256)
    assert p.shared_mem_bytes == 0 and p.total_threads() == 128 * 256
    LaunchParams.new((32, 8, 1), (64, 16, 1)).with_shared_mem(100 * 1024).validate()
    with pytest.raises(InvalidLaunchConfig):
        LaunchParams.new(1, (32, 33, 1)).validate()
    with pytest.raises(InvalidLaunchConfig):
        LaunchParams.new(1, 256).with_shared_mem(MAX_DYNAMIC_SMEM_BYTES + 1).validate()
    with pytest.raises(InvalidLaunchConfig):
        LaunchParams.new(0, 256).validate()
    assert MAX_THREADS_PER_BLOCK == 1024


def test_recorder_propagates_invalid_config():
    with pytest.raises(InvalidLaunchConfig):
        Recorder().launch(KernelId("x"), LaunchParams.new(0, 64), [KernelArg.read(0, 1)])


def test_launcher_kernel_ids_match_adjoint_table():   # crates/beacon-cuda/src/lib.rs:29-63
    pairs = [("matmul", kid.MATMUL_FWD, kid.MATMUL_BWD), ("linear", kid.LINEAR_FWD, kid.LINEAR_BWD),
             ("rmsnorm", kid.RMSNORM_FWD, kid.RMSNORM_BWD), ("layernorm", kid.LAYERNORM_FWD, kid.LAYERNORM_BWD),
             ("flash_attention", kid.ATTENTION_FWD, kid.ATTENTION_BWD), ("swiglu_mlp", kid.SWIGLU_FWD, kid.SWIGLU_BWD),
             ("residual_add", kid.RESIDUAL_ADD_FWD, kid.RESIDUAL_ADD_BWD)]
    for op, fwd, bwd in pairs:
        e = T.lookup(op)
        assert e is not None, op
        assert fwd.name() == e.forward_launcher
        assert bwd.name() == e.backward_launcher


def test_adjoint_table():                   # crates/beacon-adjoint-table/src/lib.rs:157-219
    for op in ["matmul", "linear", "rmsnorm", "layernorm", "flash_attention", "swiglu_mlp", "residual_add"]:
        e = T.lookup(op)
        assert e.op == op and e.forward_launcher and e.backward_launcher
    assert T.lookup("not_an_op") is None and not T.is_differentiable("conv2d")
    names = T.op_names()
    assert len(set(names)) == len(names) == 7
    for e in T.ADJOINT_TABLE:
        assert e.forward_launcher != e.backward_launcher
    fa = T.lookup("flash_attention")
    modes = {s.name: s.mode for s in fa.saved}
    assert modes["scores"] == T.SaveMode.RECOMPUTE and modes["q"] == T.SaveMode.STORE
    assert fa.input_grads == ("dq", "dk", "dv")
