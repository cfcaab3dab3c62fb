"""The reference's adjoint registry (crates/beacon-adjoint-table/src/lib.rs:3-155), unchanged.

Each entry names the forward and backward launcher (kernel ID) of an op, the
tensors its backward needs (Store: kept from the forward; Recompute: rebuilt in
the backward) and the gradients it produces.  The kernel IDs the C ABI exports
must equal these strings; tests/test_launcher_cpu.py checks that, as the
reference's table_consistency test does (crates/beacon-cuda/src/lib.rs:29-63).
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum


class SaveMode(Enum):
    STORE = "Store"
    RECOMPUTE = "Recompute"


@dataclass(frozen=True)
class SavedSpec:
    name: str
    mode: SaveMode


@dataclass(frozen=True)
class AdjointEntry:
    op: str
    forward_launcher: str
    backward_launcher: str
    saved: tuple
    input_grads: tuple
    param_grads: tuple

    def num_saved(self) -> int:
        return len(self.saved)

    def num_input_grads(self) -> int:
        return len(self.input_grads)

    def num_param_grads(self) -> int:
        return len(self.param_grads)


def _stored(n):
    return SavedSpec(n, SaveMode.STORE)


def _recomputed(n):
    return SavedSpec(n, SaveMode.RECOMPUTE)


# lib.rs:53-116
ADJOINT_TABLE = (
    AdjointEntry("matmul", "matmul_fwd", "matmul_bwd", (_stored("lhs"), _stored("rhs")), ("dlhs", "drhs"), ()),
    AdjointEntry("linear", "linear_fwd", "linear_bwd", (_stored("x"), _stored("weight")), ("dx",),
                 ("dweight", "dbias")),
    AdjointEntry("rmsnorm", "rmsnorm_adjoint_fwd", "rmsnorm_adjoint_bwd", (_stored("x"), _stored("rms")), ("dx",),
                 ("dweight",)),
    AdjointEntry("layernorm", "layernorm_adjoint_fwd", "layernorm_adjoint_bwd",
                 (_stored("x"), _stored("mean"), _stored("invstd")), ("dx",), ("dweight", "dbias")),
    AdjointEntry("flash_attention", "attention_adjoint_fwd", "attention_adjoint_bwd",
                 (_stored("q"), _stored("k"), _stored("v"), _stored("lse"), _recomputed("scores")),
                 ("dq", "dk", "dv"), ()),
    AdjointEntry("swiglu_mlp", "swiglu_adjoint_fwd", "swiglu_adjoint_bwd",
                 (_stored("x"), _recomputed("gate"), _recomputed("up")), ("dx",),
                 ("dgate_proj", "dup_proj", "ddown_proj")),
    AdjointEntry("residual_add", "residual_add_fwd", "residual_add_bwd", (), ("dx", "dy"), ()),
)


def lookup(op: str):
    """lib.rs:134-143"""
    for e in ADJOINT_TABLE:
        if e.op == op:
            return e
    return None


def is_differentiable(op: str) -> bool:
    return lookup(op) is not None


def op_names():
    return [e.op for e in ADJOINT_TABLE]
