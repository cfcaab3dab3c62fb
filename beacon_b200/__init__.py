"""beacon_b200 -- B200-native (sm_100a) kernels for beacon's transformer hot path.

Causal attention forward/backward, the bf16 GEMM family with fused epilogues,
RMSNorm and the SwiGLU MLP, behind the kernel IDs of the reference's
``beacon-cuda`` launcher traits and ``beacon-adjoint-table`` entries.

Submodules:
  _lib         ctypes binding of libbeacon_cuda.so (include/beacon_cuda.h)
  errors       LaunchError variants (crates/beacon-cuda/src/error.rs)
  launcher     KernelLauncher / typed traits / arena Launcher mirror
  adjoint_table the reference's ADJOINT_TABLE (crates/beacon-adjoint-table)
  ops          torch-tensor front end used by tests and bench.py
"""
from . import _lib, errors  # noqa: F401

__all__ = ["_lib", "errors"]
