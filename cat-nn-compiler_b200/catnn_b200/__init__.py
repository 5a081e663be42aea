"""catnn_b200 — B200 (sm_100a) execution backend for catnn's hot path.

Layers:
- ``libcatnn_b200.so`` (csrc/): the CUDA kernels and the C ABI of
  include/catnn_b200.h — the drop-in boundary a catnn DeviceHandler binds.
- ``ops``: one Python function per C-ABI entry point over device tensors.
- ``ir``: the reference's operator boundary (OpenOp / IrNode / eval /
  adjoint_of / DeviceHandler) dispatching to those kernels.
- ``train``: the training steps (MLP, Mixtral-style MoE) built on them.
"""
from . import errors, ops  # noqa: F401
from ._lib import LIB_PATH, load  # noqa: F401

__all__ = ["errors", "ops", "load", "LIB_PATH"]
