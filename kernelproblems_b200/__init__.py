"""B200 (sm_100a) kernels for the memory-bound Llama training-graph fragments
of SherlockNoMad/KernelProblems: RMSNorm forward/backward, residual add +
RMSNorm, token-embedding gather/scatter-add, and RoPE forward/backward.

Layers:
  include/frag.h, csrc/*.cu  the C ABI (libfrag.so) and its CUDA kernels
  _lib                       ctypes binding; raises if libfrag.so is missing
  ops                        functional API on torch CUDA tensors
  problems                   drop-in `kernel_function`s, one per reference problem
  sharding                   row-sharded / vocab-parallel multi-GPU wrappers
  configs                    workload configurations, seeded inputs, byte model
"""
from . import _lib, configs, ops  # noqa: F401
from ._lib import FragError  # noqa: F401
from .ops import (  # noqa: F401
    add_rmsnorm_fwd,
    check_status,
    dw_reduce,
    embedding_bwd,
    embedding_fwd,
    embedding_rmsnorm_fwd,
    rmsnorm_bwd,
    rmsnorm_fwd,
    rope,
)

__version__ = "0.1.0"
