"""Multi-GPU wrappers: one process per GPU, torch.distributed (NCCL) plumbing.

Rows (tokens) are data-parallel: every rank runs the fragment kernels on its
own rows with no communication.  Two fragments have a real exchange step:

  * RMSNorm backward: each rank's fp32 dweight covers only its rows; the
    global dweight is the sum over ranks (``rmsnorm_bwd_dp``).  By default the
    per-rank vectors are all-gathered and added in rank order by the same
    fixed-order kernel used inside a rank, so every rank gets bitwise the same
    dweight regardless of NCCL's reduction algorithm; ``exact_order=False``
    uses a plain NCCL all-reduce instead.  The forward recomputed inside the
    backward (``rmsnorm_fwd_bwd_dp``) exchanges its dweight the same way.
  * Vocab-parallel embedding: rank r owns table rows [lo_r, hi_r).  Forward:
    every rank gathers its own rows for the (replicated) ids, writing zero rows
    for ids it does not own, then the outputs are all-reduced; exactly one rank
    contributes a non-zero row per token, so the sum is the bit-exact row (a
    -0.0 table entry comes back as +0.0).  Backward: each rank writes its own
    shard of the fp32 table gradient from the replicated ids and gradients,
    with no communication.

The kernels default to ``kernelproblems_b200.ops``; the ``*_fn`` arguments
exist so the host logic can be exercised on CPU ranks (gloo) in tests.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from . import ops
from .configs import Rows, shard_rows

__all__ = [
    "shard_rows",
    "local_rows",
    "rmsnorm_bwd_dp",
    "add_rmsnorm_bwd_dp",
    "rmsnorm_fwd_bwd_dp",
    "embedding_fwd_vocab_parallel",
    "embedding_bwd_vocab_parallel",
    "vocab_shard",
]


def _world(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def local_rows(total: int, group=None) -> Rows:
    """This rank's contiguous row range of a `total`-row tensor."""
    w, r = _world(group)
    return shard_rows(total, w, r)


def vocab_shard(vocab: int, group=None) -> Rows:
    """This rank's contiguous vocab range [lo, hi)."""
    return local_rows(vocab, group)


def _sum_over_ranks(dw: torch.Tensor, group, exact_order: bool,
                    reduce_fn: Callable[[torch.Tensor], torch.Tensor]) -> torch.Tensor:
    world, _ = _world(group)
    if world == 1:
        return dw
    if not exact_order:
        dist.all_reduce(dw, op=dist.ReduceOp.SUM, group=group)
        return dw
    parts = torch.empty(world * dw.numel(), dtype=dw.dtype, device=dw.device)
    dist.all_gather_into_tensor(parts, dw.contiguous(), group=group)
    return reduce_fn(parts.view(world, dw.numel()))


def rmsnorm_bwd_dp(dy: torch.Tensor, x: torch.Tensor, rstd: torch.Tensor | None,
                   weight: torch.Tensor, *, eps: float = 1e-6, group=None,
                   exact_order: bool = True, dy2: torch.Tensor | None = None,
                   dres: torch.Tensor | None = None,
                   bwd_fn: Callable | None = None,
                   reduce_fn: Callable | None = None):
    """RMSNorm backward on this rank's rows; dweight summed over all ranks.

    Returns (dx for the local rows, global fp32 dweight)."""
    bwd_fn = bwd_fn or ops.rmsnorm_bwd
    reduce_fn = reduce_fn or ops.dw_reduce
    dx, dw = bwd_fn(dy, x, rstd, weight, dy2=dy2, dres=dres, eps=eps, dw_dtype=torch.float32)
    return dx, _sum_over_ranks(dw, group, exact_order, reduce_fn)


def add_rmsnorm_bwd_dp(dy: torch.Tensor, dh: torch.Tensor, h: torch.Tensor,
                       rstd: torch.Tensor, weight: torch.Tensor, *, group=None,
                       exact_order: bool = True, bwd_fn: Callable | None = None,
                       reduce_fn: Callable | None = None):
    """Backward of residual add + RMSNorm on local rows:
    d_res = dh + rmsnorm_bwd(dy), dweight summed over ranks."""
    return rmsnorm_bwd_dp(dy, h, rstd, weight, group=group, exact_order=exact_order,
                          dres=dh, bwd_fn=bwd_fn, reduce_fn=reduce_fn)


def rmsnorm_fwd_bwd_dp(x: torch.Tensor, weight: torch.Tensor, dy: torch.Tensor, *,
                       x2: torch.Tensor | None = None, x3: torch.Tensor | None = None,
                       dy2: torch.Tensor | None = None, dy3: torch.Tensor | None = None,
                       dres: torch.Tensor | None = None, eps: float = 1e-5,
                       write_y: bool = True, group=None, exact_order: bool = True,
                       fwd_bwd_fn: Callable | None = None,
                       reduce_fn: Callable | None = None):
    """The RMSNorm forward recomputed in its backward (ops.rmsnorm_fwd_bwd)
    on this rank's rows, dweight summed over all ranks.

    Returns (y or None, dx for the local rows, global fp32 dweight)."""
    fwd_bwd_fn = fwd_bwd_fn or ops.rmsnorm_fwd_bwd
    reduce_fn = reduce_fn or ops.dw_reduce
    y, _, dx, dw = fwd_bwd_fn(x, weight, dy, x2=x2, x3=x3, dy2=dy2, dy3=dy3, dres=dres, eps=eps,
                              write_y=write_y, dw_dtype=torch.float32)
    return y, dx, _sum_over_ranks(dw, group, exact_order, reduce_fn)


def embedding_fwd_vocab_parallel(ids: torch.Tensor, table_shard: torch.Tensor, vocab_lo: int,
                                 vocab_total: int, *, group=None,
                                 fwd_fn: Callable | None = None) -> torch.Tensor:
    """Vocab-parallel gather: masked local gather, then all-reduce (SUM)."""
    fwd_fn = fwd_fn or ops.embedding_fwd
    out = fwd_fn(ids, table_shard, vocab_lo=vocab_lo, vocab_total=vocab_total)
    world, _ = _world(group)
    if world > 1:
        dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
    return out


def embedding_bwd_vocab_parallel(grad: torch.Tensor, ids: torch.Tensor, vocab_lo: int,
                                 shard_rows_n: int, vocab_total: int, *,
                                 padding_idx: int = -1,
                                 bwd_fn: Callable | None = None) -> torch.Tensor:
    """This rank's fp32 table-gradient shard (rows [vocab_lo, vocab_lo+shard_rows_n))."""
    bwd_fn = bwd_fn or ops.embedding_bwd
    return bwd_fn(grad, ids, shard_rows_n, vocab_lo=vocab_lo, vocab_total=vocab_total,
                  padding_idx=padding_idx)
