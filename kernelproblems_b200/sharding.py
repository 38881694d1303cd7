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

``PeerVocabParallelEmbedding`` is the same forward with the exchange fused
into the gather: each token's owner stores its row straight into every
rank's output over NVLink peer memory (CUDA IPC), with bounded flag barriers
instead of an all-reduce (frag_embedding_fwd_vp_peer).

The kernels default to ``kernelproblems_b200.ops``; the ``*_fn`` arguments
exist so the host logic can be exercised on CPU ranks (gloo) in tests.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib, ops
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
    "PeerVocabParallelEmbedding",
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


class _DeviceArray:
    """__cuda_array_interface__ over device memory this module owns or maps."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerVocabParallelEmbedding:
    """Vocab-parallel embedding forward with the exchange fused into the
    gather over NVLink peer memory.

    Every rank allocates an output buffer of ``max_tokens x dim`` bf16 and a
    small flag block once (frag_peer_alloc), the ranks exchange their CUDA
    IPC handles (all_gather_object), and each maps every peer's buffers
    (frag_peer_open).  A call then runs one launch pair on this rank's
    current stream: every token's owning rank gathers its table row and
    stores it into every rank's output; on return (stream order) the output
    holds all rows, bit exact.  All ranks call with the same number of
    tokens, the same number of times, in the same order.

    The returned tensor is a view of the internal buffer and is overwritten
    by the next call (the next call's entry barrier waits until every rank
    has reached it, so no rank overwrites a buffer a peer's stream is still
    reading).  ``close()`` unmaps the peers and frees the buffers.
    """

    def __init__(self, max_tokens: int, dim: int, *, group=None, device: torch.device | None = None):
        world, rank = _world(group)
        if world > _lib.FRAG_PEER_MAX_RANKS:
            raise ValueError(f"at most {_lib.FRAG_PEER_MAX_RANKS} ranks")
        if dim % 8 != 0:
            raise ValueError("dim must be a multiple of 8")
        self.world, self.rank, self.group = world, rank, group
        self.max_tokens, self.dim = int(max_tokens), int(dim)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.epoch = 0
        self._own, self._opened = [], []
        lib = _lib.load()
        with torch.cuda.device(self.device):
            out_ptr, out_h = self._alloc(lib, max(16, self.max_tokens * self.dim * 2))
            ctl_ptr, ctl_h = self._alloc(lib, 256)  # flags [2][world] int32 at 0, counter at 128
            handles = [None] * world
            if world > 1:
                dist.all_gather_object(handles, (out_h, ctl_h), group=group)
            else:
                handles[0] = (out_h, ctl_h)
            outs, ctls = [], []
            for p, (oh, ch) in enumerate(handles):
                if p == rank:
                    outs.append(out_ptr)
                    ctls.append(ctl_ptr)
                else:
                    outs.append(self._open(lib, oh))
                    ctls.append(self._open(lib, ch))
        self._out_arr = (C.c_void_p * world)(*outs)
        self._flag_arr = (C.c_void_p * world)(*ctls)
        self._counter = C.c_void_p(ctl_ptr + 128)
        self._buf = torch.as_tensor(_DeviceArray(out_ptr, (self.max_tokens, self.dim), "<i2"),
                                    device=self.device).view(torch.bfloat16)

    def _alloc(self, lib, nbytes: int):
        p = C.c_void_p()
        h = (C.c_char * _lib.FRAG_IPC_HANDLE_BYTES)()
        _lib.call("frag_peer_alloc", nbytes, C.byref(p), h)
        self._own.append(p.value)
        return p.value, bytes(h)

    def _open(self, lib, handle: bytes):
        p = C.c_void_p()
        h = (C.c_char * _lib.FRAG_IPC_HANDLE_BYTES).from_buffer_copy(handle)
        _lib.call("frag_peer_open", h, C.byref(p))
        self._opened.append(p.value)
        return p.value

    def __call__(self, ids: torch.Tensor, table_shard: torch.Tensor, vocab_lo: int,
                 vocab_total: int) -> torch.Tensor:
        """out[..., :] = table[ids] (the whole vocab, gathered by the owners);
        table_shard holds this rank's rows [vocab_lo, vocab_lo + rows)."""
        if self._buf is None:
            raise RuntimeError("closed")
        ops._need(ids, "ids", torch.int64, self.device)
        ops._need(table_shard, "table_shard", torch.bfloat16, self.device)
        if table_shard.dim() != 2 or table_shard.shape[1] != self.dim or not table_shard.is_contiguous():
            raise ValueError(f"table_shard must be a contiguous [rows, {self.dim}] tensor")
        ids_c = ids.contiguous()
        T = ids_c.numel()
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > max_tokens {self.max_tokens}")
        self.epoch += 1
        with torch.cuda.device(self.device):
            st = ops._status_word(self.device)
            _lib.call("frag_embedding_fwd_vp_peer", ops._ptr(ids_c), ops._ptr(table_shard), T,
                      table_shard.shape[0], self.dim, int(vocab_lo), int(vocab_total), self._out_arr,
                      self._flag_arr, self._counter, self.rank, self.world, self.epoch, ops._ptr(st),
                      ops._stream(self.device))
        return self._buf[:T].view(*ids.shape, self.dim)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after a sync)."""
        if self._buf is None:
            return
        lib = _lib.load()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            self._buf = None
            for p in self._opened:
                lib.frag_peer_close(C.c_void_p(p))
            for p in self._own:
                lib.frag_peer_free(C.c_void_p(p))
        self._own, self._opened = [], []
