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
``PeerDweightExchange`` does the dweight exchange the same way: one
single-CTA launch stores this rank's vector into every rank's slot row and
sums the rows in rank order (frag_dw_exchange_peer), bitwise equal to the
all-gather + fixed-order sum.

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
    "PeerDweightExchange",
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
                    reduce_fn: Callable[[torch.Tensor], torch.Tensor], peer=None) -> torch.Tensor:
    world, _ = _world(group)
    if world == 1:
        return dw
    if peer is not None:
        return peer(dw)
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
                   reduce_fn: Callable | None = None,
                   peer: "PeerDweightExchange | None" = None):
    """RMSNorm backward on this rank's rows; dweight summed over all ranks.

    peer: a PeerDweightExchange of the weight's size to exchange over NVLink
    peer memory instead of NCCL (same result bit for bit as exact_order).
    Returns (dx for the local rows, global fp32 dweight)."""
    bwd_fn = bwd_fn or ops.rmsnorm_bwd
    reduce_fn = reduce_fn or ops.dw_reduce
    dx, dw = bwd_fn(dy, x, rstd, weight, dy2=dy2, dres=dres, eps=eps, dw_dtype=torch.float32)
    return dx, _sum_over_ranks(dw, group, exact_order, reduce_fn, peer)


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


class _PeerBuffers:
    """Device buffers shared between the ranks' processes over CUDA IPC: each
    rank allocates one buffer per requested size (frag_peer_alloc, zero
    filled), the ranks exchange the IPC handles once (all_gather_object on
    the group) and map every peer's buffers (frag_peer_open).
    ``ptrs[i][p]`` is rank p's buffer i as seen from this process.

    Construction and ``close()`` are collective and take the same steps on
    every rank whether or not its own allocation or mapping worked: after the
    mappings the ranks agree (an all-reduce of an ok flag), so either every
    rank has all peers mapped before any peer kernel can be launched, or
    every rank releases what it holds and raises.  ``close()`` unmaps the
    peers' buffers on every rank before any rank frees its own (freeing an
    exported buffer that a peer still maps is undefined in CUDA)."""

    def __init__(self, sizes: list[int], group, device: torch.device):
        world, rank = _world(group)
        if world > _lib.FRAG_PEER_MAX_RANKS:
            raise ValueError(f"at most {_lib.FRAG_PEER_MAX_RANKS} ranks")
        self.world, self.rank, self.device, self.group = world, rank, device, group
        self._own, self._opened = [], []
        self.ptrs = None
        _lib.load()
        err = None
        with torch.cuda.device(device):
            mine = []
            try:
                mine = [self._alloc(max(16, int(n))) for n in sizes]
            except Exception as e:  # noqa: BLE001 - reported after the agreement below
                err = e
            handles = [None] * world
            if world > 1:
                dist.all_gather_object(handles, None if err else [h for _, h in mine], group=group)
            else:
                handles[0] = None if err else [h for _, h in mine]
            if err is None and all(h is not None for h in handles):
                try:
                    self.ptrs = [[mine[i][0] if p == rank else self._open(handles[p][i])
                                  for p in range(world)] for i in range(len(sizes))]
                except Exception as e:  # noqa: BLE001
                    err = e
            if not self._agree(err is None and self.ptrs is not None):
                self.close()
                raise RuntimeError(
                    f"peer buffers unavailable on rank {rank}: "
                    + (repr(err) if err is not None else "another rank could not allocate or map its buffers")
                ) from err

    def _agree(self, ok: bool) -> bool:
        """True on every rank iff ``ok`` is true on every rank."""
        if self.world == 1:
            return ok
        t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.group)
        return bool(t.item())

    def _alloc(self, nbytes: int):
        p = C.c_void_p()
        h = (C.c_char * _lib.FRAG_IPC_HANDLE_BYTES)()
        _lib.call("frag_peer_alloc", nbytes, C.byref(p), h)
        self._own.append(p.value)
        return p.value, bytes(h)

    def _open(self, handle: bytes) -> int:
        p = C.c_void_p()
        h = (C.c_char * _lib.FRAG_IPC_HANDLE_BYTES).from_buffer_copy(handle)
        _lib.call("frag_peer_open", h, C.byref(p))
        self._opened.append(p.value)
        return p.value

    def array(self, i: int, offset: int = 0):
        """ctypes array of every rank's buffer i (+ offset bytes)."""
        return (C.c_void_p * self.world)(*[q + offset for q in self.ptrs[i]])

    def close(self) -> None:
        """Collective: every rank syncs and unmaps its peers, then (after a
        barrier) frees its own buffers."""
        lib = _lib.load()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            for p in self._opened:
                lib.frag_peer_close(C.c_void_p(p))
            self._opened = []
            if self.world > 1:
                dist.barrier(group=self.group)
            for p in self._own:
                lib.frag_peer_free(C.c_void_p(p))
            self._own = []
        self.ptrs = None


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
        if dim % 8 != 0:
            raise ValueError("dim must be a multiple of 8")
        self.max_tokens, self.dim = int(max_tokens), int(dim)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        # output rows; flags [2][world] int32 at 0 and this rank's state words at 128
        self._bufs = _PeerBuffers([self.max_tokens * self.dim * 2, 256], group, self.device)
        self.world, self.rank = self._bufs.world, self._bufs.rank
        self._out_arr = self._bufs.array(0)
        self._flag_arr = self._bufs.array(1)
        self._state = C.c_void_p(self._bufs.ptrs[1][self.rank] + 128)  # CTA counter, call count
        self._buf = torch.as_tensor(_DeviceArray(self._bufs.ptrs[0][self.rank], (self.max_tokens, self.dim),
                                                 "<i2"), device=self.device).view(torch.bfloat16)

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
        with torch.cuda.device(self.device):
            st = ops._status_word(self.device)
            _lib.call("frag_embedding_fwd_vp_peer", ops._ptr(ids_c), ops._ptr(table_shard), T,
                      table_shard.shape[0], self.dim, int(vocab_lo), int(vocab_total), self._out_arr,
                      self._flag_arr, self._state, self.rank, self.world, ops._ptr(st),
                      ops._stream(self.device))
        return self._buf[:T].view(*ids.shape, self.dim)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after a sync)."""
        if self._buf is None:
            return
        self._buf = None
        self._bufs.close()


class PeerDweightExchange:
    """The dweight exchange of a row-sharded RMSNorm backward over NVLink
    peer memory (frag_dw_exchange_peer): every rank passes its fp32 dweight
    over its own rows and gets the sum over all ranks, added in rank order
    (bitwise the same on every rank, and equal to ``ops.dw_reduce`` of the
    all-gathered [world, N] block).  One single-CTA launch per call on the
    current stream, in place of an NCCL all-gather (launch-latency bound at
    16-32 KB) followed by the reduce.  All ranks call it equally often, in
    the same order, on one stream each; ``close()`` frees the buffers."""

    def __init__(self, n: int, *, group=None, device: torch.device | None = None):
        if n % 4 != 0:
            raise ValueError("n must be a multiple of 4")
        self.n = int(n)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        world, _ = _world(group)
        self._bufs = _PeerBuffers([world * self.n * 4, 256], group, self.device)
        self.world, self.rank = self._bufs.world, self._bufs.rank
        self._slots = self._bufs.array(0)
        self._flags = self._bufs.array(1)
        self._state = C.c_void_p(self._bufs.ptrs[1][self.rank] + 128)  # call count

    def __call__(self, dw_local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if self._bufs is None:
            raise RuntimeError("closed")
        ops._need(dw_local, "dw_local", torch.float32, self.device)
        if dw_local.numel() != self.n or not dw_local.is_contiguous():
            raise ValueError(f"dw_local must be a contiguous fp32 tensor of {self.n} elements")
        out = (torch.empty(self.n, dtype=torch.float32, device=self.device) if out is None
               else ops._check_out(out, "out", torch.float32, self.device, numel=self.n))
        with torch.cuda.device(self.device):
            _lib.call("frag_dw_exchange_peer", ops._ptr(dw_local), self.n, self._slots, self._flags,
                      self._state, self.rank, self.world, ops._ptr(out), ops._stream(self.device))
        return out

    def close(self) -> None:
        if self._bufs is not None:
            self._bufs.close()
            self._bufs = None
