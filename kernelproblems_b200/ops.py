"""Functional API over libfrag.so for torch CUDA tensors.

Every op validates dtypes/shapes on the host, allocates its outputs (and any
workspace) with torch on the input's device, and launches the CUDA kernels
through the C ABI on the current stream.  Nothing here computes on the CPU:
if the library is missing the call raises.

Embedding ids are range-checked on the device.  A bad id writes a zero row and
sets a flag in a per-device status word; ``check_status()`` synchronises and
raises ``IndexError`` if any flag is set.  Set ``FRAG_SYNC_CHECK=1`` to check
after every embedding call (what torch's device-side assert would catch).
"""
from __future__ import annotations

import ctypes as C
import os
from contextlib import contextmanager

import torch

from . import _lib
from ._lib import FragError

__all__ = [
    "FragError",
    "rmsnorm_fwd",
    "add_rmsnorm_fwd",
    "rmsnorm_bwd",
    "rmsnorm_fwd_bwd",
    "rmsnorm_bwd_workspace_bytes",
    "rmsnorm_bwd_num_blocks",
    "dw_reduce",
    "embedding_fwd",
    "embedding_rmsnorm_fwd",
    "embedding_bwd",
    "rmsnorm_embedding_bwd",
    "copy_rows",
    "copy_rows_grouped",
    "convert",
    "rope",
    "rope_complex",
    "check_status",
    "reset_status",
]

_SYNC_CHECK = os.environ.get("FRAG_SYNC_CHECK", "0") not in ("", "0")
_status_words: dict[int, torch.Tensor] = {}


def _ptr(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(dev: torch.device):
    return C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


@contextmanager
def _on_device(dev: torch.device):
    if dev.type != "cuda":
        raise ValueError(f"kernelproblems_b200 ops need CUDA tensors, got device {dev}")
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if torch.cuda.current_device() == idx:
        yield
    else:
        with torch.cuda.device(idx):
            yield


def _need(t: torch.Tensor, name: str, dtype: torch.dtype, dev: torch.device | None = None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if dev is not None and t.device != dev:
        raise ValueError(f"{name} is on {t.device}, expected {dev}")


def _check_out(t: torch.Tensor, name: str, dtype: torch.dtype, dev: torch.device, *,
               shape: tuple | None = None, numel: int | None = None) -> torch.Tensor:
    """A caller-supplied output buffer is written by the kernel as one dense
    block of `shape` (or `numel` elements), so it must be exactly that: the
    right shape or element count, dtype and device, and contiguous.  Anything
    else would let the kernel write past the buffer."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name}: shape {tuple(t.shape)} != {tuple(shape)}")
    if numel is not None and t.numel() != numel:
        raise ValueError(f"{name}: {t.numel()} elements, the kernel writes {numel}")
    if t.dtype != dtype:
        raise ValueError(f"{name}: dtype {t.dtype} != {dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if t.device != dev:
        raise ValueError(f"{name} is on {t.device}, expected {dev}")
    return t


def _status_word(dev: torch.device) -> torch.Tensor:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = w
    return w


def check_status(device: torch.device | int | None = None) -> None:
    """Synchronise and raise IndexError if a kernel flagged an out-of-range id
    (embedding ids, RoPE table positions),
    RuntimeError if a kernel gave up waiting for its own copies (a bounded
    wait expired: its outputs are not valid)."""
    lib = _lib.load()
    cur = torch.cuda.current_device()
    dev_idx = cur if device is None else (device if isinstance(device, int) else device.index)
    with torch.cuda.device(dev_idx if dev_idx is not None else cur):
        flags = lib.frag_device_errors(1)
    if flags < 0:
        raise FragError("frag_device_errors", -flags)
    if flags & _lib.FRAG_DEVFLAG_WAIT_TIMEOUT:
        raise RuntimeError("a libfrag kernel's bounded wait expired; its outputs are invalid")
    if flags & _lib.FRAG_DEVFLAG_INDEX_OOB:
        raise IndexError("rope: a position was outside the freqs table")
    if device is None:
        devs = list(_status_words)
    elif isinstance(device, int):
        devs = [device]
    else:  # torch.device("cuda") without an index means the current device
        devs = [device.index if device.index is not None else cur]
    for idx in devs:
        w = _status_words.get(idx)
        if w is None:
            continue
        v = int(w.item())
        if v & _lib.FRAG_DEVFLAG_INDEX_OOB:
            w.zero_()
            raise IndexError("embedding: an index was outside [0, num_embeddings)")


def reset_status() -> None:
    for w in _status_words.values():
        w.zero_()


# ---------------------------------------------------------------- RMSNorm

def _rows(x: torch.Tensor, N: int, name: str) -> int:
    if x.shape[-1] != N:
        raise ValueError(f"{name}: last dim {x.shape[-1]} != normalized size {N}")
    if not x.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return x.numel() // N if N else 0


def rmsnorm_fwd(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, *,
                out: torch.Tensor | None = None, rstd: torch.Tensor | None = None,
                save_rstd: bool = True):
    """y = bf16((x * rstd) * w), rstd = 1/sqrt(mean(x^2)+eps) per row (fp32).

    Returns (y, rstd) with y shaped like x and rstd shaped x.shape[:-1]
    (None when save_rstd is False)."""
    _need(x, "x", torch.bfloat16)
    _need(weight, "weight", torch.bfloat16, x.device)
    N = weight.numel()
    M = _rows(x, N, "x")
    y = (torch.empty_like(x) if out is None
         else _check_out(out, "out", torch.bfloat16, x.device, shape=x.shape))
    if save_rstd and rstd is None:
        rstd = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    elif save_rstd:
        _check_out(rstd, "rstd", torch.float32, x.device, numel=M)
    wc = weight.contiguous()
    with _on_device(x.device):
        _lib.call("frag_rmsnorm_fwd", _ptr(x), _ptr(wc), _ptr(y),
                  _ptr(rstd if save_rstd else None), M, N, float(eps), _stream(x.device))
    return y, (rstd if save_rstd else None)


def add_rmsnorm_fwd(residual: torch.Tensor, x: torch.Tensor, weight: torch.Tensor,
                    eps: float = 1e-5, *, write_h: bool = True, save_rstd: bool = True,
                    h_out: torch.Tensor | None = None, y_out: torch.Tensor | None = None):
    """h = bf16(residual + x); y = rmsnorm(h) * w.  Returns (h, y, rstd)."""
    _need(residual, "residual", torch.bfloat16)
    _need(x, "x", torch.bfloat16, residual.device)
    _need(weight, "weight", torch.bfloat16, residual.device)
    if residual.shape != x.shape:
        raise ValueError(f"residual {tuple(residual.shape)} and x {tuple(x.shape)} differ")
    N = weight.numel()
    M = _rows(x, N, "x")
    _rows(residual, N, "residual")
    h = None
    if write_h:
        h = (torch.empty_like(x) if h_out is None
             else _check_out(h_out, "h_out", torch.bfloat16, x.device, shape=x.shape))
    y = (torch.empty_like(x) if y_out is None
         else _check_out(y_out, "y_out", torch.bfloat16, x.device, shape=x.shape))
    rstd = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device) if save_rstd else None
    wc = weight.contiguous()
    with _on_device(x.device):
        _lib.call("frag_add_rmsnorm_fwd", _ptr(residual), _ptr(x), _ptr(wc),
                  _ptr(h), _ptr(y), _ptr(rstd), M, N, float(eps), _stream(x.device))
    return h, y, rstd


def rmsnorm_fwd_bwd(x: torch.Tensor, weight: torch.Tensor, dy: torch.Tensor, *,
                    x2: torch.Tensor | None = None, x3: torch.Tensor | None = None,
                    dy2: torch.Tensor | None = None, dy3: torch.Tensor | None = None,
                    dres: torch.Tensor | None = None, eps: float = 1e-5,
                    write_y: bool = True, save_rstd: bool = False,
                    dw_dtype: torch.dtype | None = torch.float32,
                    workspace: torch.Tensor | None = None):
    """RMSNorm forward recomputed inside its backward, one pass
    (frag_rmsnorm_fwd_bwd).  Returns (y, rstd, dx, dw):

    h     bf16(bf16(x + x2) + x3) (x2, x3 optional), never written
    y     bf16((h * rstd) * w) like x, or None (write_y=False)
    rstd  fp32 [rows], or None (save_rstd=False)
    dx    bf16(dres + bf16(RMSNorm backward of bf16(bf16(dy + dy2) + dy3)))
    dw    fp32, bf16 or None, summed in a fixed order
    """
    _need(x, "x", torch.bfloat16)
    dev = x.device
    _need(weight, "weight", torch.bfloat16, dev)
    N = weight.numel()
    M = _rows(x, N, "x")
    if x3 is not None and x2 is None:
        raise ValueError("x3 needs x2 (the inputs are summed in order)")
    if dy3 is not None and dy2 is None:
        raise ValueError("dy3 needs dy2 (the gradients are summed in order)")
    for name, t in (("dy", dy), ("x2", x2), ("x3", x3), ("dy2", dy2), ("dy3", dy3), ("dres", dres)):
        if t is not None:
            _need(t, name, torch.bfloat16, dev)
            if t.shape != x.shape:
                raise ValueError(f"{name} {tuple(t.shape)} and x {tuple(x.shape)} differ")
            _rows(t, N, name)
    if dw_dtype not in (None, torch.float32, torch.bfloat16):
        raise TypeError("dw_dtype must be float32, bfloat16 or None")
    y = torch.empty_like(x) if write_y else None
    rstd = torch.empty(M, dtype=torch.float32, device=dev) if save_rstd else None
    dx = torch.empty_like(x)
    dw = None if dw_dtype is None else torch.empty(N, dtype=dw_dtype, device=dev)
    with _on_device(dev):
        lib = _lib.load()
        need = int(lib.frag_rmsnorm_bwd_workspace_bytes(M, N))
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
        _lib.call("frag_rmsnorm_fwd_bwd", _ptr(x), _ptr(x2), _ptr(x3), _ptr(weight.contiguous()),
                  _ptr(dy), _ptr(dy2), _ptr(dy3), _ptr(dres), _ptr(y), _ptr(rstd), _ptr(dx),
                  _ptr(dw) if dw_dtype == torch.float32 else None,
                  _ptr(dw) if dw_dtype == torch.bfloat16 else None,
                  M, N, float(eps), _ptr(workspace), workspace.numel(), _stream(dev))
    return y, rstd, dx, dw


def rmsnorm_bwd_workspace_bytes(M: int, N: int, device=None) -> int:
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with _on_device(dev):
        return int(_lib.load().frag_rmsnorm_bwd_workspace_bytes(M, N))


def rmsnorm_bwd_num_blocks(M: int, N: int, device=None) -> int:
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with _on_device(dev):
        return int(_lib.load().frag_rmsnorm_bwd_num_blocks(M, N))


def rmsnorm_bwd(dy: torch.Tensor, x: torch.Tensor, rstd: torch.Tensor | None,
                weight: torch.Tensor, *, dy2: torch.Tensor | None = None,
                dy3: torch.Tensor | None = None,
                dres: torch.Tensor | None = None, eps: float = 1e-6,
                dw_dtype: torch.dtype | None = torch.float32,
                workspace: torch.Tensor | None = None, return_partials: bool = False,
                dx_out: torch.Tensor | None = None, dw_out: torch.Tensor | None = None):
    """RMSNorm backward.  Returns (dx, dw[, partials]).

    dy2   optional second gradient summed (in bf16) into dy first
    dy3   optional third gradient (needs dy2): dy = bf16(bf16(dy + dy2) + dy3)
    rstd  saved rstd (fp32, one per row) or None to recompute it with eps
    dres  optional residual gradient added (in bf16) to dx
    dw    fp32 (dw_dtype=torch.float32), bf16, or None (not reduced)
    dx_out, dw_out  optional preallocated outputs (x-shaped bf16, N elements
          of dw_dtype), written in place and returned
    partials  the [G, N] fp32 per-row-block sums, for cross-rank reductions
    """
    _need(dy, "dy", torch.bfloat16)
    dev = dy.device
    _need(x, "x", torch.bfloat16, dev)
    _need(weight, "weight", torch.bfloat16, dev)
    N = weight.numel()
    M = _rows(x, N, "x")
    if dy.shape != x.shape:
        raise ValueError(f"dy {tuple(dy.shape)} and x {tuple(x.shape)} differ")
    _rows(dy, N, "dy")
    if dy3 is not None and dy2 is None:
        raise ValueError("dy3 needs dy2 (the gradients are summed in order)")
    for name, t in (("dy2", dy2), ("dy3", dy3), ("dres", dres)):
        if t is not None:
            _need(t, name, torch.bfloat16, dev)
            if t.shape != x.shape:
                raise ValueError(f"{name} {tuple(t.shape)} and x {tuple(x.shape)} differ")
            _rows(t, N, name)
    if rstd is not None:
        _need(rstd, "rstd", torch.float32, dev)
        if rstd.numel() != M or not rstd.is_contiguous():
            raise ValueError(f"rstd must be contiguous with {M} elements")
    dx = (torch.empty_like(x) if dx_out is None
          else _check_out(dx_out, "dx_out", torch.bfloat16, dev, shape=x.shape))
    dw = None
    if dw_dtype is not None:
        if dw_dtype not in (torch.float32, torch.bfloat16):
            raise TypeError("dw_dtype must be float32, bfloat16 or None")
        dw = (torch.empty(N, dtype=dw_dtype, device=dev) if dw_out is None
              else _check_out(dw_out, "dw_out", dw_dtype, dev, numel=N))
    with _on_device(dev):
        lib = _lib.load()
        need = int(lib.frag_rmsnorm_bwd_workspace_bytes(M, N))
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
        wc = weight.contiguous()
        tail = (_ptr(x), _ptr(rstd), _ptr(wc), _ptr(dres), _ptr(dx),
                _ptr(dw) if dw_dtype == torch.float32 else None,
                _ptr(dw) if dw_dtype == torch.bfloat16 else None,
                M, N, float(eps), _ptr(workspace), workspace.numel(), _stream(dev))
        if dy3 is None:
            _lib.call("frag_rmsnorm_bwd", _ptr(dy), _ptr(dy2), *tail)
        else:
            _lib.call("frag_rmsnorm_bwd3", _ptr(dy), _ptr(dy2), _ptr(dy3), *tail)
        if return_partials:
            # the launch planned its row blocks from the alignment of every
            # row pointer; ask for the plan of that same case
            aligned = all(t.data_ptr() % 16 == 0
                          for t in (dy, dy2, dy3, x, wc, dres, dx) if t is not None)
            G = int(lib.frag_rmsnorm_bwd_plan_blocks(M, N, int(aligned))) if M else 0
            parts = workspace[: G * N * 4].view(torch.float32).view(G, N)
            return dx, dw, parts
    return dx, dw


def dw_reduce(partials: torch.Tensor, *, out: torch.Tensor | None = None,
              out_bf16: torch.Tensor | None = None) -> torch.Tensor:
    """Fixed-order sum over the rows of a [G, N] fp32 tensor."""
    _need(partials, "partials", torch.float32)
    if partials.dim() != 2 or not partials.is_contiguous():
        raise ValueError("partials must be a contiguous [G, N] tensor")
    G, N = partials.shape
    if out is None and out_bf16 is None:
        out = torch.empty(N, dtype=torch.float32, device=partials.device)
    if out is not None:
        _check_out(out, "out", torch.float32, partials.device, numel=N)
    if out_bf16 is not None:
        _check_out(out_bf16, "out_bf16", torch.bfloat16, partials.device, numel=N)
    with _on_device(partials.device):
        _lib.call("frag_dw_reduce", _ptr(partials), G, N, _ptr(out), _ptr(out_bf16),
                  _stream(partials.device))
    return out if out is not None else out_bf16


# -------------------------------------------------------------- embedding

def embedding_fwd(ids: torch.Tensor, table: torch.Tensor, *, vocab_lo: int = 0,
                  vocab_total: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[..., :] = table[ids - vocab_lo] for ids in the shard, zero otherwise.

    table is the whole table (vocab_lo=0) or one contiguous vocab shard
    [vocab_lo, vocab_lo + table.shape[0]) of a vocab_total-row table."""
    _need(ids, "ids", torch.int64)
    _need(table, "table", torch.bfloat16, ids.device)
    if table.dim() != 2 or not table.is_contiguous():
        raise ValueError("table must be a contiguous [rows, D] tensor")
    rows, D = table.shape
    total = rows if vocab_total is None else int(vocab_total)
    ids_c = ids.contiguous()
    T = ids_c.numel()
    o = (torch.empty(*ids.shape, D, dtype=torch.bfloat16, device=ids.device) if out is None
         else _check_out(out, "out", torch.bfloat16, ids.device, shape=(*ids.shape, D)))
    with _on_device(ids.device):
        st = _status_word(ids.device)
        _lib.call("frag_embedding_fwd", _ptr(ids_c), _ptr(table), _ptr(o), T, rows, D,
                  int(vocab_lo), total, _ptr(st), _stream(ids.device))
    if _SYNC_CHECK:
        check_status(ids.device)
    return o


def embedding_rmsnorm_fwd(ids: torch.Tensor, table: torch.Tensor, weight: torch.Tensor,
                          eps: float = 1e-5, *, save_rstd: bool = False,
                          return_embedding: bool = False):
    """y = rmsnorm(table[ids]) * weight without writing the gathered rows to
    HBM (unless return_embedding).  Returns (y, rstd or None, emb or None)."""
    _need(ids, "ids", torch.int64)
    _need(table, "table", torch.bfloat16, ids.device)
    _need(weight, "weight", torch.bfloat16, ids.device)
    if table.dim() != 2 or not table.is_contiguous():
        raise ValueError("table must be a contiguous [rows, D] tensor")
    V, D = table.shape
    if weight.numel() != D:
        raise ValueError(f"weight has {weight.numel()} elements, table rows have {D}")
    ids_c = ids.contiguous()
    T = ids_c.numel()
    y = torch.empty(*ids.shape, D, dtype=torch.bfloat16, device=ids.device)
    rstd = torch.empty(ids.shape, dtype=torch.float32, device=ids.device) if save_rstd else None
    emb = torch.empty_like(y) if return_embedding else None
    wc = weight.contiguous()
    with _on_device(ids.device):
        st = _status_word(ids.device)
        _lib.call("frag_embedding_rmsnorm_fwd", _ptr(ids_c), _ptr(table), _ptr(wc), _ptr(y), _ptr(rstd),
                  _ptr(emb), T, V, D, float(eps), _ptr(st), _stream(ids.device))
    if _SYNC_CHECK:
        check_status(ids.device)
    return y, rstd, emb


def embedding_bwd(grad: torch.Tensor, ids: torch.Tensor, num_rows: int, *, vocab_lo: int = 0,
                  vocab_total: int | None = None, padding_idx: int = -1,
                  out: torch.Tensor | None = None,
                  workspace: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 table gradient G[v] = sum over tokens t (in order) with ids[t] == v of grad[t].

    Every row of G is written (no memset needed).  num_rows is the number of
    table rows this call owns (the whole vocab, or one shard at vocab_lo)."""
    _need(grad, "grad", torch.bfloat16)
    _need(ids, "ids", torch.int64, grad.device)
    D = grad.shape[-1]
    ids_c = ids.contiguous()
    T = ids_c.numel()
    if grad.numel() != T * D:
        raise ValueError(f"grad {tuple(grad.shape)} does not match {T} ids x {D}")
    g = grad.contiguous()
    total = int(num_rows) if vocab_total is None else int(vocab_total)
    G = (torch.empty(num_rows, D, dtype=torch.float32, device=grad.device) if out is None
         else _check_out(out, "out", torch.float32, grad.device, shape=(num_rows, D)))
    with _on_device(grad.device):
        lib = _lib.load()
        need = int(lib.frag_embedding_bwd_workspace_bytes(T, num_rows))
        if need == 0 and num_rows > 0:
            raise FragError("frag_embedding_bwd_workspace_bytes", 2, "unsupported sizes")
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=grad.device)
        st = _status_word(grad.device)
        _lib.call("frag_embedding_bwd", _ptr(ids_c), _ptr(g), _ptr(G), T, int(num_rows), D,
                  int(vocab_lo), total, int(padding_idx), _ptr(workspace), workspace.numel(),
                  _ptr(st), _stream(grad.device))
    if _SYNC_CHECK:
        check_status(grad.device)
    return G


def rmsnorm_embedding_bwd(x: torch.Tensor, weight: torch.Tensor, ids: torch.Tensor,
                          dy: torch.Tensor | tuple | list, num_rows: int, *,
                          rstd: torch.Tensor | None = None, dres: torch.Tensor | None = None,
                          eps: float = 1e-5, write_y: bool = False, return_d_emb: bool = False,
                          dw_dtype: torch.dtype = torch.float32, vocab_lo: int = 0,
                          vocab_total: int | None = None, padding_idx: int = -1,
                          out: torch.Tensor | None = None,
                          workspace: torch.Tensor | None = None):
    """RMSNorm backward fused into the table-gradient scatter of its input
    gradient (the first attention_norm after the token embedding).

    x      the embedding output that entered the norm, bf16 [..., D]
    dy     one bf16 gradient, or a sequence of up to three summed in order in
           bf16 (bf16(bf16(a + b) + c), as the reference graph adds them)
    rstd   saved rstd (fp32, one per token) or None to recompute it with eps
    dres   optional residual gradient added (bf16) to the norm's dx
    Returns (G fp32 [num_rows, D], dw [D] (fp32 or bf16), y or None, d_emb or None):
    y is the recomputed forward bf16(x * rstd * w) (write_y), d_emb the
    gradient the scatter consumed (return_d_emb; otherwise never stored)."""
    terms = list(dy) if isinstance(dy, (tuple, list)) else [dy]
    if not 1 <= len(terms) <= 3:
        raise ValueError("dy must be one tensor or a sequence of one to three tensors")
    _need(x, "x", torch.bfloat16)
    dev = x.device
    _need(weight, "weight", torch.bfloat16, dev)
    _need(ids, "ids", torch.int64, dev)
    D = weight.numel()
    T = _rows(x, D, "x")
    if ids.numel() != T:
        raise ValueError(f"ids has {ids.numel()} elements, x has {T} rows")
    for j, t in enumerate(terms):
        _need(t, f"dy[{j}]", torch.bfloat16, dev)
        if t.numel() != x.numel():
            raise ValueError(f"dy[{j}] {tuple(t.shape)} does not match x {tuple(x.shape)}")
        _rows(t, D, f"dy[{j}]")
    if dres is not None:
        _need(dres, "dres", torch.bfloat16, dev)
        if dres.numel() != x.numel():
            raise ValueError(f"dres {tuple(dres.shape)} does not match x {tuple(x.shape)}")
        _rows(dres, D, "dres")
    if rstd is not None:
        _need(rstd, "rstd", torch.float32, dev)
        if rstd.numel() != T or not rstd.is_contiguous():
            raise ValueError(f"rstd must be contiguous with {T} elements")
    if dw_dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("dw_dtype must be float32 or bfloat16")
    ids_c = ids.contiguous()
    total = int(num_rows) if vocab_total is None else int(vocab_total)
    G = (torch.empty(num_rows, D, dtype=torch.float32, device=dev) if out is None
         else _check_out(out, "out", torch.float32, dev, shape=(num_rows, D)))
    dw = torch.empty(D, dtype=dw_dtype, device=dev)
    y = torch.empty_like(x) if write_y else None
    d_emb = torch.empty_like(x) if return_d_emb else None
    a, b, c = (terms + [None, None])[:3]
    wc = weight.contiguous()
    with _on_device(dev):
        lib = _lib.load()
        need = int(lib.frag_rmsnorm_embedding_bwd_workspace_bytes(T, D, num_rows))
        if need == 0 and D > 0:
            raise FragError("frag_rmsnorm_embedding_bwd_workspace_bytes", 2, "unsupported sizes")
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
        st = _status_word(dev)
        _lib.call("frag_rmsnorm_embedding_bwd", _ptr(x), _ptr(wc), _ptr(rstd), _ptr(y),
                  _ptr(a), _ptr(b), _ptr(c), _ptr(dres), _ptr(d_emb), _ptr(ids_c), _ptr(G),
                  _ptr(dw) if dw_dtype == torch.float32 else None,
                  _ptr(dw) if dw_dtype == torch.bfloat16 else None,
                  T, D, int(num_rows), int(vocab_lo), total, int(padding_idx), float(eps),
                  _ptr(workspace), workspace.numel(), _ptr(st), _stream(dev))
    if _SYNC_CHECK:
        check_status(dev)
    return G, dw, y, d_emb


def copy_rows(src: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Contiguous copy of a 2-D tensor whose rows are contiguous but may be
    strided apart (a split of an FSDP all-gather buffer viewed [world, -1]).
    Returns a new [rows, cols] tensor (or fills `out`)."""
    _check_copy_src(src)
    rows, cols = src.shape
    if out is None:
        out = torch.empty(rows, cols, dtype=src.dtype, device=src.device)
    elif out.shape != src.shape or out.dtype != src.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor of src's shape and dtype")
    es = src.element_size()
    with _on_device(src.device):
        _lib.call("frag_copy_rows", _ptr(src), src.stride(0) * es, _ptr(out), cols * es, rows,
                  cols * es, _stream(src.device))
    return out


def _check_copy_src(src: torch.Tensor) -> None:
    if not isinstance(src, torch.Tensor):
        raise TypeError("src must be a torch.Tensor")
    if not src.is_cuda:
        raise ValueError("src must be a CUDA tensor")
    if src.dim() != 2 or (src.shape[1] > 1 and src.stride(1) != 1):
        raise ValueError("src must be 2-D with contiguous rows")


def copy_rows_grouped(srcs, outs=None) -> list[torch.Tensor]:
    """copy_rows for up to 16 sources in one launch (frag_copy_rows_grouped):
    the splits of one FSDP all-gather buffer viewed [world, -1].  Returns the
    contiguous copies in order (or fills the given `outs`, None entries
    allocated)."""
    srcs = list(srcs)
    if len(srcs) > _lib.FRAG_COPY_MAX_SEGMENTS:
        raise ValueError(f"at most {_lib.FRAG_COPY_MAX_SEGMENTS} sources per group")
    outs = [None] * len(srcs) if outs is None else list(outs)
    if len(outs) != len(srcs):
        raise ValueError("outs must match srcs in length")
    if not srcs:
        return []
    for src in srcs:
        _check_copy_src(src)
    dev = srcs[0].device
    if any(src.device != dev for src in srcs):
        raise ValueError("all sources must be on one device")
    segs = (_lib.CopySegment * len(srcs))()
    for i, src in enumerate(srcs):
        rows, cols = src.shape
        out = outs[i]
        if out is None:
            out = outs[i] = torch.empty(rows, cols, dtype=src.dtype, device=dev)
        elif (out.shape != src.shape or out.dtype != src.dtype or not out.is_contiguous()
              or out.device != dev):
            raise ValueError("each out must be a contiguous tensor of its src's shape and dtype")
        es = src.element_size()
        segs[i] = _lib.CopySegment(src.data_ptr(), out.data_ptr(), src.stride(0) * es, cols * es,
                                   rows, cols * es)
    with _on_device(dev):
        _lib.call("frag_copy_rows_grouped", segs, len(srcs), _stream(dev))
    return outs


_DT = {torch.bfloat16: _lib.FRAG_DT_BF16, torch.float32: _lib.FRAG_DT_F32}


def convert(src: torch.Tensor, dtype: torch.dtype, copies: int = 1):
    """bf16 <-> fp32 element type conversion (frag_convert_rows): a new
    contiguous tensor of src's shape in `dtype` (fp32 -> bf16 rounds to
    nearest even), or a tuple of `copies` (1 or 2) such tensors written by
    one pass.  src may be any view whose last dimension is contiguous and
    whose leading dimensions collapse into one row stride."""
    if not isinstance(src, torch.Tensor) or src.dtype not in _DT or dtype not in _DT:
        raise TypeError("convert takes bfloat16 / float32 tensors and dtypes")
    if not src.is_cuda:
        raise ValueError("src must be a CUDA tensor")
    if copies not in (1, 2):
        raise ValueError("copies must be 1 or 2")
    cols = src.shape[-1] if src.dim() else 1
    try:
        rows2d = src.view(-1, cols) if src.dim() else src.view(1, 1)
    except RuntimeError:
        raise ValueError("src's leading dimensions must collapse into one row stride") from None
    if cols > 1 and rows2d.stride(1) != 1:
        raise ValueError("src's last dimension must be contiguous")
    outs = [torch.empty(src.shape, dtype=dtype, device=src.device) for _ in range(copies)]
    rows = rows2d.shape[0]
    with _on_device(src.device):
        _lib.call("frag_convert_rows", _ptr(rows2d), _DT[src.dtype], rows2d.stride(0) if rows > 1 else cols,
                  _ptr(outs[0]), _ptr(outs[1]) if copies == 2 else None, _DT[dtype], cols, rows, cols,
                  _stream(src.device))
    return outs[0] if copies == 1 else tuple(outs)


# ------------------------------------------------------------------- RoPE

_LAYOUTS = {"neox": _lib.FRAG_ROPE_NEOX, "interleaved": _lib.FRAG_ROPE_INTERLEAVED}


def _rope_desc(x: torch.Tensor, out: torch.Tensor, name: str) -> _lib.RopeTensor:
    if x.dim() != 4:
        raise ValueError(f"{name} must be [B, S, H, D] (any strides, last dim contiguous)")
    if x.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError(f"{name}: the head dimension must be contiguous")
    if out.shape != x.shape:
        raise ValueError(f"{name}: output shape {tuple(out.shape)} != {tuple(x.shape)}")
    if out.dtype not in (torch.bfloat16, torch.float32) or out.device != x.device:
        raise TypeError(f"{name}: the output must be bf16 or float32 on {x.device}")
    B, S, H, D = x.shape
    odt = _lib.FRAG_ROPE_OUT_F32 if out.dtype == torch.float32 else _lib.FRAG_ROPE_OUT_BF16
    idt = _lib.FRAG_ROPE_IN_F32 if x.dtype == torch.float32 else _lib.FRAG_ROPE_IN_BF16
    if idt == _lib.FRAG_ROPE_IN_F32 and odt != _lib.FRAG_ROPE_OUT_F32:
        raise TypeError(f"{name}: a float32 input needs a float32 output")
    return _lib.RopeTensor(x.data_ptr(), out.data_ptr(), H, x.stride(0), x.stride(1), x.stride(2),
                           out.stride(0), out.stride(1), out.stride(2), odt, idt)


def rope_complex(q: torch.Tensor, k: torch.Tensor | None, positions: torch.Tensor | None,
                 freqs: torch.Tensor, *, inverse: bool = False, out_q: torch.Tensor | None = None,
                 out_k: torch.Tensor | None = None):
    """The complex multiply of the v1/v2 snapshots: q (and k) complex64
    [B, S, H, D/2] times freqs[positions] (complex64 [P, D/2]; positions None
    = s), complex64 results (new, or the given out_q / out_k), fp32
    arithmetic throughout -> (out_q, out_k)."""
    def real(t, name):
        if not isinstance(t, torch.Tensor) or t.dtype != torch.complex64 or t.dim() != 4:
            raise TypeError(f"{name} must be a complex64 [B, S, H, D/2] tensor")
        if t.stride(-1) != 1:
            raise ValueError(f"{name}: the last dimension must be contiguous")
        return torch.view_as_real(t).flatten(-2)
    oq = torch.empty(q.shape, dtype=torch.complex64, device=q.device) if out_q is None else out_q
    ok = None
    if k is not None:
        ok = torch.empty(k.shape, dtype=torch.complex64, device=k.device) if out_k is None else out_k
    rope(real(q, "q"), None if k is None else real(k, "k"), positions, theta=None, freqs=freqs,
         layout="interleaved", inverse=inverse, out_q=real(oq, "out_q"),
         out_k=None if ok is None else real(ok, "out_k"))
    return oq, ok


def _new_out(x: torch.Tensor, out_layout: str) -> torch.Tensor:
    B, S, H, D = x.shape
    if out_layout == "bshd":
        return torch.empty((B, S, H, D), dtype=x.dtype, device=x.device)
    if out_layout == "bhsd":  # [B, H, S, D] storage, returned as a [B, S, H, D] view
        return torch.empty((B, H, S, D), dtype=x.dtype, device=x.device).transpose(1, 2)
    raise ValueError("out_layout must be 'bshd' or 'bhsd'")


def rope(q: torch.Tensor, k: torch.Tensor | None = None, positions: torch.Tensor | None = None, *,
         theta: float | None = 500000.0, freqs: torch.Tensor | None = None,
         layout: str = "neox", inverse: bool = False, out_q: torch.Tensor | None = None,
         out_k: torch.Tensor | None = None, out_layout: str = "bshd"):
    """Rotary embedding of q (and k) given as [B, S, H, D] views (any strides,
    contiguous head dim).  Returns (out_q, out_k); outputs default to new
    contiguous tensors and may alias the inputs (in-place).

    positions: int32/int64 [B, S] (or [S], broadcast over B), or None for
    position = s.  freqs: complex64 [P, D/2] table indexed by position (the
    reference's freqs_cis input); without it cos/sin are computed in
    registers from theta.  inverse=True applies the conjugate rotation (the
    backward).  out_layout="bhsd" writes new outputs in the [B, H, S, D]
    storage order attention kernels read (the transpose is fused into the
    stores; the returned tensors are [B, S, H, D] views of that storage, so
    `.transpose(1, 2)` gives contiguous [B, H, S, D]).  An out_q / out_k of
    dtype float32 receives the rotated values unrounded.  float32 q and k
    (complex64 tensors viewed as (re, im) pairs, see rope_complex) take the
    interleaved layout and float32 outputs."""
    if not isinstance(q, torch.Tensor) or q.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("q must be a bfloat16 or float32 torch.Tensor")
    if not q.is_cuda:
        raise ValueError("q must be a CUDA tensor")
    dev = q.device
    if q.dtype == torch.float32 and layout != "interleaved":
        raise ValueError("float32 (complex) inputs take the interleaved layout")
    if layout not in _LAYOUTS:
        raise ValueError(f"layout must be one of {sorted(_LAYOUTS)}")
    B, S, Hq, D = q.shape
    oq = _new_out(q, out_layout) if out_q is None else out_q
    descs = [_rope_desc(q, oq, "q")]
    ok = None
    if k is not None:
        _need(k, "k", q.dtype, dev)
        if k.shape[0] != B or k.shape[1] != S or k.shape[3] != D:
            raise ValueError(f"k {tuple(k.shape)} does not match q {tuple(q.shape)}")
        ok = _new_out(k, out_layout) if out_k is None else out_k
        descs.append(_rope_desc(k, ok, "k"))
    arr = (_lib.RopeTensor * len(descs))(*descs)
    pos_ptr, pos_dtype, psb, pss = None, _lib.FRAG_POS_NONE, 0, 0
    if positions is not None:
        if positions.device != dev:
            raise ValueError("positions must be on the same device as q")
        if positions.dtype == torch.int64:
            pos_dtype = _lib.FRAG_POS_I64
        elif positions.dtype == torch.int32:
            pos_dtype = _lib.FRAG_POS_I32
        else:
            raise TypeError("positions must be int32 or int64")
        if positions.dim() == 1:
            if positions.shape[0] != S:
                raise ValueError("1-D positions must have S entries")
            psb, pss = 0, positions.stride(0)
        elif positions.dim() == 2 and tuple(positions.shape) == (B, S):
            psb, pss = positions.stride(0), positions.stride(1)
        else:
            raise ValueError(f"positions must be [B, S] or [S], got {tuple(positions.shape)}")
        pos_ptr = C.c_void_p(positions.data_ptr())
    fptr, fstride, frows = None, 0, 0
    if freqs is not None:
        if freqs.dtype != torch.complex64 or freqs.device != dev:
            raise TypeError("freqs must be a complex64 tensor on q's device")
        f2 = freqs.reshape(-1, freqs.shape[-1])
        if f2.shape[-1] != D // 2 or f2.stride(-1) != 1:
            raise ValueError(f"freqs rows must hold D/2={D // 2} contiguous complex values")
        fptr, fstride, frows = C.c_void_p(f2.data_ptr()), f2.stride(0), f2.shape[0]
        theta_v = 0.0
    else:
        if theta is None:
            raise ValueError("either theta or freqs is required")
        theta_v = float(theta)
    with _on_device(dev):
        _lib.call("frag_rope", arr, len(descs), B, S, D, pos_ptr, pos_dtype, psb, pss, fptr,
                  fstride, frows, theta_v, _LAYOUTS[layout], int(bool(inverse)), _stream(dev))
    return oq, ok
