"""Torch-CPU restatements of the reference fragments' torch graphs (test oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Each function follows the
reference ``problem.py`` it cites: same aten ops, same dtypes at every
rounding point, so on CPU it reproduces the reference ``Model`` bit for bit
(checked against tests/golden).  ``*_f64`` variants accumulate in float64 and
serve as the accuracy reference for fp32 reductions.

Third-party arithmetic: the reference graphs call PyTorch aten kernels
(``_fused_rms_norm``, ``embedding``, ``embedding_dense_backward``, complex
``mul``).  They are pinned to the installed torch 2.11.0.
``aten._fused_rms_norm_backward`` has no CPU kernel in torch 2.11, so its
registered decomposition (torch/_decomp/decompositions.py:1862-1933 in torch
2.11.0) is restated below.
"""
from __future__ import annotations

import torch

aten = torch.ops.aten


# ------------------------------------------------------------------ RMSNorm

def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float):
    """aten._fused_rms_norm (v8/f4e9e58fef73/problem.py:16,28).

    Returns (y bf16 like x, rstd fp32 [..., 1])."""
    y, rstd = aten._fused_rms_norm.default(x, [w.numel()], w, eps)
    return y, rstd


def add_rmsnorm_fwd(res: torch.Tensor, x: torch.Tensor, w: torch.Tensor, eps: float):
    """aten.add (bf16) -> aten._fused_rms_norm (v8/7884328a5557/problem.py:17-23).

    Returns (h, y, rstd); the reference itself returns only y."""
    h = aten.add.Tensor(res, x)
    y, rstd = aten._fused_rms_norm.default(h, [w.numel()], w, eps)
    return h, y, rstd


def rmsnorm_bwd(dy: torch.Tensor, x: torch.Tensor, rstd: torch.Tensor, w: torch.Tensor):
    """aten._fused_rms_norm_backward(dy, x, [N], rstd, w, [True, True]) as the
    torch 2.11 decomposition computes it (torch/_decomp/decompositions.py:1875-1933):
    fp32 math, dx and dw returned in x's dtype.  Used by
    v7/45990c83cfd6/problem.py:23 and v7/7f544ceb2120/problem.py:26."""
    N = w.numel()
    g = dy.to(torch.float32, memory_format=torch.contiguous_format)
    xf = x.to(torch.float32, memory_format=torch.contiguous_format)
    wf = w.to(torch.float32, memory_format=torch.contiguous_format)
    r = rstd
    while r.dim() < xf.dim():
        r = r.unsqueeze(-1)
    grad_x_hat = g * wf
    x_hat = xf * r
    inner = [xf.dim() - 1]
    outer = list(range(xf.dim() - 1))
    sum_val = torch.sum(x_hat * grad_x_hat, dim=inner, keepdim=True)
    dx = (grad_x_hat - (x_hat / N) * sum_val) * r
    dw_full = g * x_hat
    dw = torch.sum(dw_full, dim=outer, keepdim=False) if outer else dw_full
    return dx.to(x.dtype), dw.to(x.dtype)


def rmsnorm_dw_f64(dy: torch.Tensor, x: torch.Tensor, rstd: torch.Tensor) -> torch.Tensor:
    """dweight = sum over rows of dy * x * rstd, accumulated in float64."""
    N = x.shape[-1]
    g = dy.reshape(-1, N).double()
    xh = x.reshape(-1, N).double() * rstd.reshape(-1, 1).double()
    return (g * xh).sum(0)


def rmsnorm_recompute_bwd(x: torch.Tensor, w: torch.Tensor, dy: torch.Tensor, eps: float):
    """v7/45990c83cfd6/problem.py:17-27: rstd recomputed by _fused_rms_norm,
    then the backward.  Returns (dx bf16, dw bf16) like the reference."""
    _, rstd = aten._fused_rms_norm.default(x, [w.numel()], w, eps)
    return rmsnorm_bwd(dy, x, rstd, w)


def add_rmsnorm_bwd(dy_a: torch.Tensor, dy_b: torch.Tensor | None, h: torch.Tensor,
                    rstd: torch.Tensor, w: torch.Tensor, dres: torch.Tensor | None):
    """add -> _fused_rms_norm_backward -> add -> _to_copy(fp32)
    (v7/7f544ceb2120/problem.py:20-38; v8/d8f596b3df34/problem.py:23-43):
      dy    = bf16(dy_a + dy_b)           (when dy_b is given)
      dx,dw = rmsnorm_bwd(dy, h, rstd, w) (both bf16)
      d_res = bf16(dres + dx)             (when dres is given)
    Returns (d_res, dw fp32 of the bf16 dw)."""
    dy = aten.add.Tensor(dy_a, dy_b) if dy_b is not None else dy_a
    dx, dw = rmsnorm_bwd(dy, h, rstd, w)
    out = aten.add.Tensor(dres, dx) if dres is not None else dx
    return out, aten._to_copy.default(dw, dtype=torch.float32)


# ---------------------------------------------------------------- embedding

def embedding_fwd(table: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    """aten.embedding (v7/1e49beb8a123/problem.py:20-23)."""
    return aten.embedding.default(table, ids)


def embedding_fwd_vocab_shard(table_shard: torch.Tensor, ids: torch.Tensor, vocab_lo: int) -> torch.Tensor:
    """One rank's half of a vocab-parallel embedding: rows for ids in
    [vocab_lo, vocab_lo + shard_rows), zeros elsewhere."""
    rows = table_shard.shape[0]
    local = ids - vocab_lo
    hit = (local >= 0) & (local < rows)
    out = table_shard[local.clamp(0, max(rows - 1, 0))]
    return out * hit.unsqueeze(-1).to(out.dtype) if rows else torch.zeros(
        *ids.shape, table_shard.shape[1], dtype=table_shard.dtype)


def embedding_rmsnorm_fwd(table: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, eps: float):
    """aten.embedding -> aten._fused_rms_norm (v8/12545c1e9b06/problem.py:24,39)."""
    return aten._fused_rms_norm.default(aten.embedding.default(table, ids), [w.numel()], w, eps)


def embedding_bwd(grad: torch.Tensor, ids: torch.Tensor, num_weights: int,
                  padding_idx: int = -1) -> torch.Tensor:
    """aten.embedding_dense_backward -> _to_copy(fp32) (v7/a12a160cb11b/problem.py:16,19).
    Note the bf16 rounding of the summed rows before the fp32 cast."""
    g = aten.embedding_dense_backward.default(grad, ids, num_weights, padding_idx, False)
    return aten._to_copy.default(g, dtype=torch.float32)


def embedding_bwd_f64(grad: torch.Tensor, ids: torch.Tensor, num_weights: int,
                      padding_idx: int = -1, vocab_lo: int = 0) -> torch.Tensor:
    """sum of grad rows per id in float64 (the fp32-accuracy reference).
    With vocab_lo, returns rows [vocab_lo, vocab_lo + num_weights) only."""
    D = grad.shape[-1]
    g = grad.reshape(-1, D).double()
    i = ids.reshape(-1)
    keep = (i >= vocab_lo) & (i < vocab_lo + num_weights)
    if padding_idx >= 0:
        keep &= i != padding_idx
    out = torch.zeros(num_weights, D, dtype=torch.float64)
    out.index_add_(0, (i[keep] - vocab_lo), g[keep])
    return out


def rmsnorm_embedding_bwd(x: torch.Tensor, w: torch.Tensor, dys, rstd: torch.Tensor,
                          dres: torch.Tensor | None, ids: torch.Tensor, num_weights: int,
                          padding_idx: int = -1):
    """add -> add -> _fused_rms_norm_backward -> add -> _to_copy ->
    embedding_dense_backward -> _to_copy (v6/0b493aad68f0/problem.py:45-70,
    v8/f6251e84e3fa/problem.py:31-56):
      dy    = bf16 left-fold sum of dys (one aten.add per extra term)
      dx,dw = rmsnorm_bwd(dy, x, rstd, w)       (bf16)
      d_emb = bf16(dres + dx)                   (when dres is given)
    Returns (dw fp32 of the bf16 dw, G fp32 of the bf16 embedding gradient, d_emb, dy)."""
    dy = dys[0]
    for t in dys[1:]:
        dy = aten.add.Tensor(dy, t)
    dx, dw = rmsnorm_bwd(dy, x, rstd, w)
    d_emb = aten.add.Tensor(dres, dx) if dres is not None else dx
    G = embedding_bwd(d_emb, ids, num_weights, padding_idx)
    return aten._to_copy.default(dw, dtype=torch.float32), G, d_emb, dy


# --------------------------------------------------------------------- RoPE

def precompute_freqs_cis(dim: int, end: int, theta: float) -> torch.Tensor:
    """complex64 [end, dim/2] table exp(i * t * theta^(-2j/dim)), computed in
    fp32 the way torchtitan's llama3 model builds the freqs_cis tensor that the
    reference fragments take as input (v8/c8c60d8f7015/problem.py:13)."""
    freqs = 1.0 / (theta ** (torch.arange(0, dim, 2)[: (dim // 2)].float() / dim))
    t = torch.arange(end, device=freqs.device)
    freqs = torch.outer(t, freqs).float()
    return torch.polar(torch.ones_like(freqs), freqs)


def rope_interleaved(x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """_to_copy(f32) -> view [..., D/2, 2] -> view_as_complex -> mul(freqs)
    -> view_as_real -> view -> _to_copy(bf16)  (v8/c8c60d8f7015/problem.py:30-44,
    v8/e29b92927600/problem.py:20-33, v7/bfe872e373e4/problem.py:17-31).
    x: [B, S, H, D] (any strides); freqs: complex64 broadcastable to [B, S, H, D/2]."""
    xf = aten._to_copy.default(x, dtype=torch.float32)
    xf = xf.reshape(*x.shape[:-1], -1, 2)
    xc = aten.view_as_complex.default(xf)
    out = aten.view_as_real.default(aten.mul.Tensor(xc, freqs))
    return aten._to_copy.default(out.reshape(x.shape), dtype=torch.bfloat16)


def rope_inv_freq(dim: int, theta: float) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, dim, 2)[: (dim // 2)].float() / dim))


def rope_neox(x: torch.Tensor, positions: torch.Tensor, theta: float,
              inverse: bool = False) -> torch.Tensor:
    """Rotate-half RoPE in fp32, one rounding to bf16 at the end.
    x: [B, S, H, D]; positions: [B, S] or [S] integer; pair (j, j + D/2) is
    rotated by angle fp32(pos) * inv_freq[j] (by its negative if inverse)."""
    D = x.shape[-1]
    half = D // 2
    inv = rope_inv_freq(D, theta)
    pos = positions if positions.dim() == 2 else positions.unsqueeze(0).expand(x.shape[0], -1)
    ang = pos.to(torch.float32)[..., None] * inv  # [B, S, half]
    c = torch.cos(ang)[:, :, None, :]
    s = torch.sin(ang)[:, :, None, :]
    if inverse:
        s = -s
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(torch.bfloat16)


def rope_interleaved_theta(x: torch.Tensor, positions: torch.Tensor, theta: float,
                           inverse: bool = False) -> torch.Tensor:
    """Interleaved (complex-pair) RoPE with the freqs table built from theta."""
    D = x.shape[-1]
    pos = positions if positions.dim() == 2 else positions.unsqueeze(0).expand(x.shape[0], -1)
    table = precompute_freqs_cis(D, int(pos.max().item()) + 1, theta)
    f = table[pos.long()]  # [B, S, D/2]
    if inverse:
        f = f.conj()
    return rope_interleaved(x, f[:, :, None, :])


def neox_to_interleaved(x: torch.Tensor) -> torch.Tensor:
    """Permutation P: element j -> 2j and j + D/2 -> 2j + 1."""
    half = x.shape[-1] // 2
    return torch.stack([x[..., :half], x[..., half:]], dim=-1).reshape(x.shape)


def interleaved_to_neox(x: torch.Tensor) -> torch.Tensor:
    """P^-1."""
    y = x.reshape(*x.shape[:-1], -1, 2)
    return torch.cat([y[..., 0], y[..., 1]], dim=-1)


def rope_neox_via_interleaved(x: torch.Tensor, positions: torch.Tensor, theta: float,
                              inverse: bool = False) -> torch.Tensor:
    """neox(x) = P^-1 interleaved(P x): ties the rotate-half oracle (which has
    no reference implementation) to the reference's interleaved RoPE."""
    return interleaved_to_neox(
        rope_interleaved_theta(neox_to_interleaved(x), positions, theta, inverse))
