"""Drop-in `kernel_function`s for the reference's hot-path problems.

SherlockNoMad/KernelProblems ships each fused graph region as
``vN/<hash>/problem.py`` (a torch ``Model`` plus ``get_inputs()``) and its
Triton drop-in ``vN/<hash>/optimized_kernel.py:kernel_function(*inputs)``
returning the same structure as ``Model.forward``.  The functions below keep
those signatures, argument meanings and output structures (shapes, dtypes,
aliased views) and run the libfrag.so kernels instead:

    from kernelproblems_b200.problems import get_kernel_function
    kernel_function = get_kernel_function("v8/f4e9e58fef73")
    outs = kernel_function(*inputs)          # inputs as get_inputs() makes them

Errors are Python exceptions (TypeError/ValueError for bad inputs, FragError
for a failed launch), as the reference harness expects.  Inputs are never
modified; outputs are new tensors on the inputs' device.

Three problems are broken in the reference itself: v8/f6251e84e3fa,
v8/43f0c930291e and v8/7e38211c7f1c pass a 0-d tensor where their graphs
index a tuple.  Their drop-ins are registered: they work when given the tuple
the graph expects, and raise IndexError on the reference's own inputs, as the
reference Model does.  v8/f6251e84e3fa is broken the same way
(its first input should be the (y, rstd) pair of a _fused_rms_norm); its
drop-in is registered and works when given that pair.
"""
from __future__ import annotations

from typing import Callable

import torch

from . import ops

# --------------------------------------------------------------- RMSNorm fwd


def rms_fwd_f4e9e58fef73(add_recomputed, weight):
    """v8/f4e9e58fef73/optimized_kernel.py:43 (v7 same id): _fused_rms_norm
    (problem.py:16 eps 1e-5) -> (y [M,N] view, y [M,N] view, rstd [...,1] fp32)."""
    N = weight.shape[0]
    y, rstd = ops.rmsnorm_fwd(add_recomputed.contiguous(), weight, 1e-5)
    y2 = y.view(-1, N)
    return (y2, y2, rstd.unsqueeze(-1))


def rms_fwd_4b90e2d83144(embedding, weight, eps=1e-5):
    """v8/4b90e2d83144/optimized_kernel.py:30 -> three [M,N] views of y."""
    N = weight.shape[0]
    y, _ = ops.rmsnorm_fwd(embedding.contiguous(), weight, eps, save_rstd=False)
    y2 = y.view(-1, N)
    return (y2, y2, y2)


def rms_fwd_59f786beb25f(embedding, weight):
    """v7/59f786beb25f/problem.py:10-17 -> (y like x, rstd [...,1])."""
    y, rstd = ops.rmsnorm_fwd(embedding.contiguous(), weight, 1e-5)
    return (y, rstd.unsqueeze(-1))


def _fsdp_weight(shard_view: torch.Tensor) -> torch.Tensor:
    # [8, 512] strided view of the all-gathered flat buffer -> contiguous [4096]
    return shard_view.contiguous().view(-1)


def add_rms_unshard_8e33a91b7364(mm_223, add_62, wait_tensor_969):
    """v8/8e33a91b7364/optimized_kernel.py:99 (v6, v7 same id): h = add_62 +
    mm_223 (bf16), y = _fused_rms_norm(h, weight, 1e-5) with the weight the
    [8, 512] split 0 of the all-gather buffer viewed [8, -1], and the
    [8, 65667072] split 1 unsharded into a contiguous [128256, 4096] table ->
    (y [M, N], table)."""
    flat = wait_tensor_969.view(8, -1)
    w = ops.copy_rows(flat[:, :512]).view(-1)
    _, y, _ = ops.add_rmsnorm_fwd(add_62.contiguous(), mm_223.contiguous().view(add_62.shape), w,
                                  1e-5, write_h=False, save_rstd=False)
    table = ops.copy_rows(flat[:, 512:]).view(VOCAB, DIM)
    return (y.view(-1, w.numel()), table)


def rms_fwd_215dd2e6a519(getitem_1614, add_61):
    """v7/215dd2e6a519/problem.py:10-24: weight gathered from the FSDP shard
    view, _fused_rms_norm -> three [M,N] views of y."""
    w = _fsdp_weight(getitem_1614)
    y, _ = ops.rmsnorm_fwd(add_61.contiguous(), w, 1e-5, save_rstd=False)
    y2 = y.view(-1, w.numel())
    return (y2, y2, y2)


def rms_fwd_ac3fb0b7281f(getitem_1619, add_62):
    """v7/ac3fb0b7281f/problem.py:10-22 -> two [M,N] views of y."""
    w = _fsdp_weight(getitem_1619)
    y, _ = ops.rmsnorm_fwd(add_62.contiguous(), w, 1e-5, save_rstd=False)
    y2 = y.view(-1, w.numel())
    return (y2, y2)


def add_rms_fwd_7884328a5557(mm_220, add_61, w):
    """v8/7884328a5557/optimized_kernel.py:37: h = add_61 + mm_220 (bf16),
    y = _fused_rms_norm(h, eps 1e-5) -> (y [M,N], y [M,N]) (h not returned)."""
    N = w.shape[0]
    _, y, _ = ops.add_rmsnorm_fwd(add_61.contiguous(), mm_220.contiguous().view(add_61.shape), w,
                                  1e-5, write_h=False, save_rstd=False)
    y2 = y.view(-1, N)
    return (y2, y2)


# --------------------------------------------------------------- RMSNorm bwd


def rms_bwd_45990c83cfd6(x, weight, grad_out, eps=1e-5):
    """v7/45990c83cfd6/optimized_kernel.py:96: rstd recomputed, then
    _fused_rms_norm_backward -> (dx like x, dweight in weight's dtype)."""
    dx, dw = ops.rmsnorm_bwd(grad_out.contiguous(), x.contiguous(), None, weight, eps=eps,
                             dw_dtype=weight.dtype)
    return dx, dw


def add_rms_bwd_7f544ceb2120(mm_666, view_1776, add_recomputed, getitem_12_recomputed,
                             _unsafe_view_428, add_218):
    """v7/7f544ceb2120/optimized_kernel.py:71: dy = view_1776 + mm_666 (bf16),
    backward against add_recomputed with the saved rstd, d_res = add_218 + dx
    (bf16), dweight fp32 -> (d_res like add_218, dweight fp32)."""
    x = add_recomputed.contiguous()
    dres, dw = ops.rmsnorm_bwd(view_1776.contiguous(), x,
                               getitem_12_recomputed.contiguous().view(x.shape[:-1]),
                               _unsafe_view_428, dy2=mm_666.contiguous().view(x.shape),
                               dres=add_218.contiguous(), dw_dtype=torch.float32)
    return dres, dw


def add_rms_bwd_d8f596b3df34(mm_664, mm_666, add_recomputed, getitem_12_recomputed,
                             _unsafe_view_428, add_218):
    """v8/d8f596b3df34/optimized_kernel.py:64: dy = mm_664 + mm_666 (bf16) ->
    (d_res [M,N], dweight fp32)."""
    x = add_recomputed.contiguous()
    N = x.shape[-1]
    dres, dw = ops.rmsnorm_bwd(mm_664.contiguous().view(x.shape), x,
                               getitem_12_recomputed.contiguous().view(x.shape[:-1]),
                               _unsafe_view_428, dy2=mm_666.contiguous().view(x.shape),
                               dres=add_218.contiguous(), dw_dtype=torch.float32)
    return dres.view(-1, N), dw


def add3_rms_bwd_43f0c930291e(_fused_rms_norm_2_recomputed, mm_656, mm_658, mm_660, add_1,
                              _unsafe_view_450, add_215):
    """v8/43f0c930291e/problem.py:10-38: dy = mm_656 + mm_658 + mm_660 (each
    partial sum bf16), backward against add_1 with the saved rstd
    _fused_rms_norm_2_recomputed[1], d_res = add_215 + dx ->
    (d_res [M, N], dweight fp32).  The reference's own get_inputs passes a 0-d
    tensor as the (y, rstd) pair (indexing it raises IndexError, as the
    reference Model does)."""
    rstd = _fused_rms_norm_2_recomputed[1]
    x = add_1.contiguous()
    N = x.shape[-1]
    dres, dw = ops.rmsnorm_bwd(mm_656.contiguous().view(x.shape), x,
                               rstd.contiguous().view(x.shape[:-1]), _unsafe_view_450,
                               dy2=mm_658.contiguous().view(x.shape),
                               dy3=mm_660.contiguous().view(x.shape),
                               dres=add_215.contiguous(), dw_dtype=torch.float32)
    return dres.view(-1, N), dw


def add3_rms_bwd_ed20955ec34b(mm_672, view_1794, mm_674, embedding, getitem_1_recomputed,
                              _unsafe_view_432, add_220):
    """v7/ed20955ec34b/optimized_kernel.py:118: dy = view_1794 + mm_672 + mm_674
    (each partial sum bf16), backward against embedding with the saved rstd,
    d_res = add_220 + dx (bf16), dweight fp32 -> (d_res like add_220, dweight fp32)."""
    x = embedding.contiguous()
    dres, dw = ops.rmsnorm_bwd(view_1794.contiguous(), x,
                               getitem_1_recomputed.contiguous().view(x.shape[:-1]),
                               _unsafe_view_432, dy2=mm_672.contiguous().view(x.shape),
                               dy3=mm_674.contiguous().view(x.shape),
                               dres=add_220.contiguous(), dw_dtype=torch.float32)
    return dres, dw


# ---------------------------------------------------------------- embedding

VOCAB, DIM = 128256, 4096


def emb_fwd_1e49beb8a123(wait_tensor_871, arg583_1):
    """v7/1e49beb8a123/optimized_kernel.py:34 (also v4-v6): the all-gathered
    FSDP flat buffer viewed as table [128256, 4096] (problem.py:16-21), gather
    -> [B, S, 4096] bf16, bit exact."""
    table = wait_tensor_871.view(VOCAB, DIM)
    return ops.embedding_fwd(arg583_1, table)


def emb_bwd_a12a160cb11b(add_223, arg583_1):
    """v7/a12a160cb11b/optimized_kernel.py:37: embedding_dense_backward
    (padding_idx -1) -> fp32 [128256, 4096], summed in a fixed order."""
    return ops.embedding_bwd(add_223, arg583_1, VOCAB, padding_idx=-1)


# --------------------------------------------------------------------- RoPE


def _heads(t: torch.Tensor, S: int, D: int = 128) -> torch.Tensor:
    return t.contiguous().view(1, S, -1, D)


def rope_c8c60d8f7015(arg586_1, arg582_1, mm, mm_1):
    """v8/c8c60d8f7015/optimized_kernel.py:48: q [S,4096] and k [S,1024] as
    heads of 128, freqs_cis rows picked by int32 positions, complex multiply
    -> (q [1,S,32,128], k [1,S,8,128]) bf16."""
    S = mm.shape[0]
    return ops.rope(_heads(mm, S), _heads(mm_1, S), arg586_1.view(1, S), freqs=arg582_1,
                    layout="interleaved")


def rope_f32q_0f38bc55457c(mm, mm_1, arg586_1, arg582_1):
    """v7/0f38bc55457c/optimized_kernel.py:84: as c8c60d8f7015, but q is
    returned in fp32 (the graph never rounds it back to bf16) ->
    (q fp32 [1,S,32,128], k bf16 [1,S,8,128])."""
    S = mm.shape[0]
    qv = _heads(mm, S)
    oq = torch.empty(qv.shape, dtype=torch.float32, device=mm.device)
    return ops.rope(qv, _heads(mm_1, S), arg586_1.view(1, S), freqs=arg582_1,
                    layout="interleaved", out_q=oq)


def rope_97032595d968(mm, mm_1, arg586_1, arg582_1):
    """v8/97032595d968/optimized_kernel.py:44: as c8c60d8f7015, argument order
    (mm, mm_1, positions, freqs)."""
    return rope_c8c60d8f7015(arg586_1, arg582_1, mm, mm_1)


def rope_493cad38cac9(mm_217, view_788):
    """v8/493cad38cac9/optimized_kernel.py:48: q [S,4096] x freqs [1,S,1,64]
    indexed by token -> [1,S,32,128]."""
    S = mm_217.shape[0]
    oq, _ = ops.rope(_heads(mm_217, S), None, None, freqs=view_788.reshape(S, -1),
                     layout="interleaved")
    return oq


def rope_e29b92927600(mm_218, view_788):
    """v8/e29b92927600/optimized_kernel.py:54 (v7 same id): k [S,1024] ->
    [1,S,8,128]."""
    S = mm_218.shape[0]
    ok, _ = ops.rope(_heads(mm_218, S), None, None, freqs=view_788.reshape(S, -1),
                     layout="interleaved")
    return ok


def _rope_bwd_strided(grad_bhsd: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    # grad arrives as [1, H, S, D] (a transposed view of [S, H, D] storage)
    _, H, S, D = grad_bhsd.shape
    x = grad_bhsd.transpose(1, 2)  # [1, S, H, D], head dim contiguous
    out, _ = ops.rope(x, None, None, freqs=freqs.reshape(S, -1), layout="interleaved")
    return out.view(S, H * D)


def rope_bwd_bfe872e373e4(getitem_641, clone_63):
    """v7/bfe872e373e4/optimized_kernel.py:54: q-grad [1,32,S,128] strided view
    times clone_63 (already conjugated upstream) -> [S, 4096]."""
    return _rope_bwd_strided(getitem_641, clone_63)


def rope_bwd_7e38211c7f1c(_scaled_dot_product_flash_attention_backward_31, clone_62):
    """v8/7e38211c7f1c/problem.py:10-31: the k-gradient is entry [1] of the
    SDPA backward's outputs ([1, 8, S, 128], a transposed view) -> [S, 1024].
    The reference's own get_inputs passes a 0-d tensor there (indexing it
    raises IndexError, as the reference Model does)."""
    return _rope_bwd_strided(_scaled_dot_product_flash_attention_backward_31[1], clone_62)


def rope_bwd_5c65f62b0422(getitem_642, clone_62):
    """v7/5c65f62b0422/optimized_kernel.py:45: k-grad [1,8,S,128] -> [S, 1024]."""
    return _rope_bwd_strided(getitem_642, clone_62)


def rope_bwd_03d64c25b654(_conj_62, getitem_642):
    """v6/03d64c25b654/optimized_kernel.py:51: clone(conj freqs) x k-grad
    -> [S, 1024]."""
    return _rope_bwd_strided(getitem_642, _conj_62)


# ------------------------------------------------- SURVEY "next" fusions

_SPLITS_873 = [512, 2097152, 524288, 524288, 2097152, 512, 7340032, 7340032, 7340032]
_SHAPES_873 = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (4096,), (14336, 4096)]


def emb_rms_12545c1e9b06(wait_tensor_871, arg583_1, wait_tensor_873):
    """v8/12545c1e9b06/optimized_kernel.py:66: embedding gather fused with the
    first attention_norm RMSNorm (eps 1e-5), the norm weight taken from split 0
    of the second FSDP buffer (problem.py:27-39); the gathered rows are never
    written to HBM.  Also returns the contiguous copies of splits 1-6 the graph
    makes (FSDP unshard copies: plain data movement, done with torch)."""
    table = wait_tensor_871.view(VOCAB, DIM)
    parts = wait_tensor_873.view(8, -1).split(_SPLITS_873, dim=1)
    w = parts[0].contiguous().view(-1)
    y, _, _ = ops.embedding_rmsnorm_fwd(arg583_1, table, w, 1e-5)
    y2 = y.view(-1, DIM)
    clones = [parts[i + 1].contiguous().view(_SHAPES_873[i]) for i in range(6)]
    return (y2, y2, y2, *clones)


def rope_sdpa_6b92d6e665ab(arg586_1, arg582_1, mm_217, mm_218):
    """v4/6b92d6e665ab/optimized_kernel.py: q and k RoPE returned as the
    [1, H, S, 128] transposed views attention consumes; the reference graph
    computes each twice, so two independent results are returned too."""
    S = mm_217.shape[0]
    pos = arg586_1.view(1, S)
    q, k = ops.rope(_heads(mm_217, S), _heads(mm_218, S), pos, freqs=arg582_1, layout="interleaved")
    q2, k2 = ops.rope(_heads(mm_217, S), _heads(mm_218, S), pos, freqs=arg582_1, layout="interleaved")
    return (q.transpose(1, 2), k.transpose(1, 2), q2.transpose(1, 2), k2.transpose(1, 2))


# ------------------------------------------- RMSNorm bwd -> embedding bwd


def _norm_emb_chain(w, embedding, mm_670, mm_672, mm_674, add_220, ids, rstd=None, write_y=True):
    x = embedding.contiguous()
    N = w.numel()
    dys = [m.contiguous() for m in (mm_670, mm_672, mm_674)]
    G, dw, y, _ = ops.rmsnorm_embedding_bwd(x, w, ids, dys, VOCAB, rstd=rstd,
                                            dres=add_220.contiguous(), eps=1e-5, write_y=write_y)
    return G, dw, (y.view(-1, N) if y is not None else None)


def norm_emb_bwd_0b493aad68f0(embedding, _unsafe_view_432, mm_670, mm_672, mm_674, add_220, arg583_1):
    """v6/0b493aad68f0/optimized_kernel.py:100: _fused_rms_norm of the
    embedding output (rstd recomputed in the fused kernel), dy = mm_670 +
    mm_672 + mm_674 (bf16), d_emb = add_220 + dx, scattered into the fp32
    table gradient without storing d_emb -> (y, y, y [M,N] views, dweight
    fp32 [4096], table gradient fp32 [128256, 4096])."""
    G, dw, y = _norm_emb_chain(_unsafe_view_432, embedding, mm_670, mm_672, mm_674, add_220, arg583_1)
    return (y, y, y, dw, G)


def norm_emb_bwd_118d525f44e0(getitem_791, embedding, mm_670, mm_672, mm_674, add_220, arg583_1):
    """v5/118d525f44e0/optimized_kernel.py:72 and v4/680e4c57cdc8/optimized_kernel.py:69:
    as 0b493aad68f0 with the weight gathered from the [8, 512] FSDP shard view."""
    G, dw, y = _norm_emb_chain(_fsdp_weight(getitem_791), embedding, mm_670, mm_672, mm_674, add_220,
                               arg583_1)
    return (y, y, y, dw, G)


def norm_emb_bwd_f6251e84e3fa(_fused_rms_norm_recomputed, mm_670, mm_672, mm_674, embedding,
                              _unsafe_view_432, add_220, arg583_1):
    """v8/f6251e84e3fa/problem.py:22-57: the saved rstd is
    _fused_rms_norm_recomputed[1] (fp32 [1, S, 1]) -> (dweight fp32, table
    gradient fp32).  The reference's own get_inputs passes a 0-d tensor here,
    so indexing it raises IndexError, as the reference Model does."""
    rstd = _fused_rms_norm_recomputed[1]
    x = embedding.contiguous()
    G, dw, _ = _norm_emb_chain(_unsafe_view_432, x, mm_670, mm_672, mm_674, add_220, arg583_1,
                               rstd=rstd.contiguous().view(x.shape[:-1]), write_y=False)
    return (dw, G)


PROBLEMS: dict[str, Callable] = {
    "v6/0b493aad68f0": norm_emb_bwd_0b493aad68f0,
    "v5/118d525f44e0": norm_emb_bwd_118d525f44e0,
    "v4/680e4c57cdc8": norm_emb_bwd_118d525f44e0,
    "v8/f6251e84e3fa": norm_emb_bwd_f6251e84e3fa,
    "v8/12545c1e9b06": emb_rms_12545c1e9b06,
    "v4/6b92d6e665ab": rope_sdpa_6b92d6e665ab,
    "v8/f4e9e58fef73": rms_fwd_f4e9e58fef73,
    "v7/f4e9e58fef73": rms_fwd_f4e9e58fef73,
    "v8/4b90e2d83144": rms_fwd_4b90e2d83144,
    "v7/59f786beb25f": rms_fwd_59f786beb25f,
    "v7/215dd2e6a519": rms_fwd_215dd2e6a519,
    "v6/215dd2e6a519": rms_fwd_215dd2e6a519,
    "v7/ac3fb0b7281f": rms_fwd_ac3fb0b7281f,
    "v6/ac3fb0b7281f": rms_fwd_ac3fb0b7281f,
    "v8/7884328a5557": add_rms_fwd_7884328a5557,
    "v8/8e33a91b7364": add_rms_unshard_8e33a91b7364,
    "v7/8e33a91b7364": add_rms_unshard_8e33a91b7364,
    "v6/8e33a91b7364": add_rms_unshard_8e33a91b7364,
    "v7/45990c83cfd6": rms_bwd_45990c83cfd6,
    "v7/7f544ceb2120": add_rms_bwd_7f544ceb2120,
    "v8/d8f596b3df34": add_rms_bwd_d8f596b3df34,
    "v7/ed20955ec34b": add3_rms_bwd_ed20955ec34b,
    "v8/43f0c930291e": add3_rms_bwd_43f0c930291e,
    "v7/1e49beb8a123": emb_fwd_1e49beb8a123,
    "v6/1e49beb8a123": emb_fwd_1e49beb8a123,
    "v5/1e49beb8a123": emb_fwd_1e49beb8a123,
    "v4/1e49beb8a123": emb_fwd_1e49beb8a123,
    "v7/a12a160cb11b": emb_bwd_a12a160cb11b,
    "v8/c8c60d8f7015": rope_c8c60d8f7015,
    "v6/c8c60d8f7015": rope_c8c60d8f7015,
    "v7/0f38bc55457c": rope_f32q_0f38bc55457c,
    "v8/97032595d968": rope_97032595d968,
    "v6/97032595d968": rope_97032595d968,
    "v8/493cad38cac9": rope_493cad38cac9,
    "v7/493cad38cac9": rope_493cad38cac9,
    "v8/e29b92927600": rope_e29b92927600,
    "v7/e29b92927600": rope_e29b92927600,
    "v7/bfe872e373e4": rope_bwd_bfe872e373e4,
    "v7/5c65f62b0422": rope_bwd_5c65f62b0422,
    "v8/7e38211c7f1c": rope_bwd_7e38211c7f1c,
    "v6/03d64c25b654": rope_bwd_03d64c25b654,
}


def get_kernel_function(problem: str) -> Callable:
    """`problem` is "vN/<hash>" or a bare hash (the newest snapshot wins)."""
    if problem in PROBLEMS:
        return PROBLEMS[problem]
    for v in ("v8", "v7", "v6", "v5", "v4"):
        key = f"{v}/{problem}"
        if key in PROBLEMS:
            return PROBLEMS[key]
    raise KeyError(f"no drop-in for problem {problem!r}; known: {sorted(PROBLEMS)}")
