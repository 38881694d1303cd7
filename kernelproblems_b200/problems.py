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
drop-in is registered and works when given that pair.  Five v1 graphs
(v1/b3f1b1135abc, v1/3e3eb10963d7, v1/b508c9141fed, v1/d800447a68f6,
v1/db48e1361360) call device(...) without importing it and raise NameError
as shipped; their drop-ins compute what the v2 snapshots of the same graphs
compute.
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
    # [8, 512] view of the all-gathered flat buffer -> contiguous [4096] (a
    # copy only when the shards are strided apart)
    if shard_view.is_contiguous():
        return shard_view.view(-1)
    return ops.copy_rows(shard_view).view(-1)


WORLD = 8   # FSDP ranks whose shards one all-gather buffer holds


def _splits(flat: torch.Tensor, sizes) -> tuple:
    """split_with_sizes(flat.view(8, -1), sizes, 1): strided views, no copy."""
    return torch.split(flat.view(WORLD, -1), list(sizes), dim=1)


def _add_rms_weight0(mm, res, w):
    _, y, _ = ops.add_rmsnorm_fwd(res.contiguous(), mm.contiguous().view(res.shape), w.view(-1), 1e-5,
                                  write_h=False, save_rstd=False)
    return y.view(-1, w.numel())


def _add_rms_table(mm, res, flat):
    # splits [512, 65667072]: the norm weight and the unsharded lm_head /
    # embedding table, both copied out in one grouped launch
    w, table = ops.copy_rows_grouped(_splits(flat, [512, flat.numel() // WORLD - 512]))
    return _add_rms_weight0(mm, res, w), table.view(VOCAB, DIM)


def add_rms_unshard_8e33a91b7364(mm_223, add_62, wait_tensor_969):
    """v8/8e33a91b7364/optimized_kernel.py:99 (v6, v7 same id): h = add_62 +
    mm_223 (bf16), y = _fused_rms_norm(h, weight, 1e-5) with the weight the
    [8, 512] split 0 of the all-gather buffer viewed [8, -1], and the
    [8, 65667072] split 1 unsharded into a contiguous [128256, 4096] table ->
    (y [M, N], table)."""
    return _add_rms_table(mm_223, add_62, wait_tensor_969)


def add_rms_unshard_t_013a3088b488(mm_223, add_62, wait_tensor_969):
    """v5/013a3088b488/problem.py:16-55: as v8/8e33a91b7364, with the table
    returned transposed for the lm_head -> (y [M, N], table.t() [4096, 128256])."""
    y, table = _add_rms_table(mm_223, add_62, wait_tensor_969)
    return (y, table.t())


def add_rms_unshard_tt_18b859c50de2(mm_223, add_62, wait_tensor_969):
    """v4/18b859c50de2/problem.py:12-33 (v1-v3 same id): v5/013a3088b488's
    graph with reshape for _unsafe_view and the table transposed twice, so
    the second output is the contiguous [128256, 4096] table itself."""
    y, table = _add_rms_table(mm_223, add_62, wait_tensor_969)
    return (y, table.t().t())


# splits of one decoder layer's parameters in the [8, 27264000] view of its
# all-gather buffer, and the shapes they are unsharded into (the ninth split
# is not used by the graph)
LAYER_SPLITS = (512, 2097152, 524288, 524288, 2097152, 512, 7340032, 7340032, 7340032)
LAYER_SHAPES = ((4096,), (4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (4096,),
                (14336, 4096), (14336, 4096))


def _add_rms_layer(mm, res, flat):
    parts = ops.copy_rows_grouped(_splits(flat, LAYER_SPLITS)[:len(LAYER_SHAPES)])
    y = _add_rms_weight0(mm, res, parts[0])
    return y, [c.view(shape) for c, shape in zip(parts, LAYER_SHAPES)], parts


def add_rms_layer_unshard_94985bdb7630(mm_216, add_60, wait_tensor_966):
    """v8/94985bdb7630/problem.py:16-106: h = add_60 + mm_216, y =
    _fused_rms_norm(h, split 0 as the weight, 1e-5), and splits 1-7 of the
    [8, 27264000] view unsharded -> (y x3 [8192, 4096], [4096, 4096],
    [1024, 4096], [1024, 4096], [4096, 4096], [4096], [14336, 4096] x2)."""
    y, shaped, _ = _add_rms_layer(mm_216, add_60, wait_tensor_966)
    return (y, y, y, *shaped[1:])


def add_rms_layer_unshard_7815074de963(mm_209, add_58, wait_tensor_963):
    """v8/7815074de963/problem.py:16-103: as v8/94985bdb7630, with split 7
    returned as the raw contiguous clone [8, 7340032]."""
    y, shaped, parts = _add_rms_layer(mm_209, add_58, wait_tensor_963)
    return (y, y, y, *shaped[1:7], parts[7])


def rms_fwd_215dd2e6a519(getitem_1614, add_61):
    """v7/215dd2e6a519/problem.py:10-24 (v1-v4/84496d824942 the same graph
    with reshape): weight gathered from the FSDP shard view, _fused_rms_norm
    -> three [M,N] views of y."""
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


def rms_fwd_ffn_unshard_2a844503364a(getitem_1619, add_62, getitem_1620, getitem_1621, getitem_1622):
    """v4/2a844503364a/problem.py:18-74 (v1-v3 same id): ac3fb0b7281f's
    norm, plus the three FFN weights unsharded from their [8, 7340032] views
    of the all-gather buffers and returned transposed -> (y x2, w1.t()
    [4096, 14336], w3.t() [4096, 14336], w2.t() [14336, 4096]).  The weight
    and the three matrices are copied in one grouped launch."""
    w, a, b, c = ops.copy_rows_grouped([getitem_1619, getitem_1620, getitem_1621, getitem_1622])
    y, _ = ops.rmsnorm_fwd(add_62.contiguous(), w.view(-1), 1e-5, save_rstd=False)
    y2 = y.view(-1, w.numel())
    return (y2, y2, a.view(14336, 4096).t(), b.view(14336, 4096).t(), c.view(4096, 14336).t())


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


# ------------------------------- RMSNorm forward recomputed in its backward


def _recompute_bwd(w, x, dys, *, xs=(), dres=None, write_y=True):
    """One frag_rmsnorm_fwd_bwd pass: h = x [+ xs...] (bf16 adds in order),
    y = RMSNorm(h) when asked, dh of the summed gradients, dres added,
    dweight fp32 -> (y [M, N] or None, dx like x, dweight)."""
    x = x.contiguous()
    v = [t.contiguous().view(x.shape) for t in dys]
    vx = [t.contiguous().view(x.shape) for t in xs]
    y, _, dx, dw = ops.rmsnorm_fwd_bwd(
        x, w, v[0], x2=vx[0] if vx else None, x3=vx[1] if len(vx) > 1 else None,
        dy2=v[1] if len(v) > 1 else None, dy3=v[2] if len(v) > 2 else None,
        dres=None if dres is None else dres.contiguous(), eps=1e-5, write_y=write_y,
        dw_dtype=torch.float32)
    return (None if y is None else y.view(-1, w.numel())), dx, dw


def rms_fwd_bwd3_822931829090(add_1, _unsafe_view_450, mm_656, mm_658, mm_660, add_215):
    """v6/822931829090/problem.py:19-66: y, rstd = _fused_rms_norm(add_1),
    dy = (mm_656 + mm_658) + mm_660, dx = add_215 + _fused_rms_norm_backward
    -> (y x3 [M, N], dx, dweight fp32), one pass."""
    y, dx, dw = _recompute_bwd(_unsafe_view_450, add_1, (mm_656, mm_658, mm_660), dres=add_215)
    return (y, y, y, dx, dw)


def rms_fwd_bwd3_363b7b58c971(getitem_818, add_1, mm_656, mm_658, mm_660, add_215):
    """v4/363b7b58c971/problem.py:19-75 (v1-v3 same id, v5/92ce4a0c7b2c):
    822931829090 with the weight gathered from its [8, 512] FSDP view."""
    return rms_fwd_bwd3_822931829090(add_1, _fsdp_weight(getitem_818), mm_656, mm_658, mm_660,
                                     add_215)


def rms_fwd_bwd2_e9198b707240(add_62_recomputed, _unsafe_view_986, mm_230, mm_232, getitem_420):
    """v6/e9198b707240/problem.py:18-56: y, rstd = _fused_rms_norm(x),
    dy = mm_230 + mm_232, dx = getitem_420 + backward -> (y x2, dx, dweight)."""
    y, dx, dw = _recompute_bwd(_unsafe_view_986, add_62_recomputed, (mm_230, mm_232),
                               dres=getitem_420)
    return (y, y, dx, dw)


def rms_fwd_bwd2_84c0a03c4374(getitem_1624, add_62_recomputed, mm_230, mm_232, getitem_420):
    """v4/84c0a03c4374/problem.py:18-65 (v1-v3 same id, v5/401b52261ef5):
    e9198b707240 with the weight from its [8, 512] FSDP view."""
    return rms_fwd_bwd2_e9198b707240(add_62_recomputed, _fsdp_weight(getitem_1624), mm_230, mm_232,
                                     getitem_420)


def add_rms_fwd_bwd_408ac0979ac5(mm_3, embedding, _unsafe_view_428, mm_664, mm_666, add_218):
    """v6/408ac0979ac5/problem.py:19-63: h = embedding + mm_3 (bf16, never
    written), y, rstd = _fused_rms_norm(h), dy = mm_664 + mm_666, dx =
    add_218 + backward at h -> (y x2, dx, dweight)."""
    y, dx, dw = _recompute_bwd(_unsafe_view_428, embedding, (mm_664, mm_666), xs=(mm_3,),
                               dres=add_218)
    return (y, y, dx, dw)


def add_rms_fwd_bwd_9c745ea697a7(mm_3, embedding, getitem_787, mm_664, mm_666, add_218):
    """v4/9c745ea697a7/problem.py:19-72 (v1-v3 same id, v5/cbfdd7549926):
    408ac0979ac5 with the weight from its [8, 512] FSDP view."""
    return add_rms_fwd_bwd_408ac0979ac5(mm_3, embedding, _fsdp_weight(getitem_787), mm_664, mm_666,
                                        add_218)


def add_rms_bwd_28b45679fca1(mm_223, add_62_recomputed, mm_226, view_3253):
    """v6/28b45679fca1/problem.py:17-41: h = add_62_recomputed + mm_223, rstd
    of h recomputed, dh = _fused_rms_norm_backward(mm_226, h) -> (dh,
    dweight fp32); h and y are never written."""
    _, dx, dw = _recompute_bwd(view_3253, add_62_recomputed, (mm_226,), xs=(mm_223,), write_y=False)
    return (dx, dw)


def add_rms_bwd_f7ad66842c19(mm_223, add_62_recomputed, mm_226, wait_tensor_970):
    """v4/f7ad66842c19/problem.py:17-48 (v1-v3 same id, v5/ac7d64b3c769):
    28b45679fca1 with the weight the [4096] buffer viewed [8, 512], split
    [512] and viewed back (no copy in the graph either)."""
    return add_rms_bwd_28b45679fca1(mm_223, add_62_recomputed, mm_226,
                                    _fsdp_weight(wait_tensor_970.view(WORLD, -1)))


def add2_rms_bwd_3c6c589cdf81(mm_220, add_61, mm_223, mm_226, view_3253):
    """v8/3c6c589cdf81/problem.py:18-53: h = (add_61 + mm_220) + mm_223
    (bf16), rstd recomputed, dh = backward(mm_226, h) -> (dh [M, N], dweight)."""
    _, dx, dw = _recompute_bwd(view_3253, add_61, (mm_226,), xs=(mm_220, mm_223), write_y=False)
    return (dx.view(-1, view_3253.numel()), dw)


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


def rope_bwd_dc55b25cdcb2(_conj_63, getitem_641):
    """v6/dc55b25cdcb2/problem.py:15-43: clone(conj freqs) x q-grad
    [1, 32, S, 128] (a transposed view) -> [S, 4096]."""
    return _rope_bwd_strided(getitem_641, _conj_63)


def rope_bwd_qkv_a1318bc813d2(_conj_62, _conj_63, getitem_641, getitem_642, getitem_643):
    """v4/a1318bc813d2/problem.py:18-85 (v5/a1bb72d946b0 with view for
    reshape): q-grad x _conj_63 and k-grad x _conj_62 (two tables, two
    launches), each viewed [S, H*128] and transposed; the v-grad passes
    through as the same transposed view of its storage (no copy, as in the
    graph) -> (dq.t() [4096, S], dk.t() [1024, S], dv.t() [1024, S])."""
    dq = _rope_bwd_strided(getitem_641, _conj_63)
    dk = _rope_bwd_strided(getitem_642, _conj_62)
    _, H, S, D = getitem_643.shape
    dv = getitem_643.transpose(1, 2).reshape(1, S, H * D).reshape(S, H * D)
    return (dq.t(), dk.t(), dv.t())


def rope_c64_075cb40f3d5d(arg586_1, arg582_1, view_as_complex_60, view_as_complex_61):
    """v2/075cb40f3d5d/problem.py:17-29 (v1 same id): complex64 q and k
    times freqs_cis[pos] (index -> mul -> mul), complex64 out."""
    S = view_as_complex_60.shape[1]
    return ops.rope_complex(view_as_complex_60, view_as_complex_61, arg586_1.view(1, S), arg582_1)


def _rope_c64_conj(conj, x):
    # x * clone(conj), conj [1, S, 1, D/2] read as a table indexed by s
    S = x.shape[1]
    oq, _ = ops.rope_complex(x, None, None, conj.reshape(S, -1))
    return oq


def rope_c64_bwd_9cd8f72e74ce(_conj_63, view_as_complex_127):
    """v2/9cd8f72e74ce/problem.py:15-18 (v1 same id): complex64 q-grad
    [1, S, 32, 64] times clone(_conj_63) -> complex64."""
    return _rope_c64_conj(_conj_63, view_as_complex_127)


def rope_c64_bwd_f23f9bb4567a(_conj_62, view_as_complex_126):
    """v2/f23f9bb4567a/problem.py:15-18 (v1 same id): the k-grad
    [1, S, 8, 64] times clone(_conj_62)."""
    return _rope_c64_conj(_conj_62, view_as_complex_126)


def rope_c64_layers_d7efc428b2f5(arg586_1, arg582_1, *qk):
    """v2/d7efc428b2f5/problem.py:81-509 (v1 same id): the complex RoPE of
    33 (q, k) pairs (the layers' recomputed projections), each times
    freqs_cis[pos] -> 66 complex64 outputs in input order; one launch per
    pair."""
    if len(qk) % 2:
        raise ValueError("expected (q, k) pairs")
    S = qk[0].shape[1]
    pos = arg586_1.view(1, S)
    outs = []
    for i in range(0, len(qk), 2):
        outs.extend(ops.rope_complex(qk[i], qk[i + 1], pos, arg582_1))
    return tuple(outs)


def _to_f32_pairs(x4):
    # [1, S, H, 128] bf16 -> fp32 viewed [1, S, H, 64, 2]
    return x4.view(*x4.shape[:-1], -1, 2)


def cast_f32_twice_dcf660c50ef3(mm_217):
    """v2/dcf660c50ef3/problem.py:14-37 (v1, v3 same id; v2/5d51b24b8d83 for
    the k projection): the projection viewed [1, S, H, 128] and widened to
    fp32 twice (two independent tensors, written by one pass) -> two
    [1, S, H, 64, 2] views for view_as_complex."""
    S = mm_217.shape[0]
    a, b = ops.convert(mm_217.contiguous().view(1, S, -1, 128), torch.float32, copies=2)
    return (_to_f32_pairs(a), _to_f32_pairs(b))


def cast_bwd_qkv_b3f1b1135abc(getitem_641, getitem_642, getitem_643):
    """v2/b3f1b1135abc/problem.py:16-43 (v1, v3 same id): the SDPA-layout q
    and k gradients transposed to [1, S, H, 128] and widened to fp32 (viewed
    [.., 64, 2]); the v gradient passes through as the transposed view of its
    storage -> (dq fp32, dk fp32, dv.t() [1024, S])."""
    dq = ops.convert(getitem_641.transpose(1, 2), torch.float32)
    dk = ops.convert(getitem_642.transpose(1, 2), torch.float32)
    _, H, S, D = getitem_643.shape
    dv = getitem_643.transpose(1, 2).reshape(1, S, H * D).reshape(S, H * D)
    return (_to_f32_pairs(dq), _to_f32_pairs(dk), dv.t())


def cast_bf16_t_d800447a68f6(view_as_real_127):
    """v2/d800447a68f6/problem.py:14-26 (v1, v3; v2/3e3eb10963d7 for k): the
    RoPE result [1, S, H, 64, 2] fp32 rounded to bf16, viewed [S, H*128] and
    transposed -> [H*128, S]."""
    _, S, H, P, _ = view_as_real_127.shape
    y = ops.convert(view_as_real_127.reshape(1, S, H, 2 * P), torch.bfloat16)
    return y.view(S, H * 2 * P).t()


def cast_bf16_bhsd_db48e1361360(view_as_real_recomputed):
    """v2/db48e1361360/problem.py:14-22 (v1, v3; v2/b508c9141fed for k): the
    recomputed RoPE result rounded to bf16, returned as the [1, H, S, 128]
    transposed view attention reads."""
    _, S, H, P, _ = view_as_real_recomputed.shape
    y = ops.convert(view_as_real_recomputed.reshape(1, S, H, 2 * P), torch.bfloat16)
    return y.transpose(1, 2)


# ------------------------------------------ fused chains across the path

def emb_rms_12545c1e9b06(wait_tensor_871, arg583_1, wait_tensor_873):
    """v8/12545c1e9b06/optimized_kernel.py:66: embedding gather fused with the
    first attention_norm RMSNorm (eps 1e-5), the norm weight taken from split 0
    of the second FSDP buffer (problem.py:27-39); the gathered rows are never
    written to HBM.  Also returns the contiguous copies of splits 1-6 the graph
    makes, unsharded with the weight in one grouped copy."""
    table = wait_tensor_871.view(VOCAB, DIM)
    parts = ops.copy_rows_grouped(_splits(wait_tensor_873, LAYER_SPLITS)[:7])
    y, _, _ = ops.embedding_rmsnorm_fwd(arg583_1, table, parts[0].view(-1), 1e-5)
    y2 = y.view(-1, DIM)
    clones = [c.view(shape) for c, shape in zip(parts[1:7], LAYER_SHAPES[1:7])]
    return (y2, y2, y2, *clones)


def rope_sdpa_6b92d6e665ab(arg586_1, arg582_1, mm_217, mm_218):
    """v4/6b92d6e665ab/optimized_kernel.py (v5/ca76bd89ec38 the same graph
    with _unsafe_view): q and k RoPE returned as the
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
    "v3/680e4c57cdc8": norm_emb_bwd_118d525f44e0,
    "v2/680e4c57cdc8": norm_emb_bwd_118d525f44e0,
    "v1/680e4c57cdc8": norm_emb_bwd_118d525f44e0,
    "v8/f6251e84e3fa": norm_emb_bwd_f6251e84e3fa,
    "v8/12545c1e9b06": emb_rms_12545c1e9b06,
    "v4/6b92d6e665ab": rope_sdpa_6b92d6e665ab,
    "v5/ca76bd89ec38": rope_sdpa_6b92d6e665ab,
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
    "v5/013a3088b488": add_rms_unshard_t_013a3088b488,
    "v4/18b859c50de2": add_rms_unshard_tt_18b859c50de2,
    "v3/18b859c50de2": add_rms_unshard_tt_18b859c50de2,
    "v2/18b859c50de2": add_rms_unshard_tt_18b859c50de2,
    "v1/18b859c50de2": add_rms_unshard_tt_18b859c50de2,
    "v8/94985bdb7630": add_rms_layer_unshard_94985bdb7630,
    "v8/7815074de963": add_rms_layer_unshard_7815074de963,
    "v4/84496d824942": rms_fwd_215dd2e6a519,
    "v3/84496d824942": rms_fwd_215dd2e6a519,
    "v2/84496d824942": rms_fwd_215dd2e6a519,
    "v1/84496d824942": rms_fwd_215dd2e6a519,
    "v4/2a844503364a": rms_fwd_ffn_unshard_2a844503364a,
    "v3/2a844503364a": rms_fwd_ffn_unshard_2a844503364a,
    "v2/2a844503364a": rms_fwd_ffn_unshard_2a844503364a,
    "v1/2a844503364a": rms_fwd_ffn_unshard_2a844503364a,
    "v7/45990c83cfd6": rms_bwd_45990c83cfd6,
    "v6/822931829090": rms_fwd_bwd3_822931829090,
    "v5/92ce4a0c7b2c": rms_fwd_bwd3_363b7b58c971,
    "v4/363b7b58c971": rms_fwd_bwd3_363b7b58c971,
    "v3/363b7b58c971": rms_fwd_bwd3_363b7b58c971,
    "v2/363b7b58c971": rms_fwd_bwd3_363b7b58c971,
    "v1/363b7b58c971": rms_fwd_bwd3_363b7b58c971,
    "v6/e9198b707240": rms_fwd_bwd2_e9198b707240,
    "v5/401b52261ef5": rms_fwd_bwd2_84c0a03c4374,
    "v4/84c0a03c4374": rms_fwd_bwd2_84c0a03c4374,
    "v3/84c0a03c4374": rms_fwd_bwd2_84c0a03c4374,
    "v2/84c0a03c4374": rms_fwd_bwd2_84c0a03c4374,
    "v1/84c0a03c4374": rms_fwd_bwd2_84c0a03c4374,
    "v6/408ac0979ac5": add_rms_fwd_bwd_408ac0979ac5,
    "v5/cbfdd7549926": add_rms_fwd_bwd_9c745ea697a7,
    "v4/9c745ea697a7": add_rms_fwd_bwd_9c745ea697a7,
    "v3/9c745ea697a7": add_rms_fwd_bwd_9c745ea697a7,
    "v2/9c745ea697a7": add_rms_fwd_bwd_9c745ea697a7,
    "v1/9c745ea697a7": add_rms_fwd_bwd_9c745ea697a7,
    "v6/28b45679fca1": add_rms_bwd_28b45679fca1,
    "v5/ac7d64b3c769": add_rms_bwd_f7ad66842c19,
    "v4/f7ad66842c19": add_rms_bwd_f7ad66842c19,
    "v3/f7ad66842c19": add_rms_bwd_f7ad66842c19,
    "v2/f7ad66842c19": add_rms_bwd_f7ad66842c19,
    "v1/f7ad66842c19": add_rms_bwd_f7ad66842c19,
    "v8/3c6c589cdf81": add2_rms_bwd_3c6c589cdf81,
    "v7/7f544ceb2120": add_rms_bwd_7f544ceb2120,
    "v8/d8f596b3df34": add_rms_bwd_d8f596b3df34,
    "v7/ed20955ec34b": add3_rms_bwd_ed20955ec34b,
    "v8/43f0c930291e": add3_rms_bwd_43f0c930291e,
    "v7/1e49beb8a123": emb_fwd_1e49beb8a123,
    "v6/1e49beb8a123": emb_fwd_1e49beb8a123,
    "v5/1e49beb8a123": emb_fwd_1e49beb8a123,
    "v4/1e49beb8a123": emb_fwd_1e49beb8a123,
    "v3/1e49beb8a123": emb_fwd_1e49beb8a123,
    "v2/1e49beb8a123": emb_fwd_1e49beb8a123,
    "v1/1e49beb8a123": emb_fwd_1e49beb8a123,
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
    "v3/dcf660c50ef3": cast_f32_twice_dcf660c50ef3,
    "v2/dcf660c50ef3": cast_f32_twice_dcf660c50ef3,
    "v1/dcf660c50ef3": cast_f32_twice_dcf660c50ef3,
    "v3/5d51b24b8d83": cast_f32_twice_dcf660c50ef3,
    "v2/5d51b24b8d83": cast_f32_twice_dcf660c50ef3,
    "v1/5d51b24b8d83": cast_f32_twice_dcf660c50ef3,
    "v3/b3f1b1135abc": cast_bwd_qkv_b3f1b1135abc,
    "v2/b3f1b1135abc": cast_bwd_qkv_b3f1b1135abc,
    "v1/b3f1b1135abc": cast_bwd_qkv_b3f1b1135abc,
    "v3/d800447a68f6": cast_bf16_t_d800447a68f6,
    "v2/d800447a68f6": cast_bf16_t_d800447a68f6,
    "v1/d800447a68f6": cast_bf16_t_d800447a68f6,
    "v3/3e3eb10963d7": cast_bf16_t_d800447a68f6,
    "v2/3e3eb10963d7": cast_bf16_t_d800447a68f6,
    "v1/3e3eb10963d7": cast_bf16_t_d800447a68f6,
    "v3/db48e1361360": cast_bf16_bhsd_db48e1361360,
    "v2/db48e1361360": cast_bf16_bhsd_db48e1361360,
    "v1/db48e1361360": cast_bf16_bhsd_db48e1361360,
    "v3/b508c9141fed": cast_bf16_bhsd_db48e1361360,
    "v2/b508c9141fed": cast_bf16_bhsd_db48e1361360,
    "v1/b508c9141fed": cast_bf16_bhsd_db48e1361360,
    "v2/075cb40f3d5d": rope_c64_075cb40f3d5d,
    "v1/075cb40f3d5d": rope_c64_075cb40f3d5d,
    "v2/9cd8f72e74ce": rope_c64_bwd_9cd8f72e74ce,
    "v1/9cd8f72e74ce": rope_c64_bwd_9cd8f72e74ce,
    "v2/f23f9bb4567a": rope_c64_bwd_f23f9bb4567a,
    "v1/f23f9bb4567a": rope_c64_bwd_f23f9bb4567a,
    "v2/d7efc428b2f5": rope_c64_layers_d7efc428b2f5,
    "v1/d7efc428b2f5": rope_c64_layers_d7efc428b2f5,
    "v6/dc55b25cdcb2": rope_bwd_dc55b25cdcb2,
    "v5/a1bb72d946b0": rope_bwd_qkv_a1318bc813d2,
    "v4/a1318bc813d2": rope_bwd_qkv_a1318bc813d2,
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
