"""RMSNorm backward fused into the embedding backward (ops.rmsnorm_embedding_bwd)
against the CPU oracle of the reference chain
(v6/0b493aad68f0/problem.py:45-70, oracle.fragments.rmsnorm_embedding_bwd).

  * y and d_emb (bf16 tensors of the graph) within the bf16 tolerance,
  * the table gradient equal, within fp32 rounding (rtol 1e-4), to the
    float64 sum of the d_emb rows the kernel itself produced, with every
    untouched row exactly zero,
  * dweight within rtol 1e-4 of a float64 sum,
  * bitwise identical results on a second call (fixed summation order),
over the TMA-ring kernel and the generic fallback, runs that cross many CTA
ranges (one id for every token), padding, vocab shards and empty inputs."""
import pytest
import torch

from conftest import assert_bf16_close, assert_f32_close
from kernelproblems_b200 import ops
from oracle import fragments as F

pytestmark = pytest.mark.gpu


def _make(T, D, V, n_dy, with_dres, seed, id_hi=None, pad=None):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, D, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(D, generator=g)).bfloat16()
    dys = [torch.randn(T, D, generator=g).bfloat16() for _ in range(n_dy)]
    dres = torch.randn(T, D, generator=g).bfloat16() if with_dres else None
    ids = torch.randint(0, id_hi or V, (T,), generator=g)
    if pad is not None and T:
        ids[::7] = pad
    return x, w, dys, dres, ids


def _check(x, w, dys, dres, ids, V, *, rstd_saved=False, padding_idx=-1, vocab_lo=0, rows=None,
           misalign=False):
    T, D = x.shape
    rows = V if rows is None else rows
    _, rstd = F.rmsnorm_fwd(x, w, 1e-5)
    rstd = rstd.view(T)
    dev = "cuda"
    gx, gw, gids = x.to(dev), w.to(dev), ids.to(dev)
    gdys = [d.to(dev) for d in dys]
    gdres = dres.to(dev) if dres is not None else None
    if misalign:
        # x at a 2-byte storage offset: not 16-byte aligned (generic kernel)
        buf = torch.empty(T * D + 1, dtype=x.dtype, device=dev)
        buf[1:].copy_(gx.flatten())
        gx = buf[1:].view(T, D)
    kw = dict(rstd=rstd.to(dev) if rstd_saved else None, dres=gdres, eps=1e-5, write_y=True,
              return_d_emb=True, vocab_lo=vocab_lo, vocab_total=V, padding_idx=padding_idx)
    G, dw, y, d_emb = ops.rmsnorm_embedding_bwd(gx, gw, gids, gdys, rows, **kw)
    G2, dw2, _, _ = ops.rmsnorm_embedding_bwd(gx, gw, gids, gdys, rows, **kw)
    torch.cuda.synchronize()
    ops.check_status()
    assert torch.equal(G, G2) and torch.equal(dw, dw2), "not reproducible"

    if T == 0:
        assert torch.count_nonzero(G) == 0 and torch.count_nonzero(dw) == 0
        return
    y_ref, _ = F.rmsnorm_fwd(x, w, 1e-5)
    assert_bf16_close(y.cpu(), y_ref, "y")
    dw_ref, _, d_ref, dy_ref = F.rmsnorm_embedding_bwd(x, w, dys, rstd.view(T, 1), dres, ids, V, padding_idx)
    # d_emb = bf16(dres + bf16(dx)): a one-ulp difference in the rounded dx
    # survives cancellation, so the bound scales with the summands
    dx_ref = d_ref.float() - (dres.float() if dres is not None else 0)
    mag = dx_ref.abs() + (dres.float().abs() if dres is not None else 0)
    assert_bf16_close(d_emb.cpu(), d_ref, "d_emb", atol=1e-2 + 1.6e-2 * mag)
    assert_f32_close(dw.cpu(), F.rmsnorm_dw_f64(dy_ref, x, rstd), "dweight vs float64", atol=1e-3)
    assert_bf16_close(dw.cpu(), dw_ref, "dweight vs the reference graph", atol=5e-2)
    # the scatter itself: G == float64 sum of the kernel's own d_emb rows
    keep = (ids != padding_idx) if padding_idx >= 0 else torch.ones_like(ids, dtype=torch.bool)
    g64 = F.embedding_bwd_f64(d_emb.cpu().float(), torch.where(keep, ids, -1), rows, -1, vocab_lo)
    cnt = torch.bincount((ids[keep & (ids >= vocab_lo) & (ids < vocab_lo + rows)] - vocab_lo),
                         minlength=rows).double()
    assert_f32_close(G.cpu(), g64, "table gradient", atol=(1e-4 * cnt.sqrt()).unsqueeze(1))
    assert torch.count_nonzero(G.cpu()[cnt == 0]) == 0


@pytest.mark.parametrize("n_dy,with_dres,rstd_saved", [(3, True, False), (1, False, True), (2, True, True)])
def test_chain_tma(n_dy, with_dres, rstd_saved):
    x, w, dys, dres, ids = _make(1000, 4096, 5000, n_dy, with_dres, seed=1 + n_dy, id_hi=300)
    _check(x, w, dys, dres, ids, 5000, rstd_saved=rstd_saved)


def test_chain_reference_ids():
    # the reference problem's id distribution: randint(0, 100), ~80 tokens per row
    x, w, dys, dres, ids = _make(8192, 4096, 128256, 3, True, seed=11, id_hi=100)
    _check(x, w, dys, dres, ids, 128256)


def test_chain_one_id_spans_every_range():
    # a single run over all tokens: every CTA range holds a slice of it
    x, w, dys, dres, ids = _make(3000, 1024, 64, 2, True, seed=5)
    ids[:] = 17
    _check(x, w, dys, dres, ids, 64)


def test_chain_vpt2_width():
    x, w, dys, dres, ids = _make(700, 8192, 900, 3, True, seed=7, id_hi=50)
    _check(x, w, dys, dres, ids, 900)


def test_chain_padding_and_shard():
    x, w, dys, dres, ids = _make(900, 512, 1000, 2, True, seed=9, pad=3)
    _check(x, w, dys, dres, ids, 1000, padding_idx=3)
    _check(x, w, dys, dres, ids, 1000, padding_idx=3, vocab_lo=250, rows=500)


def test_chain_generic_width_and_alignment():
    x, w, dys, dres, ids = _make(400, 100, 60, 3, True, seed=13)   # D % 8 != 0
    _check(x, w, dys, dres, ids, 60)
    x, w, dys, dres, ids = _make(300, 256, 40, 2, False, seed=17)
    _check(x, w, dys, dres, ids, 40, rstd_saved=True, misalign=True)


@pytest.mark.parametrize("T", [0, 1])
def test_chain_tiny(T):
    x, w, dys, dres, ids = _make(T, 256, 32, 3, True, seed=19 + T)
    _check(x, w, dys, dres, ids, 32)


def test_chain_index_out_of_range_flags():
    x, w, dys, dres, ids = _make(64, 256, 32, 1, False, seed=23)
    ids[5] = 32
    ops.reset_status()
    ops.rmsnorm_embedding_bwd(x.cuda(), w.cuda(), ids.cuda(), [d.cuda() for d in dys], 32)
    with pytest.raises(IndexError):
        ops.check_status()


def test_chain_problem_v8_with_saved_rstd():
    """v8/f6251e84e3fa with a proper (y, rstd) pair as its first input."""
    from kernelproblems_b200.problems import PROBLEMS
    from oracle.problems import ORACLES
    g = torch.Generator().manual_seed(29)
    S, D = 8192, 4096
    emb = torch.randn(1, S, D, generator=g).bfloat16()
    w = torch.randn(D, generator=g).bfloat16()
    mms = [torch.randn(S, D, generator=g).bfloat16() for _ in range(3)]
    add_220 = torch.randn(1, S, D, generator=g).bfloat16()
    ids = torch.randint(0, 100, (1, S), generator=g)
    y, rstd = F.rmsnorm_fwd(emb, w, 1e-5)
    cpu_in = [(y, rstd), *mms, emb, w, add_220, ids]
    gpu_in = [(y.cuda(), rstd.cuda()), *[m.cuda() for m in mms], emb.cuda(), w.cuda(), add_220.cuda(),
              ids.cuda()]
    dw, G = PROBLEMS["v8/f6251e84e3fa"](*gpu_in)
    torch.cuda.synchronize()
    dw_ref, _ = ORACLES["v8/f6251e84e3fa"](*cpu_in)
    assert dw.dtype == torch.float32 and tuple(dw.shape) == (D,)
    assert G.dtype == torch.float32 and tuple(G.shape) == (128256, D)
    assert_bf16_close(dw.cpu(), dw_ref, "dweight vs the reference graph", atol=5e-2)
    # table gradient against the float64 sum of the oracle's d_emb (the CPU
    # reference accumulates it in bf16, see test_gpu_problems)
    v = [m.view(emb.shape) for m in mms]
    _, _, d_emb, _ = F.rmsnorm_embedding_bwd(emb, w, v, rstd, add_220, ids, 128256)
    assert_f32_close(G.cpu(), F.embedding_bwd_f64(d_emb, ids, 128256), "table gradient vs float64",
                     atol=0.125)
