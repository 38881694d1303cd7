"""GPU parity: embedding gather (bit exact) and the deterministic fp32 backward."""
import pytest
import torch

from conftest import assert_f32_close
from kernelproblems_b200 import configs as cf
from kernelproblems_b200 import ops
from oracle import fragments as ora

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _table(V, D, seed=7):
    return cf.randn((V, D), std=0.02, seed=seed)


def test_embedding_fwd_c2_bit_exact():
    c = cf.C2
    ids = cf.embedding_ids(c)
    table = _table(c.vocab, c.dim)
    out = ops.embedding_fwd(ids.to(DEV), table.to(DEV))
    assert torch.equal(out.cpu(), ora.embedding_fwd(table, ids))


@pytest.mark.parametrize("T,V,D", [(5, 10, 8), (1, 3, 4096), (77, 1000, 12), (300, 50, 1024), (64, 64, 200)])
def test_embedding_fwd_shapes(T, V, D):
    g = torch.Generator().manual_seed(T * 31 + D)
    ids = torch.randint(0, V, (T,), generator=g)
    table = _table(V, D, seed=T)
    out = ops.embedding_fwd(ids.to(DEV), table.to(DEV))
    assert torch.equal(out.cpu(), ora.embedding_fwd(table, ids))


def test_embedding_fwd_vocab_shards_sum_to_full():
    c = cf.EmbeddingCfg("small", (4, 256), 1000, 256)
    ids = cf.embedding_ids(c)
    table = _table(c.vocab, c.dim)
    full = ora.embedding_fwd(table, ids)
    acc = torch.zeros(*ids.shape, c.dim, dtype=torch.float32)
    for r in range(8):
        sh = cf.shard_rows(c.vocab, 8, r)
        part = ops.embedding_fwd(ids.to(DEV), table[sh.lo:sh.hi].contiguous().to(DEV),
                                 vocab_lo=sh.lo, vocab_total=c.vocab).cpu()
        assert torch.equal(part, ora.embedding_fwd_vocab_shard(table[sh.lo:sh.hi], ids, sh.lo))
        acc += part.float()
    assert torch.equal(acc.to(torch.bfloat16), full)


def test_embedding_fwd_out_of_range_flags():
    table = _table(16, 64).to(DEV)
    ids = torch.tensor([0, 15, 16, -1, 3], dtype=torch.int64, device=DEV)
    ops.reset_status()
    out = ops.embedding_fwd(ids, table)
    with pytest.raises(IndexError):
        ops.check_status()
    assert torch.count_nonzero(out[2]) == 0 and torch.count_nonzero(out[3]) == 0
    assert torch.equal(out[1], table[15])
    ops.check_status()  # flag was cleared


def test_embedding_bwd_c2():
    c = cf.C2
    ids = cf.embedding_ids(c)
    grad = cf.randn((*c.batch, c.dim), seed=8)
    G = ops.embedding_bwd(grad.to(DEV), ids.to(DEV), c.vocab)
    ref = ora.embedding_bwd_f64(grad, ids, c.vocab)
    Gc = G.cpu()
    touched = torch.zeros(c.vocab, dtype=torch.bool)
    touched[ids.reshape(-1)] = True
    assert torch.count_nonzero(Gc[~touched]) == 0, "untouched rows must be exactly zero"
    rows = touched.nonzero().squeeze(1)
    # absolute floor for cancelling sums: 1e-4 * sqrt(count) * rms(grad)
    cnt = torch.bincount(ids.reshape(-1), minlength=c.vocab)[rows].double()
    atol = (1e-4 * cnt.sqrt()).unsqueeze(1)
    assert_f32_close(Gc[rows], ref[rows], "G", atol=atol)
    # Against the reference graph itself: its CPU kernel accumulates in bf16,
    # so only rows hit by exactly one token are comparable, and those are exact.
    single = rows[cnt == 1]
    eager = ora.embedding_bwd(grad, ids, c.vocab)
    assert torch.equal(Gc[single], eager[single]), "single-token rows must be exact copies"


def test_embedding_bwd_deterministic_hot_ids():
    V, D, T = 5000, 512, 20000
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, 20, (T,), generator=g)  # heavy collisions
    grad = cf.randn((T, D), seed=9)
    G1 = ops.embedding_bwd(grad.to(DEV), ids.to(DEV), V)
    G2 = ops.embedding_bwd(grad.to(DEV), ids.to(DEV), V)
    assert torch.equal(G1, G2), "table gradient must be bitwise reproducible"
    ref = ora.embedding_bwd_f64(grad, ids, V)
    assert_f32_close(G1.cpu()[:20], ref[:20], "G", atol=1e-4 * (T / 20) ** 0.5)


@pytest.mark.parametrize("T,V,D,pad", [(0, 10, 64, -1), (1, 1, 8, -1), (1000, 3, 40, -1),
                                       (256, 100, 4096, 5), (33, 7, 12, 2), (4096, 1, 1024, -1)])
def test_embedding_bwd_edges(T, V, D, pad):
    g = torch.Generator().manual_seed(T + V)
    ids = torch.randint(0, V, (T,), generator=g)
    grad = cf.randn((T, D), seed=T + 1)
    G = ops.embedding_bwd(grad.to(DEV), ids.to(DEV), V, padding_idx=pad).cpu()
    ref = ora.embedding_bwd_f64(grad, ids, V, padding_idx=pad)
    assert_f32_close(G, ref, "G", atol=1e-4 * max(T, 1) ** 0.5)
    if pad >= 0:
        assert torch.count_nonzero(G[pad]) == 0


def test_embedding_bwd_vocab_shards():
    V, D, T = 1000, 256, 3000
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, V, (T,), generator=g)
    grad = cf.randn((T, D), seed=12)
    parts = []
    for r in range(3):
        sh = cf.shard_rows(V, 3, r)
        parts.append(ops.embedding_bwd(grad.to(DEV), ids.to(DEV), sh.n, vocab_lo=sh.lo,
                                       vocab_total=V).cpu())
    full = ops.embedding_bwd(grad.to(DEV), ids.to(DEV), V).cpu()
    assert torch.equal(torch.cat(parts), full), "shards must equal the matching rows of the full gradient"
