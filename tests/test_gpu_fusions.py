"""GPU parity of the fused fragments: embedding gather + RMSNorm (the gathered
rows never reach HBM) and RoPE writing the attention [B, H, S, D] layout."""
import pytest
import torch

from conftest import assert_bf16_close, assert_f32_close
from kernelproblems_b200 import configs as cf
from kernelproblems_b200 import ops
from oracle import fragments as ora

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("T,V,D,eps", [(8192, 128256, 4096, 1e-5), (77, 1000, 4096, 1e-6),
                                       (33, 500, 8192, 1e-5), (5, 50, 1000, 1e-5), (3, 7, 24, 1e-6)])
def test_embedding_rmsnorm_fwd(T, V, D, eps):
    g = torch.Generator().manual_seed(T + D)
    ids = torch.randint(0, V, (T,), generator=g)
    table = cf.randn((V, D), std=0.02, seed=T)
    w = cf.rmsnorm_weight(D, seed=D)
    y, rstd, emb = ops.embedding_rmsnorm_fwd(ids.to(DEV), table.to(DEV), w.to(DEV), eps,
                                             save_rstd=True, return_embedding=True)
    ey, er = ora.embedding_rmsnorm_fwd(table, ids, w, eps)
    assert_bf16_close(y, ey, "y")
    assert_f32_close(rstd, er.reshape(rstd.shape), "rstd")
    assert torch.equal(emb.cpu(), ora.embedding_fwd(table, ids)), "gathered rows bit exact"


@pytest.mark.parametrize("T,V,D,save_rstd,emb", [
    (2000, 5000, 4096, True, False),   # ring: ~5 rows per CTA, rstd only
    (20000, 50000, 4096, False, True),  # ring: 46 rows per CTA, the 8-stage ring wraps 5 times
    (460000, 3000, 64, True, True),     # > 1024 rows per CTA: the row-per-CTA kernel instead
])
def test_embedding_rmsnorm_fwd_ring_shapes(T, V, D, save_rstd, emb):
    g = torch.Generator().manual_seed(T)
    ids = torch.randint(0, V, (T,), generator=g)
    ids[7] = V + 3  # out of range: a zero row, flagged
    ids[T // 2] = -1
    table = cf.randn((V, D), std=0.02, seed=V)
    w = cf.rmsnorm_weight(D, seed=D + 1)
    ops.reset_status()
    y, rstd, e = ops.embedding_rmsnorm_fwd(ids.to(DEV), table.to(DEV), w.to(DEV), 1e-5,
                                           save_rstd=save_rstd, return_embedding=emb)
    with pytest.raises(IndexError):
        ops.check_status()
    bad = torch.tensor([7, T // 2])
    assert torch.count_nonzero(y[bad]) == 0
    keep = torch.ones(T, dtype=torch.bool)
    keep[bad] = False
    ey, er = ora.embedding_rmsnorm_fwd(table, ids.clamp(0, V - 1), w, 1e-5)
    assert_bf16_close(y[keep.to(DEV)], ey[keep], "y")
    if save_rstd:
        assert_f32_close(rstd[keep.to(DEV)], er.reshape(-1)[keep], "rstd")
    if emb:
        assert torch.count_nonzero(e[bad]) == 0
        assert torch.equal(e[keep.to(DEV)].cpu(), ora.embedding_fwd(table, ids.clamp(0, V - 1))[keep])


def test_embedding_rmsnorm_out_of_range():
    table = cf.randn((16, 64), std=0.02, seed=1).to(DEV)
    w = cf.rmsnorm_weight(64).to(DEV)
    ids = torch.tensor([3, 16, -2], dtype=torch.int64, device=DEV)
    ops.reset_status()
    y, _, _ = ops.embedding_rmsnorm_fwd(ids, table, w)
    with pytest.raises(IndexError):
        ops.check_status()
    assert torch.count_nonzero(y[1:]) == 0


@pytest.mark.parametrize("layout", ["neox", "interleaved"])
def test_rope_sdpa_layout(layout):
    B, S, Hq, Hk, D = 2, 512, 8, 2, 128
    q = cf.randn((B, S, Hq, D), seed=90)
    k = cf.randn((B, S, Hk, D), seed=91)
    pos = torch.arange(S).expand(B, S).contiguous()
    oq, ok = ops.rope(q.to(DEV), k.to(DEV), pos.to(DEV), theta=500000.0, layout=layout, out_layout="bhsd")
    assert oq.transpose(1, 2).is_contiguous() and ok.transpose(1, 2).is_contiguous()
    ref = ora.rope_neox if layout == "neox" else ora.rope_interleaved_theta
    assert_bf16_close(oq, ref(q, pos, 500000.0), "q")
    assert_bf16_close(ok, ref(k, pos, 500000.0), "k")
