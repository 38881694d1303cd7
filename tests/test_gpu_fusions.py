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
