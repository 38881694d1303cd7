"""The multi-GPU wrappers on one GPU with no process group (world size 1):
the real kernels run and the wrappers must return exactly what the plain ops
return (row range = all rows, no exchange).  The exchange itself is covered by
tests/test_sharding_gloo.py on CPU ranks."""
import pytest
import torch

from kernelproblems_b200 import configs as cf
from kernelproblems_b200 import ops, sharding

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_local_rows_single_rank():
    r = sharding.local_rows(37)
    assert (r.lo, r.hi) == (0, 37)
    v = sharding.vocab_shard(128256)
    assert (v.lo, v.hi) == (0, 128256)


def test_rmsnorm_dp_wrappers_equal_the_ops():
    M, N = 96, 4096
    x, x2 = cf.randn((M, N), seed=1).to(DEV), cf.randn((M, N), seed=2).to(DEV)
    dy, dy2 = cf.randn((M, N), seed=3).to(DEV), cf.randn((M, N), seed=4).to(DEV)
    dres = cf.randn((M, N), seed=5).to(DEV)
    w = cf.rmsnorm_weight(N, seed=6).to(DEV)
    _, rstd = ops.rmsnorm_fwd(x, w, 1e-5)
    dx, dw = sharding.rmsnorm_bwd_dp(dy, x, rstd, w, eps=1e-5, dres=dres)
    ex, ew = ops.rmsnorm_bwd(dy, x, rstd, w, eps=1e-5, dres=dres)
    assert torch.equal(dx, ex) and torch.equal(dw, ew)
    y, dx, dw = sharding.rmsnorm_fwd_bwd_dp(x, w, dy, x2=x2, dy2=dy2, dres=dres)
    ey, _, ex, ew = ops.rmsnorm_fwd_bwd(x, w, dy, x2=x2, dy2=dy2, dres=dres)
    assert torch.equal(y, ey) and torch.equal(dx, ex) and torch.equal(dw, ew)


def test_vocab_parallel_embedding_single_rank():
    ec = cf.EmbeddingCfg("dp1", (2, 64), 1000, 256)
    ids = cf.embedding_ids(ec).to(DEV)
    table = cf.randn((1000, 256), std=0.02, seed=7).to(DEV)
    out = sharding.embedding_fwd_vocab_parallel(ids, table, 0, 1000)
    assert torch.equal(out, ops.embedding_fwd(ids, table))
    g = cf.randn((2, 64, 256), seed=8).to(DEV)
    G = sharding.embedding_bwd_vocab_parallel(g, ids, 0, 1000, 1000)
    assert torch.equal(G, ops.embedding_bwd(g, ids, 1000))


def test_peer_vocab_parallel_embedding_single_rank():
    """The fused peer-memory forward with one rank (no peers): its barriers
    complete on its own flags and the output is the plain gather, bit for
    bit, over repeated calls (the epoch advances)."""
    ec = cf.EmbeddingCfg("peer1", (4, 100), 5000, 512)
    ids = cf.embedding_ids(ec).to(DEV)
    table = cf.randn((5000, 512), std=0.02, seed=9).to(DEV)
    emb = sharding.PeerVocabParallelEmbedding(ids.numel(), 512)
    try:
        for _ in range(3):
            out = emb(ids, table, 0, 5000)
            assert torch.equal(out, ops.embedding_fwd(ids, table))
        ops.check_status(torch.device(DEV))
        bad = ids.clone()
        bad[0, 0] = 5000  # outside the vocabulary: a zero row and the index flag
        out = emb(bad, table, 0, 5000)
        assert int(torch.count_nonzero(out[0, 0])) == 0
        with pytest.raises(IndexError):
            ops.check_status(torch.device(DEV))
    finally:
        emb.close()


def test_peer_dweight_exchange_single_rank():
    """One rank: the exchange returns its own vector (plus +0), bit for bit,
    over repeated calls, and the wrapper passes it through rmsnorm_bwd_dp."""
    N = 4096
    ex = sharding.PeerDweightExchange(N)
    try:
        for seed in range(3):
            v = torch.randn(N, generator=torch.Generator().manual_seed(seed)).to(DEV)
            out = ex(v)
            assert torch.equal(out, ops.dw_reduce(v.view(1, N)))
        x, dy = cf.randn((64, N), seed=1).to(DEV), cf.randn((64, N), seed=2).to(DEV)
        w = cf.rmsnorm_weight(N, seed=3).to(DEV)
        _, rstd = ops.rmsnorm_fwd(x, w)
        dx, dw = sharding.rmsnorm_bwd_dp(dy, x, rstd, w, peer=ex)
        ex_dx, ex_dw = ops.rmsnorm_bwd(dy, x, rstd, w)
        assert torch.equal(dx, ex_dx) and torch.equal(dw, ex_dw)
        ops.check_status(torch.device(DEV))
    finally:
        ex.close()


def test_peer_exchanges_replay_from_a_cuda_graph():
    """Both peer kernels keep their call count on the device, so a captured
    launch replays correctly (one rank: the flags advance with every replay)."""
    N = 1024
    ex = sharding.PeerDweightExchange(N)
    ec = cf.EmbeddingCfg("peerg", (2, 64), 3000, 256)
    ids = cf.embedding_ids(ec).to(DEV)
    table = cf.randn((3000, 256), std=0.02, seed=4).to(DEV)
    emb = sharding.PeerVocabParallelEmbedding(ids.numel(), 256)
    try:
        v = torch.randn(N, device=DEV)
        out = torch.empty(N, device=DEV)
        ex(v, out=out)  # first call outside capture
        holder = {}
        emb(ids, table, 0, 3000)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ex(v, out=out)
            holder["y"] = emb(ids, table, 0, 3000)
        ref = ops.embedding_fwd(ids, table)
        for k in range(3):
            v.copy_(torch.randn(N, generator=torch.Generator().manual_seed(k)).to(DEV))
            out.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, ops.dw_reduce(v.view(1, N)))
            assert torch.equal(holder["y"], ref)
        ops.check_status(torch.device(DEV))
        del g
    finally:
        ex.close()
        emb.close()
