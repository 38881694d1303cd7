"""The peer-memory exchanges on two GPUs, one process each (NCCL only for
the one-time IPC handle exchange and the reference all-gather):
  * the fused vocab-parallel embedding forward: every rank's output equals
    the plain gather from the whole table bit for bit, over repeated calls,
    including ids outside the vocabulary;
  * the dweight exchange: every rank gets the fixed rank-order sum of the
    all-gathered per-rank vectors bit for bit, over repeated calls.
Skipped with fewer than two GPUs (the single-rank paths are in
test_gpu_sharding.py)."""
import datetime
import os
import pickle
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]
WORLD = 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, q):
    import torch.distributed as dist

    from kernelproblems_b200 import configs as cf
    from kernelproblems_b200 import ops, sharding
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    emb = None
    try:
        V, D = 10000, 1024
        full = cf.randn((V, D), std=0.02, seed=3).to(dev)
        sh = cf.shard_rows(V, WORLD, rank)
        shard = full[sh.lo:sh.hi].contiguous()
        ec = cf.EmbeddingCfg("peer2", (4, 512), V, D)
        ids = cf.embedding_ids(ec).to(dev)
        emb = sharding.PeerVocabParallelEmbedding(ids.numel(), D)
        ok = True
        for _ in range(4):
            out = emb(ids, shard, sh.lo, V)
            ok &= torch.equal(out, ops.embedding_fwd(ids, full))
        bad = ids.clone()
        bad[1, 7] = -3
        out = emb(bad, shard, sh.lo, V)
        ok &= int(torch.count_nonzero(out[1, 7])) == 0
        ok &= torch.equal(out[0], ops.embedding_fwd(ids[0], full))
        flags = ops._lib.load().frag_device_errors(1)
        dist.barrier()
        q.put(pickle.dumps((rank, bool(ok), int(flags))))
    except Exception as e:
        q.put(pickle.dumps((rank, False, repr(e))))
    finally:
        if emb is not None:
            emb.close()
        dist.destroy_process_group()


def _rank_dw(rank, port, q):
    import torch.distributed as dist

    from kernelproblems_b200 import ops, sharding
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    ex = None
    try:
        N = 8192
        ex = sharding.PeerDweightExchange(N)
        ok = True
        for step in range(5):
            v = torch.randn(N, generator=torch.Generator().manual_seed(100 * step + rank)).to(dev)
            got = ex(v)
            parts = torch.empty(WORLD, N, device=dev)
            dist.all_gather_into_tensor(parts.view(-1), v)
            ok &= torch.equal(got, ops.dw_reduce(parts))
        flags = ops._lib.load().frag_device_errors(1)
        dist.barrier()
        q.put(pickle.dumps((rank, bool(ok), int(flags))))
    except Exception as e:
        q.put(pickle.dumps((rank, False, repr(e))))
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


def _run(target):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [pickle.loads(q.get(timeout=300)) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_peer_vocab_parallel_two_gpus():
    for rank, ok, flags in _run(_rank):
        assert ok, f"rank {rank}: output differs from the full gather ({flags})"
        assert flags == 0, f"rank {rank}: device error flags {flags}"


def test_peer_dweight_exchange_two_gpus():
    for rank, ok, flags in _run(_rank_dw):
        assert ok, f"rank {rank}: exchanged dweight differs from the rank-order sum ({flags})"
        assert flags == 0, f"rank {rank}: device error flags {flags}"
