"""Multi-rank host logic of kernelproblems_b200.sharding on CPU ranks (gloo,
world size 2), with the CUDA kernels replaced by oracle functions: row
sharding, the dweight exchange (all-gather + fixed-order sum, and plain
all-reduce) of the RMSNorm backward and of the forward recomputed in it, the
vocab-parallel embedding forward (masked gather +
all-reduce) and backward (per-rank table-gradient shard), and host-side
failure detection (a rank that raises before a collective, and a rank that
stalls until the process group's timeout ends the other rank's collective), and the
collective setup and teardown of the peer-memory buffers (a rank that cannot
map its peer makes every rank release its buffers and raise)."""
import datetime
import os
import pickle
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _entry(rank, fn, port, q, timeout_s):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                                timeout=datetime.timedelta(seconds=timeout_s))
        res = fn(rank)
        # plain pickle copies tensors by value: a torch queue would pass them
        # through shared memory that this process may release before the
        # parent has read it
        q.put((rank, "ok", pickle.dumps(res)))
    except Exception as e:  # reported to the parent, which asserts on it
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-800:]}"))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def run_ranks(fn, timeout_s=30):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(r, fn, port, q, timeout_s)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(WORLD):
        r, status, res = q.get(timeout=timeout_s * 4)
        out[r] = (status, pickle.loads(res) if status == "ok" else res)
    for p in procs:
        p.join(timeout=timeout_s)
        if p.is_alive():
            p.kill()
    return out


# ---- rank bodies (module level so spawn can pickle them) -------------------

def _cpu_rms_bwd(dy, x, rstd, w, dy2=None, dres=None, eps=1e-6, dw_dtype=torch.float32):
    from oracle import fragments as F
    dxf, _ = F.add_rmsnorm_bwd(dy, dy2, x, rstd, w, dres)
    g = dy if dy2 is None else torch.ops.aten.add.Tensor(dy, dy2)
    return dxf, F.rmsnorm_dw_f64(g, x, rstd).float()


def _ordered_sum(parts):
    acc = torch.zeros(parts.shape[1], dtype=torch.float32)
    for i in range(parts.shape[0]):
        acc += parts[i]
    return acc


def _inputs(M=37, N=64):
    from kernelproblems_b200 import configs as cf
    from oracle import fragments as F
    x = cf.randn((M, N), seed=1)
    w = cf.rmsnorm_weight(N, seed=2)
    dy = cf.randn((M, N), seed=3)
    _, rstd = F.rmsnorm_fwd(x, w, 1e-6)
    return x, w, dy, rstd.reshape(M)


def _body_rms(rank, exact_order=True):
    from kernelproblems_b200 import sharding
    x, w, dy, rstd = _inputs()
    rows = sharding.local_rows(x.shape[0])
    sl = slice(rows.lo, rows.hi)
    dx, dw = sharding.rmsnorm_bwd_dp(dy[sl].contiguous(), x[sl].contiguous(), rstd[sl].contiguous(), w,
                                     exact_order=exact_order, bwd_fn=_cpu_rms_bwd,
                                     reduce_fn=_ordered_sum)
    return rows.lo, rows.hi, dx, dw


def _cpu_fwd_bwd(x, w, dy, x2=None, x3=None, dy2=None, dy3=None, dres=None, eps=1e-5,
                 write_y=True, dw_dtype=torch.float32):
    from oracle import fragments as F
    add = torch.ops.aten.add.Tensor
    h = x if x2 is None else add(x, x2)
    h = h if x3 is None else add(h, x3)
    g = dy if dy2 is None else add(dy, dy2)
    g = g if dy3 is None else add(g, dy3)
    y, rstd = F.rmsnorm_fwd(h, w, eps)
    dx, _ = F.rmsnorm_bwd(g, h, rstd, w)
    if dres is not None:
        dx = add(dres, dx)
    return (y if write_y else None), rstd, dx, F.rmsnorm_dw_f64(g, h, rstd).float()


def _fwd_bwd_inputs(M=37, N=64):
    from kernelproblems_b200 import configs as cf
    return ([cf.randn((M, N), seed=20 + i) for i in range(2)], cf.rmsnorm_weight(N, seed=22),
            [cf.randn((M, N), seed=23 + i) for i in range(2)], cf.randn((M, N), seed=25))


def _body_fwd_bwd(rank):
    from kernelproblems_b200 import sharding
    (x, x2), w, (dy, dy2), dres = _fwd_bwd_inputs()
    rows = sharding.local_rows(x.shape[0])
    sl = slice(rows.lo, rows.hi)
    y, dx, dw = sharding.rmsnorm_fwd_bwd_dp(
        x[sl].contiguous(), w, dy[sl].contiguous(), x2=x2[sl].contiguous(), dy2=dy2[sl].contiguous(),
        dres=dres[sl].contiguous(), fwd_bwd_fn=_cpu_fwd_bwd, reduce_fn=_ordered_sum)
    return rows.lo, rows.hi, y, dx, dw


def _body_rms_allreduce(rank):
    return _body_rms(rank, exact_order=False)


def _body_emb(rank):
    from kernelproblems_b200 import configs as cf
    from kernelproblems_b200 import sharding
    from oracle import fragments as F
    V, D = 50, 16
    ids = torch.randint(0, V, (3, 11), generator=torch.Generator().manual_seed(5))
    table = cf.randn((V, D), std=0.02, seed=6)
    sh = sharding.vocab_shard(V)
    out = sharding.embedding_fwd_vocab_parallel(
        ids, table[sh.lo:sh.hi].contiguous(), sh.lo, V,
        fwd_fn=lambda i, t, vocab_lo, vocab_total: F.embedding_fwd_vocab_shard(t, i, vocab_lo).float())
    grad = cf.randn((3, 11, D), seed=7)
    G = sharding.embedding_bwd_vocab_parallel(
        grad, ids, sh.lo, sh.n, V,
        bwd_fn=lambda g, i, n, vocab_lo, vocab_total, padding_idx: F.embedding_bwd_f64(
            g, i, n, padding_idx, vocab_lo))
    return sh.lo, sh.hi, out, G


def _body_rank1_raises(rank):
    t = torch.ones(4)
    if rank == 1:
        raise RuntimeError("rank 1 fails before the collective")
    dist.all_reduce(t)  # rank 0 must get an error, not hang
    return t


_STALL_S = 8.0


def _body_rank1_stalls(rank):
    """Rank 1 stays alive but never joins the collective: rank 0's collective
    must end with an error once the process group's timeout expires."""
    import time
    if rank == 1:
        time.sleep(_STALL_S)
        return None
    t0 = time.monotonic()
    try:
        dist.all_reduce(torch.ones(4))
    except Exception as e:  # the expected outcome
        return ("error", time.monotonic() - t0, f"{type(e).__name__}: {e}"[:200])
    return ("completed", time.monotonic() - t0, "")


def _peer_buffers_body(fail_rank):
    """_PeerBuffers with the device calls replaced by fakes: rank `fail_rank`
    cannot map its peer's buffer (-1: nobody fails)."""
    import contextlib

    from kernelproblems_b200 import _lib, sharding

    def body(rank):
        events = []

        class FakeLib:
            def frag_peer_close(self, p):
                events.append(("close", p.value))
                return 0

            def frag_peer_free(self, p):
                events.append(("free", p.value))
                return 0

        def fake_alloc(self, n):
            ptr = 4096 * (rank + 1) + 256 * len(self._own)
            self._own.append(ptr)
            return ptr, b"%d" % ptr

        def fake_open(self, h):
            if rank == fail_rank:
                raise _lib.FragError("frag_peer_open", 5)
            self._opened.append(int(h) + 1)
            return int(h) + 1

        sharding._PeerBuffers._alloc = fake_alloc
        sharding._PeerBuffers._open = fake_open
        _lib.load = lambda: FakeLib()
        torch.cuda.device = lambda d: contextlib.nullcontext()
        torch.cuda.synchronize = lambda *a, **k: None
        try:
            b = sharding._PeerBuffers([64, 256], None, torch.device("cpu"))
        except RuntimeError as e:
            return ("raised", str(e)[:200], events)
        ptrs = [list(row) for row in b.ptrs]
        b.close()
        return ("ok", ptrs, events)
    return body


def _peer_ok(rank):
    return _peer_buffers_body(-1)(rank)


def _peer_rank1_fails(rank):
    return _peer_buffers_body(1)(rank)


# ---- tests ------------------------------------------------------------------

@pytest.mark.parametrize("body", [_body_rms, _body_rms_allreduce])
def test_rmsnorm_bwd_dp_two_ranks(body):
    from oracle import fragments as F
    out = run_ranks(body)
    assert all(s == "ok" for s, _ in out.values()), out
    x, w, dy, rstd = _inputs()
    full_dx, _ = F.rmsnorm_bwd(dy, x, rstd, w)
    full_dw = F.rmsnorm_dw_f64(dy, x, rstd)
    dws = []
    for r in range(WORLD):
        lo, hi, dx, dw = out[r][1]
        assert torch.equal(dx, full_dx[lo:hi]), "local rows only, unchanged"
        assert torch.allclose(dw.double(), full_dw, rtol=1e-5, atol=1e-4)
        dws.append(dw)
    assert torch.equal(dws[0], dws[1]), "every rank holds the same dweight"


def test_rmsnorm_fwd_bwd_dp_two_ranks():
    from oracle import fragments as F
    out = run_ranks(_body_fwd_bwd)
    assert all(s == "ok" for s, _ in out.values()), out
    (x, x2), w, (dy, dy2), dres = _fwd_bwd_inputs()
    full_y, _, full_dx, _ = _cpu_fwd_bwd(x, w, dy, x2=x2, dy2=dy2, dres=dres)
    add = torch.ops.aten.add.Tensor
    h, g = add(x, x2), add(dy, dy2)
    _, rstd = F.rmsnorm_fwd(h, w, 1e-5)
    full_dw = F.rmsnorm_dw_f64(g, h, rstd)
    for r in range(WORLD):
        lo, hi, y, dx, dw = out[r][1]
        assert torch.equal(y, full_y[lo:hi]) and torch.equal(dx, full_dx[lo:hi]), "local rows only"
        assert torch.allclose(dw.double(), full_dw, rtol=1e-5, atol=1e-4)
    assert torch.equal(out[0][1][4], out[1][1][4]), "every rank holds the same dweight"


def test_vocab_parallel_embedding_two_ranks():
    from kernelproblems_b200 import configs as cf
    from oracle import fragments as F
    out = run_ranks(_body_emb)
    assert all(s == "ok" for s, _ in out.values()), out
    V, D = 50, 16
    ids = torch.randint(0, V, (3, 11), generator=torch.Generator().manual_seed(5))
    table = cf.randn((V, D), std=0.02, seed=6)
    full = F.embedding_fwd(table, ids)
    grad = cf.randn((3, 11, D), seed=7)
    Gfull = F.embedding_bwd_f64(grad, ids, V)
    covered = []
    for r in range(WORLD):
        lo, hi, o, G = out[r][1]
        assert torch.equal(o.to(torch.bfloat16), full), "all-reduced gather is the exact row"
        assert torch.equal(G, Gfull[lo:hi])
        covered.append((lo, hi))
    assert covered[0][0] == 0 and covered[-1][1] == V and covered[0][1] == covered[1][0]


def test_rank_failure_is_reported_not_hung():
    out = run_ranks(_body_rank1_raises, timeout_s=5)
    assert out[1][0] == "error" and "fails before" in out[1][1]
    assert out[0][0] == "error", "the surviving rank's collective must end with an error"


def test_stalled_rank_ends_collective_by_timeout():
    out = run_ranks(_body_rank1_stalls, timeout_s=3)
    assert out[0][0] == "ok", out[0]
    outcome, elapsed, msg = out[0][1]
    assert outcome == "error", "the waiting rank's collective must fail, not complete"
    assert elapsed < _STALL_S - 1.0, f"error came after {elapsed:.1f}s: the timeout did not end the wait"


def test_peer_buffers_map_every_peer_and_free_after_all_unmapped():
    out = run_ranks(_peer_ok)
    assert all(st == "ok" for st, _ in out.values()), out
    for r in range(WORLD):
        status, ptrs, events = out[r][1]
        assert status == "ok"
        own = [4096 * (r + 1), 4096 * (r + 1) + 256]
        peer = [4096 * (2 - r) + 1, 4096 * (2 - r) + 256 + 1]
        assert [row[r] for row in ptrs] == own and [row[1 - r] for row in ptrs] == peer
        # every mapping is closed before this rank frees its own buffers
        assert events == [("close", q) for q in peer] + [("free", q) for q in own]


def test_peer_buffers_fail_together_when_one_rank_cannot_map():
    out = run_ranks(_peer_rank1_fails)
    assert all(st == "ok" for st, _ in out.values()), out
    for r in range(WORLD):
        status, msg, events = out[r][1]
        assert status == "raised", "every rank raises, none is left waiting in a peer kernel"
        assert "peer buffers unavailable" in msg
        own = [4096 * (r + 1), 4096 * (r + 1) + 256]
        assert [e for e in events if e[0] == "free"] == [("free", q) for q in own], "own buffers released"
    assert "another rank" in out[0][1][1] and "frag_peer_open" in out[1][1][1]
