"""The reference's own Triton drop-ins (fetched into oracle/_ref/triton by
oracle/triton_ref.py, with the size patches listed there) against the CPU
oracle on seeded inputs, on the GPU this library runs on.

This is what the benchmark's Triton comparison rests on: the kernels it
times beside this library's are checked here to compute the same fragment.
Tolerances are the benchmark's: embedding gather bit exact, bf16 outputs
atol 1e-2 / rtol 1.6e-2, fp32 rstd / table gradient rtol 1e-4.  Where a
reference kernel rounds differently from its own graph the test says so.
"""
import pytest
import torch

from conftest import BF16_ATOL, assert_bf16_close, assert_f32_close
from kernelproblems_b200 import configs as cf
from oracle import fragments as ora
from oracle import triton_ref

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not triton_ref.available(),
                                 reason="oracle/_ref/triton missing: run oracle/triton_ref.py --reference <checkout>")]
DEV = "cuda"


def test_rmsnorm_fwd_c0():
    x = cf.randn((4, 2048, 4096), seed=1)
    w = cf.rmsnorm_weight(4096, seed=2)
    y, y2, rstd = triton_ref.kernel_function("v8/f4e9e58fef73")(x.to(DEV), w.to(DEV))
    ey, er = ora.rmsnorm_fwd(x, w, 1e-5)  # the problem's eps (hard-coded in the kernel)
    assert_bf16_close(y.view(ey.shape), ey, "y")
    assert y.data_ptr() == y2.data_ptr()
    assert_f32_close(rstd.reshape(-1), er.reshape(-1), "rstd")


def test_rmsnorm_bwd_c1():
    x, g = cf.randn((1, 8192, 4096), seed=3), cf.randn((1, 8192, 4096), seed=4)
    w = cf.rmsnorm_weight(4096, seed=5)
    dx, dw = triton_ref.kernel_function("v7/45990c83cfd6")(x.to(DEV), w.to(DEV), g.to(DEV), 1e-6)
    _, er = ora.rmsnorm_fwd(x, w, 1e-6)
    edx, _ = ora.rmsnorm_bwd(g, x, er, w)
    assert_bf16_close(dx, edx, "dx")
    assert dw.dtype == torch.bfloat16  # the kernel returns dweight in the weight's dtype
    assert_bf16_close(dw, ora.rmsnorm_dw_f64(g, x, er).to(torch.bfloat16), "dweight (bf16)")


def test_embedding_fwd_c2_bit_exact():
    c = cf.C2
    table = cf.randn((c.vocab * c.dim,), std=0.02, seed=6)
    ids = cf.embedding_ids(c)
    out = triton_ref.kernel_function("v7/1e49beb8a123")(table.to(DEV), ids.to(DEV))
    assert torch.equal(out.cpu(), ora.embedding_fwd(table.view(c.vocab, c.dim), ids))


def test_embedding_bwd_c2():
    """fp32 atomics in the reference kernel: summation order varies, the
    float64 sum is the accuracy reference.  Compared on the touched rows;
    every other row must be zero."""
    c = cf.EmbeddingCfg("c2-2k", (1, 2048), 128256, 4096)  # the kernel fixes vocab 128256
    ids = cf.embedding_ids(c)
    g = cf.randn((1, 2048, 4096), seed=7)
    G = triton_ref.kernel_function("v7/a12a160cb11b")(g.to(DEV), ids.to(DEV))
    u, inv = torch.unique(ids.reshape(-1), return_inverse=True)
    ref = ora.embedding_bwd_f64(g, inv, u.numel())
    assert_f32_close(G[u.to(DEV)], ref, "touched rows", atol=1e-5)
    untouched = torch.ones(c.vocab, dtype=torch.bool, device=DEV)
    untouched[u.to(DEV)] = False
    assert int(torch.count_nonzero(G[untouched])) == 0


def _pos_and_freqs(S_total, S_seq, theta=500000.0):
    pos = torch.arange(S_seq).repeat(S_total // S_seq)
    return pos, ora.precompute_freqs_cis(128, S_seq, theta)


def test_rope_fwd_c3_interleaved():
    T = 8192
    pos, fr = _pos_and_freqs(T, 4096)
    q, k = cf.randn((T, 4096), seed=8), cf.randn((T, 1024), seed=9)
    oq, ok = triton_ref.kernel_function("v8/c8c60d8f7015")(
        pos.view(1, T).to(torch.int32).to(DEV), fr.to(DEV), q.to(DEV), k.to(DEV))
    f = fr[pos].view(1, T, 1, 64)
    assert_bf16_close(oq, ora.rope_interleaved(q.view(1, T, 32, 128), f), "q")
    assert_bf16_close(ok, ora.rope_interleaved(k.view(1, T, 8, 128), f), "k")


@pytest.mark.parametrize("problem,H", [("v7/bfe872e373e4", 32), ("v7/5c65f62b0422", 8)])
def test_rope_bwd_c3_strided(problem, H):
    T = 8192
    pos, fr = _pos_and_freqs(T, 4096)
    conj = fr[pos].conj().resolve_conj().view(1, T, 1, 64)
    g = cf.randn((T * H * 128,), seed=10 + H).as_strided([1, H, T, 128], [T * H * 128, 128, H * 128, 1])
    out = triton_ref.kernel_function(problem)(g.to(DEV), conj.to(DEV))
    ref = ora.rope_interleaved(g.transpose(1, 2), conj).reshape(T, H * 128)
    assert_bf16_close(out, ref, "grad")


def test_add_rmsnorm_fwd_c4_width():
    """The reference kernel rounds x * rstd to bf16 before the weight
    multiply (v8/7884328a5557/optimized_kernel.py:32) where the graph
    multiplies in fp32: within the bf16 tolerance, not equal."""
    M, N = 2048, 8192
    mm, res = cf.randn((M, N), seed=12), cf.randn((1, M, N), seed=13)
    w = cf.rmsnorm_weight(N, seed=14)
    y, y2 = triton_ref.kernel_function("v8/7884328a5557")(mm.to(DEV), res.to(DEV), w.to(DEV))
    _, ey, _ = ora.add_rmsnorm_fwd(res, mm.view(1, M, N), w, 1e-5)
    assert_bf16_close(y, ey.view(M, N), "y")
    assert y.data_ptr() == y2.data_ptr()


def test_add_rmsnorm_bwd_c4_width():
    """dy = bf16(mm + view); d_res = bf16(dres + dx) -- the reference kernel
    adds the unrounded dx (v7/7f544ceb2120/optimized_kernel.py:45) where its
    graph rounds dx to bf16 first, so one ulp of |dx| is allowed on top of
    the bf16 tolerance; dweight fp32."""
    M, N = 2048, 8192
    w = cf.rmsnorm_weight(N, seed=15)
    h = cf.randn((1, M, N), seed=16)
    _, er = ora.rmsnorm_fwd(h, w, 1e-5)
    mm, v, dres = cf.randn((M, N), seed=17), cf.randn((1, M, N), seed=18), cf.randn((1, M, N), seed=19)
    out, dw = triton_ref.kernel_function("v7/7f544ceb2120")(
        mm.to(DEV), v.to(DEV), h.to(DEV), er.reshape(1, M, 1).to(DEV), w.to(DEV), dres.to(DEV))
    g = torch.ops.aten.add.Tensor(v, mm.view(1, M, N))
    edx, _ = ora.add_rmsnorm_bwd(g, None, h, er, w, dres)
    t = (edx.float() - dres.float()).abs().clamp_min(2.0 ** -126)
    ulp = torch.exp2(torch.floor(torch.log2(t)) - 7)
    assert_bf16_close(out, edx, "d_res", atol=BF16_ATOL + ulp)
    terms = g.double() * h.double() * er.reshape(1, M, 1).double()
    assert_f32_close(dw, ora.rmsnorm_dw_f64(g, h, er), "dweight",
                     atol=1e-4 * terms.pow(2).sum((0, 1)).sqrt())
