"""GPU parity: RoPE (neox and interleaved, computed and table cos/sin, forward
and inverse, strided views) vs the CPU oracle."""
import pytest
import torch

from conftest import assert_bf16_close
from kernelproblems_b200 import configs as cf
from kernelproblems_b200 import ops
from oracle import fragments as ora

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_rope_neox_c3_fwd_bwd():
    c = cf.C3
    q = cf.randn((c.B, c.S, c.Hq, c.D), seed=40)
    k = cf.randn((c.B, c.S, c.Hk, c.D), seed=41)
    pos = cf.rope_positions(c)
    oq, ok = ops.rope(q.to(DEV), k.to(DEV), pos.to(DEV), theta=c.theta)
    assert_bf16_close(oq, ora.rope_neox(q, pos, c.theta), "q")
    assert_bf16_close(ok, ora.rope_neox(k, pos, c.theta), "k")
    gq = cf.randn((c.B, c.S, c.Hq, c.D), seed=42)
    gk = cf.randn((c.B, c.S, c.Hk, c.D), seed=43)
    dq, dk = ops.rope(gq.to(DEV), gk.to(DEV), pos.to(DEV), theta=c.theta, inverse=True)
    assert_bf16_close(dq, ora.rope_neox(gq, pos, c.theta, inverse=True), "dq")
    assert_bf16_close(dk, ora.rope_neox(gk, pos, c.theta, inverse=True), "dk")


def test_rope_round_trip_full_size():
    c = cf.C3
    q = cf.randn((c.B, c.S, c.Hq, c.D), device=DEV, seed=44)
    pos = cf.rope_positions(c, device=DEV)
    oq, _ = ops.rope(q, None, pos, theta=c.theta)
    back, _ = ops.rope(oq, None, pos, theta=c.theta, inverse=True)
    # rotation then its inverse: identity up to two bf16 roundings
    assert_bf16_close(back, q, "inverse(rope(q))", atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("layout", ["neox", "interleaved"])
@pytest.mark.parametrize("B,S,H,D", [(1, 7, 3, 128), (2, 33, 5, 64), (1, 4, 2, 32), (1, 5, 4, 96), (1, 3, 2, 256)])
def test_rope_shapes(layout, B, S, H, D):
    x = cf.randn((B, S, H, D), seed=B * 100 + S)
    pos = torch.randint(0, 5000, (B, S), generator=torch.Generator().manual_seed(S))
    o, _ = ops.rope(x.to(DEV), None, pos.to(DEV), theta=10000.0, layout=layout)
    if layout == "neox":
        ref = ora.rope_neox(x, pos, 10000.0)
    else:
        ref = ora.rope_interleaved_theta(x, pos, 10000.0)
    assert_bf16_close(o, ref, f"{layout} D={D}")


def test_rope_interleaved_table_reference_fragment():
    """v8/c8c60d8f7015: int32 positions index a random complex64 freqs table."""
    S, Hq, Hk, D = 8192, 32, 8, 128
    g = torch.Generator().manual_seed(50)
    pos = torch.randint(0, 100, (1, S), generator=g, dtype=torch.int32)
    freqs = torch.randn((S, D // 2), dtype=torch.complex64, generator=g)
    q = cf.randn((1, S, Hq, D), seed=51)
    k = cf.randn((1, S, Hk, D), seed=52)
    oq, ok = ops.rope(q.to(DEV), k.to(DEV), pos.to(DEV), freqs=freqs.to(DEV), layout="interleaved")
    f = freqs[pos.squeeze(0).long()].view(1, S, 1, D // 2)
    assert_bf16_close(oq, ora.rope_interleaved(q, f), "q")
    assert_bf16_close(ok, ora.rope_interleaved(k, f), "k")


def test_rope_interleaved_table_strided_bwd_fragment():
    """v7/bfe872e373e4: grad arrives as a [1, H, S, D] transposed view of [S, H, D]
    storage; freqs indexed by token."""
    S, H, D = 8192, 32, 128
    g = torch.Generator().manual_seed(60)
    store = cf.randn((S * H * D,), seed=61)
    gv = store.as_strided((1, H, S, D), (S * H * D, D, H * D, 1))
    freqs = torch.randn((1, S, 1, D // 2), dtype=torch.complex64, generator=g)
    x = gv.transpose(1, 2)  # [1, S, H, D] view, strides (.., H*D, D, 1)
    xd = store.to(DEV).as_strided((1, H, S, D), (S * H * D, D, H * D, 1)).transpose(1, 2)
    o, _ = ops.rope(xd, None, None, freqs=freqs.to(DEV).reshape(S, D // 2), layout="interleaved")
    assert_bf16_close(o, ora.rope_interleaved(x, freqs), "grad")


def test_rope_in_place():
    x = cf.randn((2, 16, 4, 128), seed=70)
    pos = torch.arange(16)
    xd = x.to(DEV)
    ops.rope(xd, None, pos.to(DEV), theta=500000.0, out_q=xd)
    assert_bf16_close(xd, ora.rope_neox(x, pos, 500000.0), "in place")


@pytest.mark.parametrize("D", [128, 6])
def test_rope_fp32_output_is_unrounded(D):
    """out_q in float32 (v7/0f38bc55457c returns q that way): the rotated
    values of the bf16 input, not rounded; k still bf16."""
    from conftest import assert_f32_close
    S, Hq, Hk = 32, 4, 2
    g = torch.Generator().manual_seed(31)
    q = torch.randn(1, S, Hq, D, generator=g).bfloat16()
    k = torch.randn(1, S, Hk, D, generator=g).bfloat16()
    freqs = torch.randn(64, D // 2, generator=g, dtype=torch.complex64)
    pos = torch.randint(0, 64, (1, S), generator=g, dtype=torch.int32)
    oq = torch.empty(1, S, Hq, D, dtype=torch.float32, device="cuda")
    oq, ok = ops.rope(q.cuda(), k.cuda(), pos.cuda(), freqs=freqs.cuda(), layout="interleaved",
                      out_q=oq)
    f = freqs[pos[0].long()].view(1, S, 1, D // 2)
    ref_q = torch.view_as_real(torch.view_as_complex(q.float().reshape(1, S, Hq, -1, 2)) * f).reshape(q.shape)
    assert oq.dtype == torch.float32 and ok.dtype == torch.bfloat16
    assert_f32_close(oq.cpu(), ref_q, "fp32 q", rtol=1e-5, atol=1e-5)
    assert_bf16_close(ok.cpu(), ora.rope_interleaved(k, f), "bf16 k")


@pytest.mark.parametrize("D2,Hq,Hk", [(64, 32, 8), (12, 3, 2), (8, 4, 0)])
def test_rope_complex64(D2, Hq, Hk):
    """ops.rope_complex (fp32 inputs, the v1/v2 snapshots' complex multiply):
    complex64 q, k times freqs[pos], fp32 throughout; D/2 = 12 takes the
    generic kernel."""
    from conftest import assert_f32_close
    S = 48
    g = torch.Generator().manual_seed(D2 + Hq)
    q = torch.randn(1, S, Hq, D2, generator=g, dtype=torch.complex64)
    k = torch.randn(1, S, Hk, D2, generator=g, dtype=torch.complex64) if Hk else None
    freqs = torch.randn(100, D2, generator=g, dtype=torch.complex64)
    pos = torch.randint(0, 100, (1, S), generator=g, dtype=torch.int32)
    oq, ok = ops.rope_complex(q.cuda(), None if k is None else k.cuda(), pos.cuda(), freqs.cuda())
    f = freqs[pos[0].long()].view(1, S, 1, D2)
    assert oq.dtype == torch.complex64 and oq.shape == q.shape
    assert_f32_close(torch.view_as_real(oq.cpu()), torch.view_as_real(q * f), "q", rtol=1e-5, atol=1e-5)
    if k is not None:
        assert_f32_close(torch.view_as_real(ok.cpu()), torch.view_as_real(k * f), "k", rtol=1e-5,
                         atol=1e-5)
    # the backward: multiply by the conjugate table
    gq, _ = ops.rope_complex(oq, None, pos.cuda(), freqs.cuda(), inverse=True)
    assert_f32_close(torch.view_as_real(gq.cpu()), torch.view_as_real(q * f * f.conj()), "q round trip",
                     rtol=1e-4, atol=1e-4)


def test_rope_complex64_errors():
    q = torch.zeros(1, 4, 2, 64, dtype=torch.complex64, device="cuda")
    qr = torch.view_as_real(q).flatten(-2)
    f = torch.zeros(4, 64, dtype=torch.complex64, device="cuda")
    with pytest.raises(ValueError):
        ops.rope(qr, None, None, freqs=f, layout="neox", out_q=torch.empty_like(qr))
    with pytest.raises(TypeError):
        ops.rope(qr, None, None, freqs=f, layout="interleaved",
                 out_q=torch.empty(qr.shape, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(TypeError):
        ops.rope_complex(qr, None, None, f)          # not complex
