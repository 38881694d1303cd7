"""GPU parity of frag_rmsnorm_fwd_bwd (ops.rmsnorm_fwd_bwd): the RMSNorm
forward recomputed inside its backward, against the CPU oracle composed from
the same aten ops (bf16 adds of the inputs, _fused_rms_norm, the backward,
the residual add), over the TMA-ring kernel (16-byte aligned rows) and the
generic kernels (any other shape or alignment)."""
import pytest
import torch

from conftest import assert_bf16_close, assert_bf16_sum_close, assert_f32_close
from kernelproblems_b200 import configs as cf
from kernelproblems_b200 import ops
from oracle import fragments as ora

pytestmark = pytest.mark.gpu
DEV = "cuda"
add = torch.ops.aten.add.Tensor


def _oracle(xs, w, dys, dres, eps):
    h = xs[0]
    for t in xs[1:]:
        h = add(h, t)
    g = dys[0]
    for t in dys[1:]:
        g = add(g, t)
    y, rstd = ora.rmsnorm_fwd(h, w, eps)
    dx, _ = ora.rmsnorm_bwd(g, h, rstd, w)
    out = add(dres, dx) if dres is not None else dx
    return y, rstd.reshape(-1), out, ora.rmsnorm_dw_f64(g, h, rstd)


# (shape, x terms, dy terms, dres)
CASES = [
    ((1, 8192, 4096), 1, 3, True),    # v6/822931829090
    ((1, 8192, 4096), 2, 2, True),    # v6/408ac0979ac5
    ((1, 8192, 4096), 3, 1, False),   # v8/3c6c589cdf81
    ((2, 512, 8192), 3, 3, True),     # every input, width 8192
    ((300, 2048), 2, 1, False),
    ((37, 1000), 2, 2, True),         # N % 8 != 0: generic kernels
    ((5, 24), 3, 3, True),
]


@pytest.mark.parametrize("shape,nx,ndy,has_dres", CASES)
def test_rmsnorm_fwd_bwd(shape, nx, ndy, has_dres):
    N = shape[-1]
    xs = [cf.randn(shape, seed=10 + i) for i in range(nx)]
    dys = [cf.randn(shape, seed=20 + i) for i in range(ndy)]
    dres = cf.randn(shape, seed=30) if has_dres else None
    w = cf.rmsnorm_weight(N, seed=31)
    g = [t.to(DEV) for t in xs + dys]
    y, rstd, dx, dw = ops.rmsnorm_fwd_bwd(
        g[0], w.to(DEV), g[nx], x2=g[1] if nx > 1 else None, x3=g[2] if nx > 2 else None,
        dy2=g[nx + 1] if ndy > 1 else None, dy3=g[nx + 2] if ndy > 2 else None,
        dres=None if dres is None else dres.to(DEV), eps=1e-5, save_rstd=True)
    ey, er, edx, edw = _oracle(xs, w, dys, dres, 1e-5)
    assert_bf16_close(y, ey, "y")
    assert_f32_close(rstd, er, "rstd")
    if dres is None:
        assert_bf16_close(dx, edx, "dx")
    else:
        assert_bf16_sum_close(dx, edx, dres, "dres + dx")
    assert_f32_close(dw, edw, "dweight vs float64", atol=1e-3)


def test_rmsnorm_fwd_bwd_unaligned_and_options():
    # operands 2 bytes off 16-byte alignment take the generic kernels
    shape = (33, 4096)
    xs = [cf.randn(shape, seed=40 + i) for i in range(2)]
    dy = cf.randn(shape, seed=43)
    w = cf.rmsnorm_weight(4096, seed=44)
    buf = torch.empty(xs[0].numel() + 1, dtype=torch.bfloat16, device=DEV)
    buf[1:].copy_(xs[0].flatten())
    x0 = buf[1:].view(shape)
    y, rstd, dx, dw = ops.rmsnorm_fwd_bwd(x0, w.to(DEV), dy.to(DEV), x2=xs[1].to(DEV), eps=1e-5,
                                          write_y=False, dw_dtype=torch.bfloat16)
    assert y is None and rstd is None and dw.dtype == torch.bfloat16
    _, _, edx, edw = _oracle(xs, w, [dy], None, 1e-5)
    assert_bf16_close(dx, edx, "dx")
    assert_bf16_close(dw.float(), edw.float(), "dweight bf16", atol=5e-2)
    # the fused forward rounds rstd like the forward kernel
    h = add(xs[0], xs[1])
    y2, r2, _, _ = ops.rmsnorm_fwd_bwd(h.to(DEV), w.to(DEV), dy.to(DEV), eps=1e-5, save_rstd=True)
    fy, fr = ops.rmsnorm_fwd(h.to(DEV), w.to(DEV), 1e-5)
    assert_bf16_close(y2, fy, "y vs the forward kernel")
    assert_f32_close(r2, fr, "rstd vs the forward kernel")


def test_rmsnorm_fwd_bwd_empty_and_errors():
    w = cf.rmsnorm_weight(64, seed=1).to(DEV)
    e = torch.empty(0, 64, dtype=torch.bfloat16, device=DEV)
    y, _, dx, dw = ops.rmsnorm_fwd_bwd(e, w, e)
    torch.cuda.synchronize()
    assert y.shape == (0, 64) and dx.shape == (0, 64) and torch.count_nonzero(dw) == 0
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        ops.rmsnorm_fwd_bwd(x, w, x, x3=x)          # x3 without x2
    with pytest.raises(ValueError):
        ops.rmsnorm_fwd_bwd(x, w, x, dy3=x)         # dy3 without dy2
    with pytest.raises(ValueError):
        ops.rmsnorm_fwd_bwd(x, w, x[:2])            # shapes differ
