"""GPU parity: RMSNorm forward / add+RMSNorm forward / backward vs the CPU oracle."""
import pytest
import torch

from conftest import assert_bf16_close, assert_f32_close
from kernelproblems_b200 import configs as cf
from kernelproblems_b200 import ops
from oracle import fragments as ora

pytestmark = pytest.mark.gpu
DEV = "cuda"

FWD_SHAPES = [
    ((4, 2048, 4096), 1e-6),  # C0
    ((64, 4096), 1e-5),
    ((1, 4096), 1e-5),
    ((37, 8192), 1e-5),
    ((7, 16384), 1e-6),  # 4 chunks / thread
    ((5, 1000), 1e-5),  # N % 8 != 0 -> generic kernel
    ((3, 24), 1e-5),
    ((2, 20000), 1e-6),  # N > 16384 -> generic kernel
]


def _inputs(shape, seed=0):
    x = cf.randn(shape, seed=seed)
    w = cf.rmsnorm_weight(shape[-1], seed=seed + 1)
    return x, w


@pytest.mark.parametrize("shape,eps", FWD_SHAPES)
def test_rmsnorm_fwd(shape, eps):
    x, w = _inputs(shape)
    y, rstd = ops.rmsnorm_fwd(x.to(DEV), w.to(DEV), eps)
    ey, er = ora.rmsnorm_fwd(x, w, eps)
    assert_bf16_close(y, ey, "y")
    assert_f32_close(rstd, er.reshape(rstd.shape), "rstd")


def test_rmsnorm_fwd_unaligned_view():
    x, w = _inputs((9, 4097))
    xs = x[:, 1:].contiguous()  # fresh buffer, then view it at a 2-byte offset
    buf = torch.empty(xs.numel() + 1, dtype=torch.bfloat16, device=DEV)
    buf[1:].copy_(xs.flatten())
    xv = buf[1:].view(9, 4096)
    y, rstd = ops.rmsnorm_fwd(xv, w[1:].to(DEV), 1e-5)
    ey, er = ora.rmsnorm_fwd(xs, w[1:].contiguous(), 1e-5)
    assert_bf16_close(y, ey, "y")
    assert_f32_close(rstd, er.reshape(rstd.shape), "rstd")


@pytest.mark.parametrize("shape,eps", [((2, 1024, 8192), 1e-5), ((33, 4096), 1e-5), ((5, 1000), 1e-5)])
def test_add_rmsnorm_fwd(shape, eps):
    res = cf.randn(shape, seed=3)
    x = cf.randn(shape, seed=4)
    w = cf.rmsnorm_weight(shape[-1], seed=5)
    h, y, rstd = ops.add_rmsnorm_fwd(res.to(DEV), x.to(DEV), w.to(DEV), eps)
    eh, ey, er = ora.add_rmsnorm_fwd(res, x, w, eps)
    assert torch.equal(h.cpu(), eh), "h = bf16(res + x) must be bit exact"
    assert_bf16_close(y, ey, "y")
    assert_f32_close(rstd, er.reshape(rstd.shape), "rstd")


def _dw_atol(dy, x, rstd):
    """Absolute floor for near-zero dweight columns: 1e-4 * ||terms||_2."""
    N = x.shape[-1]
    t = dy.reshape(-1, N).double() * x.reshape(-1, N).double() * rstd.reshape(-1, 1).double()
    return 1e-4 * t.pow(2).sum(0).sqrt()


BWD_SHAPES = [
    (4, 2048, 4096),  # C1
    (100, 4096),
    (1, 4096),
    (33, 8192),
    (5, 1000),  # generic kernels
    (3, 24),
    (2, 20000),
]


@pytest.mark.parametrize("shape", BWD_SHAPES)
@pytest.mark.parametrize("variant", ["saved_rstd", "recompute", "add_add"])
def test_rmsnorm_bwd(shape, variant):
    eps = 1e-6
    x, w = _inputs(shape, seed=10)
    dy = cf.randn(shape, seed=12)
    _, rstd = ora.rmsnorm_fwd(x, w, eps)
    dy2 = cf.randn(shape, seed=13) if variant == "add_add" else None
    dres = cf.randn(shape, seed=14) if variant == "add_add" else None
    r_arg = None if variant == "recompute" else rstd.reshape(shape[:-1]).to(DEV)
    dx, dw = ops.rmsnorm_bwd(dy.to(DEV), x.to(DEV), r_arg, w.to(DEV),
                             dy2=None if dy2 is None else dy2.to(DEV),
                             dres=None if dres is None else dres.to(DEV), eps=eps)
    edx, _ = ora.add_rmsnorm_bwd(dy, dy2, x, rstd, w, dres)
    assert_bf16_close(dx, edx, "dx")
    g = dy if dy2 is None else torch.ops.aten.add.Tensor(dy, dy2)
    ref = ora.rmsnorm_dw_f64(g, x, rstd)
    assert_f32_close(dw, ref, "dw", atol=_dw_atol(g, x, rstd))


@pytest.mark.parametrize("shape", [(4, 2048, 4096), (33, 8192), (5, 1000)])
@pytest.mark.parametrize("rstd_saved", [True, False])
def test_rmsnorm_bwd_three_gradients(shape, rstd_saved):
    """dy = bf16(bf16(dy + dy2) + dy3) (v7/ed20955ec34b), TMA ring and generic kernels."""
    eps = 1e-5
    x, w = _inputs(shape, seed=40)
    dy, dy2, dy3, dres = (cf.randn(shape, seed=41 + j) for j in range(4))
    _, rstd = ora.rmsnorm_fwd(x, w, eps)
    r_arg = rstd.reshape(shape[:-1]).to(DEV) if rstd_saved else None
    dx, dw = ops.rmsnorm_bwd(dy.to(DEV), x.to(DEV), r_arg, w.to(DEV), dy2=dy2.to(DEV),
                             dy3=dy3.to(DEV), dres=dres.to(DEV), eps=eps)
    g = torch.ops.aten.add.Tensor(torch.ops.aten.add.Tensor(dy, dy2), dy3)
    edx, _ = ora.add_rmsnorm_bwd(g, None, x, rstd, w, dres)
    # bf16(dres + bf16(dx)): a one-ulp difference in the rounded dx survives
    # cancellation, so the bound scales with the summands
    mag = (edx.float() - dres.float()).abs() + dres.float().abs()
    assert_bf16_close(dx, edx, "d_res", atol=1e-2 + 1.6e-2 * mag)
    assert_f32_close(dw, ora.rmsnorm_dw_f64(g, x, rstd), "dw", atol=_dw_atol(g, x, rstd))


def test_rmsnorm_bwd_deterministic():
    shape = (4, 2048, 4096)
    x, w = _inputs(shape, seed=20)
    dy = cf.randn(shape, seed=21)
    _, rstd = ora.rmsnorm_fwd(x, w, 1e-6)
    args = (dy.to(DEV), x.to(DEV), rstd.reshape(shape[:-1]).to(DEV), w.to(DEV))
    _, dw1 = ops.rmsnorm_bwd(*args)
    _, dw2 = ops.rmsnorm_bwd(*args)
    assert torch.equal(dw1, dw2), "dweight must be bitwise reproducible"


def test_rmsnorm_bwd_bf16_dw_and_partials():
    shape = (300, 4096)
    x, w = _inputs(shape, seed=30)
    dy = cf.randn(shape, seed=31)
    _, rstd = ora.rmsnorm_fwd(x, w, 1e-6)
    dx, dwb, parts = ops.rmsnorm_bwd(dy.to(DEV), x.to(DEV), rstd.reshape(300).to(DEV), w.to(DEV),
                                     dw_dtype=torch.bfloat16, return_partials=True)
    assert dwb.dtype == torch.bfloat16
    full = ops.dw_reduce(parts.contiguous())
    assert torch.equal(full.to(torch.bfloat16), dwb)
    assert_f32_close(full, ora.rmsnorm_dw_f64(dy, x, rstd), "dw", atol=_dw_atol(dy, x, rstd))


def test_rmsnorm_bwd_empty_batch():
    w = cf.rmsnorm_weight(64).to(DEV)
    x = torch.empty(0, 64, dtype=torch.bfloat16, device=DEV)
    dx, dw = ops.rmsnorm_bwd(x, x, torch.empty(0, device=DEV), w)
    assert dx.shape == (0, 64) and torch.count_nonzero(dw) == 0
