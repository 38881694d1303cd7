"""Caller-supplied output buffers on the GPU: a buffer of the wrong shape,
dtype or layout raises ValueError before the kernel could write past it, and
the partials returned for an unaligned call are laid out with the row blocks
that call actually used."""
import pytest
import torch

from conftest import assert_f32_close
from kernelproblems_b200 import configs as cf
from kernelproblems_b200 import ops
from oracle import fragments as ora

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_rmsnorm_fwd_out_checked():
    x = cf.randn((64, 4096), device=DEV, seed=1)
    w = cf.rmsnorm_weight(4096, device=DEV, seed=2)
    with pytest.raises(ValueError):
        ops.rmsnorm_fwd(x, w, out=torch.empty(63, 4096, dtype=torch.bfloat16, device=DEV))
    with pytest.raises(ValueError):
        ops.rmsnorm_fwd(x, w, out=torch.empty(64, 4096, dtype=torch.float32, device=DEV))
    with pytest.raises(ValueError):
        ops.rmsnorm_fwd(x, w, rstd=torch.empty(32, dtype=torch.float32, device=DEV))
    y = torch.empty_like(x)
    r = torch.empty(64, dtype=torch.float32, device=DEV)
    y2, r2 = ops.rmsnorm_fwd(x, w, out=y, rstd=r)
    assert y2 is y and r2 is r


def test_add_rmsnorm_fwd_outs_checked():
    x = cf.randn((8, 8192), device=DEV, seed=3)
    w = cf.rmsnorm_weight(8192, device=DEV, seed=4)
    with pytest.raises(ValueError):
        ops.add_rmsnorm_fwd(x, x, w, h_out=torch.empty(4, 8192, dtype=torch.bfloat16, device=DEV))
    with pytest.raises(ValueError):
        ops.add_rmsnorm_fwd(x, x, w, y_out=torch.empty(8192, 8, dtype=torch.bfloat16, device=DEV).t())


def test_embedding_outs_checked():
    ids = torch.randint(0, 100, (2, 16), device=DEV)
    table = cf.randn((100, 256), device=DEV, seed=5)
    with pytest.raises(ValueError):
        ops.embedding_fwd(ids, table, out=torch.empty(2, 15, 256, dtype=torch.bfloat16, device=DEV))
    g = cf.randn((2, 16, 256), device=DEV, seed=6)
    with pytest.raises(ValueError):
        ops.embedding_bwd(g, ids, 100, out=torch.empty(99, 256, dtype=torch.float32, device=DEV))
    with pytest.raises(ValueError):
        ops.embedding_bwd(g, ids, 100, out=torch.empty(100, 256, dtype=torch.bfloat16, device=DEV))
    x = cf.randn((32, 256), device=DEV, seed=7)
    w = cf.rmsnorm_weight(256, device=DEV, seed=8)
    with pytest.raises(ValueError):
        ops.rmsnorm_embedding_bwd(x, w, ids, x, 100,
                                  out=torch.empty(100, 128, dtype=torch.float32, device=DEV))


def test_dw_reduce_out_checked():
    parts = torch.randn(5, 64, device=DEV)
    with pytest.raises(ValueError):
        ops.dw_reduce(parts, out=torch.empty(63, device=DEV))
    with pytest.raises(ValueError):
        ops.dw_reduce(parts, out_bf16=torch.empty(64, device=DEV))


def test_partials_of_an_unaligned_call_use_its_row_blocks():
    """An input at an odd storage offset takes the generic kernels, whose row
    blocks differ from the ring kernel's: the returned partials must still
    sum to dweight."""
    M, N = 300, 4096
    x, dy = cf.randn((M, N), seed=9), cf.randn((M, N), seed=10)
    w = cf.rmsnorm_weight(N, seed=11)
    _, rstd = ora.rmsnorm_fwd(x, w, 1e-6)
    buf = torch.empty(M * N + 1, dtype=torch.bfloat16, device=DEV)
    buf[1:].copy_(dy.flatten())
    dyv = buf[1:].view(M, N)  # 2-byte offset: not 16-byte aligned
    dx, dw, parts = ops.rmsnorm_bwd(dyv, x.to(DEV), rstd.reshape(M).to(DEV), w.to(DEV),
                                    return_partials=True)
    assert torch.equal(ops.dw_reduce(parts.contiguous()), dw)
    terms = dy.double() * x.double() * rstd.reshape(M, 1).double()
    assert_f32_close(dw, ora.rmsnorm_dw_f64(dy, x, rstd), "dw",
                     atol=1e-4 * terms.pow(2).sum(0).sqrt())
