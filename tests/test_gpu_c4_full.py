"""Configuration C4 at its own size: residual add + RMSNorm forward and its
backward over res, x [16, 8192, 8192] (131,072 rows of width 8192, 2 GiB per
tensor, about 16 GB on the device at once).

At this size the backward's row blocks are ~886 rows per CTA (one CTA per
SM) and every row offset needs 64-bit arithmetic past 2^30 elements, so
smaller cases do not cover it.  Checked:
  * a few hundred sampled rows -- the first and last rows, both rows on each
    side of every row-block boundary of the backward's partition, and seeded
    random rows -- against the CPU oracle: h bit exact, y and d_res within
    the bf16 tolerance, rstd within rtol 1e-4;
  * rstd of every row against a float64 torch reference on the GPU;
  * dweight against the float64 column sum over all rows (GPU, chunked),
    rtol 1e-4 with a floor of 1e-4 x the column's L2 norm.
"""
import pytest
import torch

from conftest import assert_bf16_close, assert_f32_close
from kernelproblems_b200 import configs as cf
from kernelproblems_b200 import ops
from oracle import fragments as ora

pytestmark = pytest.mark.gpu
DEV = "cuda"
C = cf.C4
M, N, EPS = C.M, C.N, C.eps


def _sample_rows(G: int) -> list[int]:
    rpb = -(-M // G)
    rows = {0, 1, M - 2, M - 1}
    for b in range(1, G):
        rows |= {b * rpb - 1, b * rpb}
    g = torch.Generator().manual_seed(4)
    rows |= set(torch.randint(0, M, (64,), generator=g).tolist())
    return sorted(r for r in rows if 0 <= r < M)


def _rows(t: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    return t.reshape(M, -1)[idx].cpu()


def test_c4_forward_and_backward_at_full_size():
    w = cf.rmsnorm_weight(N, device=DEV, seed=20)
    res = cf.randn(C.shape, device=DEV, seed=21)
    x = cf.randn(C.shape, device=DEV, seed=22)
    h, y, rstd = ops.add_rmsnorm_fwd(res, x, w, EPS)
    G = ops.rmsnorm_bwd_num_blocks(M, N)
    rows = _sample_rows(G)
    idx = torch.tensor(rows, device=DEV)
    wc = w.cpu()
    eh, ey, er = ora.add_rmsnorm_fwd(_rows(res, idx), _rows(x, idx), wc, EPS)
    assert torch.equal(_rows(h, idx), eh), "h = bf16(res + x) must be bit exact"
    assert_bf16_close(_rows(y, idx), ey, "y")
    assert_f32_close(rstd.reshape(M)[idx].cpu(), er.reshape(-1), "rstd (sampled rows)")
    hm = h.reshape(M, N)
    r64 = torch.cat([torch.rsqrt(hm[i:i + 4096].double().pow(2).mean(-1) + EPS)
                     for i in range(0, M, 4096)])
    assert_f32_close(rstd.reshape(M), r64, "rstd (every row, float64 reference)")
    del res, x, y
    torch.cuda.empty_cache()

    dy = cf.randn(C.shape, device=DEV, seed=24)
    dh = cf.randn(C.shape, device=DEV, seed=25)
    d_res, dw = ops.rmsnorm_bwd(dy, h, rstd, w, dres=dh, eps=EPS)
    dh_s = _rows(dh, idx)
    edx, _ = ora.add_rmsnorm_bwd(_rows(dy, idx), None, eh, er, wc, dh_s)
    # bf16(dres + bf16(dx)): a one-ulp difference in the rounded dx survives
    # cancellation, so the bound scales with the summands
    mag = (edx.float() - dh_s.float()).abs() + dh_s.float().abs()
    assert_bf16_close(_rows(d_res, idx), edx, "d_res", atol=1e-2 + 1.6e-2 * mag)
    s = torch.zeros(N, dtype=torch.float64, device=DEV)
    q = torch.zeros_like(s)
    dym, rm = dy.reshape(M, N), rstd.reshape(M)
    for i in range(0, M, 4096):
        t = dym[i:i + 4096].double() * hm[i:i + 4096].double() * rm[i:i + 4096, None].double()
        s += t.sum(0)
        q += t.pow(2).sum(0)
    assert_f32_close(dw, s, "dweight (float64 column sum over all rows)", atol=1e-4 * q.sqrt().cpu())
