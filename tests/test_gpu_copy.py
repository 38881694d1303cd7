"""ops.copy_rows (frag_copy_rows): the FSDP unshard copy, bit exact against
torch's own contiguous copy of the same strided view, over the vector kernel
(16-byte aligned rows) and the byte kernel (anything else)."""
import pytest
import torch

from kernelproblems_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,row,gap", [(8, 16032 * 4096, 512), (8, 512, 65667072 // 1024),
                                           (3, 1000, 24), (1, 4096, 0), (5, 7, 3), (64, 40, 8)])
def test_copy_rows_from_flat_buffer(world, row, gap):
    g = torch.Generator(device="cuda").manual_seed(world * 7 + row)
    flat = torch.randn(world * (row + gap), generator=g, device="cuda").to(torch.bfloat16)
    view = flat.view(world, row + gap)[:, gap:]       # [world, row], rows strided apart
    out = ops.copy_rows(view)
    assert out.is_contiguous() and out.shape == (world, row)
    assert torch.equal(out, view.contiguous())


def test_copy_rows_unaligned_and_fp32():
    base = torch.arange(4 * 37 + 1, dtype=torch.float32, device="cuda")
    view = base[1:].view(4, 37)                       # 4-byte aligned only
    assert torch.equal(ops.copy_rows(view), view.contiguous())
    b16 = torch.arange(6 * 33 + 3, device="cuda").to(torch.bfloat16)
    v16 = b16[3:].view(6, 33)
    assert torch.equal(ops.copy_rows(v16), v16.contiguous())


def test_copy_rows_empty_and_errors():
    e = torch.empty(0, 16, device="cuda", dtype=torch.bfloat16)
    assert ops.copy_rows(e).shape == (0, 16)
    with pytest.raises(ValueError):
        ops.copy_rows(torch.zeros(4, 4, device="cuda").t())   # columns not contiguous
