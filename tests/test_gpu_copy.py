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


def _layer_buffer(world, splits, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(world * sum(splits), generator=g, device="cuda").to(torch.bfloat16)


@pytest.mark.parametrize("world,splits", [
    (8, [512, 2097152, 524288, 524288, 2097152, 512, 7340032, 7340032]),   # one decoder layer
    (8, [512, 65667072]),                                                  # norm weight + table
    (3, [8, 1000, 24, 4096, 40]),
    (2, [8] * 16),                                                        # the segment limit
    (5, [0, 64, 0, 128]),                                                 # empty splits
])
def test_copy_rows_grouped_splits(world, splits):
    flat = _layer_buffer(world, splits, world * 31 + len(splits))
    parts = torch.split(flat.view(world, -1), splits, dim=1)
    outs = ops.copy_rows_grouped(parts)
    assert len(outs) == len(parts)
    for o, v in zip(outs, parts):
        assert o.is_contiguous() and o.shape == v.shape
        assert torch.equal(o, v.contiguous())


def test_copy_rows_grouped_into_outs_and_unaligned():
    flat = _layer_buffer(4, [40, 24, 8], 5)
    parts = torch.split(flat.view(4, -1), [40, 24, 8], dim=1)
    outs = [torch.full(p.shape, 7.0, device="cuda", dtype=torch.bfloat16) for p in parts]
    got = ops.copy_rows_grouped(parts, [outs[0], None, outs[2]])
    assert got[0] is outs[0] and got[2] is outs[2]
    for o, v in zip(got, parts):
        assert torch.equal(o, v.contiguous())
    # rows 2 bytes off 16-byte alignment: one frag_copy_rows per segment
    odd = torch.split(flat.view(4, -1)[:, 1:], [39, 24, 8], dim=1)
    for o, v in zip(ops.copy_rows_grouped(odd), odd):
        assert torch.equal(o, v.contiguous())


def test_copy_rows_grouped_errors():
    flat = _layer_buffer(2, [8] * 17, 9)
    parts = torch.split(flat.view(2, -1), [8] * 17, dim=1)
    with pytest.raises(ValueError):
        ops.copy_rows_grouped(parts)                       # 17 > 16 segments
    with pytest.raises(ValueError):
        ops.copy_rows_grouped(parts[:2], [None])           # outs length
    assert ops.copy_rows_grouped([]) == []


@pytest.mark.parametrize("shape,src_dt,dst_dt", [
    ((1, 8192, 32, 128), torch.bfloat16, torch.float32),    # the RoPE input widening
    ((1, 8192, 8, 128), torch.float32, torch.bfloat16),     # the RoPE result rounding
    ((37, 1000), torch.float32, torch.bfloat16),
    ((5, 13), torch.bfloat16, torch.float32),                # cols % 8 != 0: element kernel
    ((64, 256), torch.float32, torch.float32),
])
def test_convert(shape, src_dt, dst_dt):
    g = torch.Generator(device="cuda").manual_seed(len(shape) * 100 + shape[-1])
    x = (torch.randn(shape, generator=g, device="cuda") * 3).to(src_dt)
    y = ops.convert(x, dst_dt)
    assert y.dtype == dst_dt and y.shape == x.shape and y.is_contiguous()
    assert torch.equal(y, x.to(dst_dt)), "conversion must match torch's _to_copy bit for bit"


def test_convert_strided_two_copies_and_errors():
    g = torch.Generator(device="cuda").manual_seed(7)
    base = torch.randn(64, 160, generator=g, device="cuda")
    rows = base[:, 16:144]                                    # rows 160 apart, 128 wide
    a, b = ops.convert(rows, torch.bfloat16, copies=2)
    assert a.data_ptr() != b.data_ptr()
    assert torch.equal(a, rows.to(torch.bfloat16)) and torch.equal(b, a)
    odd = base[:, 1:130]                                      # unaligned rows: element kernel
    assert torch.equal(ops.convert(odd, torch.bfloat16), odd.to(torch.bfloat16))
    t = torch.randn(8, 4, 16, generator=g, device="cuda").transpose(0, 1)   # [4, 8, 16] view
    with pytest.raises(ValueError):
        ops.convert(t, torch.bfloat16)                        # rows do not collapse
    with pytest.raises(TypeError):
        ops.convert(base.to(torch.float16), torch.float32)
    with pytest.raises(ValueError):
        ops.convert(base, torch.float32, copies=3)
