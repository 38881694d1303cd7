"""Host-side checks of the ops layer that need no GPU: a caller-supplied
output buffer must match what the kernel writes (shape or element count,
dtype, contiguity, device), or the call raises before any launch."""
import pytest
import torch

from kernelproblems_b200 import ops

CPU = torch.device("cpu")


def test_check_out_accepts_the_exact_buffer():
    t = torch.empty(4, 8, dtype=torch.bfloat16)
    assert ops._check_out(t, "out", torch.bfloat16, CPU, shape=(4, 8)) is t
    r = torch.empty(2, 2, dtype=torch.float32)
    assert ops._check_out(r, "rstd", torch.float32, CPU, numel=4) is r


@pytest.mark.parametrize("bad,kw", [
    (torch.empty(4, 7, dtype=torch.bfloat16), dict(shape=(4, 8))),        # too small
    (torch.empty(5, 8, dtype=torch.bfloat16), dict(shape=(4, 8))),        # too large
    (torch.empty(4, 8, dtype=torch.float32), dict(shape=(4, 8))),         # wrong dtype
    (torch.empty(8, 4, dtype=torch.bfloat16).t(), dict(shape=(4, 8))),    # not contiguous
    (torch.empty(3, dtype=torch.bfloat16), dict(numel=4)),                # element count
])
def test_check_out_rejects_a_wrong_buffer(bad, kw):
    with pytest.raises(ValueError):
        ops._check_out(bad, "out", torch.bfloat16, CPU, **kw)


def test_check_out_rejects_another_device():
    t = torch.empty(4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops._check_out(t, "out", torch.bfloat16, torch.device("cuda", 0), shape=(4, 8))


def test_check_out_rejects_a_non_tensor():
    with pytest.raises(TypeError):
        ops._check_out([0] * 4, "out", torch.bfloat16, CPU, numel=4)
