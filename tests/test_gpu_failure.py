"""Device-side failure detection without a GPU fault.

* A bounded wait runs out: frag_selftest_bounded_wait waits, with the same
  wait every TMA kernel uses, on an mbarrier that nothing arrives on.  The
  wait must give up after its limit, set FRAG_DEVFLAG_WAIT_TIMEOUT in the
  library's error word (ops.check_status raises RuntimeError), and leave the
  context usable: a kernel launched afterwards still gives correct results.
* A RoPE position outside the freqs table (the reference's freqs_cis[pos]
  raises): the kernel reads nothing outside the table, flags
  FRAG_DEVFLAG_INDEX_OOB (ops.check_status raises IndexError) and copies that
  token unrotated; every other token is rotated as usual."""
import ctypes as C

import pytest
import torch

from conftest import assert_bf16_close
from kernelproblems_b200 import _lib, ops
from oracle import fragments as F

pytestmark = pytest.mark.gpu


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_bounded_wait_gives_up_and_context_survives():
    lib = _lib.load()
    torch.cuda.synchronize()
    lib.frag_device_errors(1)
    assert lib.frag_selftest_bounded_wait(2_000_000, _stream()) == 0   # ~1 ms at 2 GHz
    torch.cuda.synchronize()
    flags = lib.frag_device_errors(0)
    assert flags & _lib.FRAG_DEVFLAG_WAIT_TIMEOUT
    with pytest.raises(RuntimeError):
        ops.check_status()                       # reads and clears the word
    assert lib.frag_device_errors(0) == 0
    # the context is still usable
    g = torch.Generator().manual_seed(3)
    x = torch.randn(64, 4096, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(4096, generator=g)).bfloat16()
    y, rstd = ops.rmsnorm_fwd(x.cuda(), w.cuda(), 1e-5)
    torch.cuda.synchronize()
    y_ref, _ = F.rmsnorm_fwd(x, w, 1e-5)
    assert_bf16_close(y.cpu(), y_ref, "y after a timed-out wait")


def test_bounded_wait_rejects_bad_limits():
    lib = _lib.load()
    assert lib.frag_selftest_bounded_wait(0, _stream()) == 1  # FRAG_ERR_INVALID_ARG
    assert lib.frag_selftest_bounded_wait(5_000_000_000, _stream()) == 1  # FRAG_ERR_INVALID_ARG


@pytest.mark.parametrize("vec", [True, False])
def test_rope_position_outside_table_is_flagged(vec):
    S, H, D = 64, 4, 128 if vec else 6
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, S, H, D, generator=g).bfloat16()
    freqs = F.precompute_freqs_cis(D, S, 5e5)            # S rows
    pos = torch.arange(S, dtype=torch.int32)
    pos[7] = S                                           # one past the table
    pos[9] = -1
    ops.check_status()
    oq, _ = ops.rope(q.cuda(), None, pos.cuda().view(1, S), freqs=freqs.cuda(),
                     layout="interleaved")
    torch.cuda.synchronize()
    with pytest.raises(IndexError):
        ops.check_status()
    oq = oq.cpu()
    good = torch.ones(S, dtype=torch.bool)
    good[7] = good[9] = False
    ref = F.rope_interleaved(q[:, good], freqs[pos[good].long()].view(1, -1, 1, D // 2))
    assert_bf16_close(oq[:, good], ref, "valid tokens")
    assert torch.equal(oq[:, ~good], q[:, ~good]), "flagged tokens are copied unrotated"
