"""Pin the oracle: on the seeded golden inputs, every per-problem oracle must
reproduce the reference Model's CPU outputs bit for bit (sha256 recorded by
tests/golden/make_golden.py from the reference's own problem.py)."""
import hashlib
import sys
from pathlib import Path

import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

from inputs import make_inputs  # noqa: E402
from conftest import ORACLE_PREFIX as PREFIX  # noqa: E402
from oracle.problems import ORACLES  # noqa: E402

FIXTURES = sorted(GOLDEN.glob("v*_*.pt"))


def _sha(t):
    c = t.detach().contiguous()
    if c.dtype == torch.complex64:
        c = torch.view_as_real(c)
    return hashlib.sha256(c.view(torch.uint8).numpy().tobytes()).hexdigest()


def test_every_registered_problem_has_a_fixture():
    from kernelproblems_b200.problems import PROBLEMS
    have = {f.stem.replace("_", "/", 1) for f in FIXTURES}
    assert set(PROBLEMS) <= have
    assert set(PROBLEMS) == set(ORACLES)



@pytest.mark.parametrize("fixture", FIXTURES, ids=lambda p: p.stem)
def test_oracle_reproduces_reference(fixture):
    fx = torch.load(fixture, weights_only=False)
    torch.set_num_threads(8)
    ni, no = PREFIX.get(fx["problem"].split("/")[1], (len(fx["inputs"]), len(fx["outputs"])))
    inputs = make_inputs(fx["inputs"][:ni])
    outs = ORACLES[fx["problem"]](*inputs)
    outs = outs if isinstance(outs, (tuple, list)) else (outs,)
    assert len(outs) == no
    for i, (o, ref) in enumerate(zip(outs, fx["outputs"][:no])):
        assert list(o.shape) == ref["shape"], f"output {i} shape"
        assert str(o.dtype).split(".")[-1] == ref["dtype"], f"output {i} dtype"
        assert _sha(o) == ref["sha256"], f"output {i} differs from the reference bits"
