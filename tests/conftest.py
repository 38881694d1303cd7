"""Shared pytest setup: the `gpu` marker and tolerance helpers.

Tolerances (from the benchmark's parity rules):
  bf16 outputs    |a - b| <= 1e-2 + 1.6e-2 * |b|
  fp32 rstd / dw  |a - b| <= 1e-4 * |b| (+ a small absolute floor for
                  near-zero dweight columns, 1e-4 * rms of the column terms)
  embedding fwd   bit exact
"""
import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

BF16_ATOL = 1e-2
BF16_RTOL = 1.6e-2
F32_RTOL = 1e-4


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libfrag.so")
    config.addinivalue_line("markers", "slow: full-size cases")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def assert_bf16_close(actual: torch.Tensor, expected: torch.Tensor, what: str = "",
                      atol: float = BF16_ATOL, rtol: float = BF16_RTOL):
    a = actual.detach().float().cpu()
    e = expected.detach().float().cpu()
    assert a.shape == e.shape, f"{what}: shape {tuple(a.shape)} != {tuple(e.shape)}"
    err = (a - e).abs()
    bound = atol + rtol * e.abs()
    bad = err > bound
    if bad.any():
        i = int(torch.argmax((err - bound).flatten()))
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {a.numel()} elements out of tolerance; worst at flat "
            f"{i}: got {a.flatten()[i].item()} want {e.flatten()[i].item()}")


# Problems whose graph repeats one op chain over many input groups: the
# oracle is pinned on the first groups (inputs, outputs) -- the same aten ops
# as the rest -- instead of generating every input (v1-v2/d7efc428b2f5: 33
# (q, k) pairs, 5.5 GB of complex64 inputs).
ORACLE_PREFIX = {"d7efc428b2f5": (6, 4)}


def bf16_ulp(t: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 values at |t| (8 significant bits)."""
    a = t.detach().float().abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(a)) - 7)


def assert_bf16_sum_close(actual: torch.Tensor, expected: torch.Tensor, addend: torch.Tensor,
                          what: str = "", max_flips: int = 16):
    """For outputs bf16(addend + bf16(t)): the intermediate bf16(t) may round
    the other way when t lands near a rounding boundary (its fp32 value comes
    from a differently ordered row reduction), which moves the output by one
    bf16 ulp of |t| -- far above the plain bf16 tolerance when addend and t
    cancel.  Every element must be within the plain tolerance plus one ulp of
    |t| = |expected - addend|, and at most `max_flips` may need the ulp."""
    a = actual.detach().float().cpu()
    e = expected.detach().float().cpu()
    t = e - addend.detach().float().cpu().reshape(e.shape)
    err = (a - e).abs()
    plain = BF16_ATOL + BF16_RTOL * e.abs()
    bad = err > plain + bf16_ulp(t)
    if bad.any():
        i = int(torch.argmax((err - plain - bf16_ulp(t)).flatten()))
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {a.numel()} elements beyond one ulp of the addend-free "
            f"term; worst at flat {i}: got {a.flatten()[i].item()} want {e.flatten()[i].item()}")
    flips = int((err > plain).sum())
    assert flips <= max_flips, f"{what}: {flips} one-ulp roundings of the intermediate (> {max_flips})"


def assert_f32_close(actual: torch.Tensor, expected: torch.Tensor, what: str = "",
                     rtol: float = F32_RTOL, atol: float = 0.0):
    a = actual.detach().double().cpu()
    e = expected.detach().double().cpu()
    assert a.shape == e.shape, f"{what}: shape {tuple(a.shape)} != {tuple(e.shape)}"
    err = (a - e).abs()
    bound = atol + rtol * e.abs()
    bad = err > bound
    if bad.any():
        i = int(torch.argmax((err - bound).flatten()))
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {a.numel()} out of rtol {rtol}; worst at flat {i}: "
            f"got {a.flatten()[i].item()} want {e.flatten()[i].item()}")
