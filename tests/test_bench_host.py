"""Host-side helpers of bench.py (no GPU): the e2e host-memory guard and the
config record both arms emit."""
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


def test_e2e_fits_when_every_rank_has_room(monkeypatch):
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "8")
    ok, why = bench._host_memory_fits(21_800_000_000, 1, torch.device("cpu"), avail=600 * 10**9)
    assert ok and why == ""


def test_e2e_skips_with_a_reason_when_ranks_would_exhaust_the_host(monkeypatch):
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "8")
    ok, why = bench._host_memory_fits(21_800_000_000, 1, torch.device("cpu"), avail=196 * 10**9)
    assert not ok
    assert "8 ranks" in why and "196 GB" in why


def test_e2e_unknown_memory_is_assumed_to_fit(monkeypatch):
    monkeypatch.delenv("LOCAL_WORLD_SIZE", raising=False)
    ok, _ = bench._host_memory_fits(10**12, 1, torch.device("cpu"), avail=0)
    assert ok


def test_both_arms_report_the_same_config():
    names = bench.SUITE
    a = bench.config_dict("suite", 2, bench.suite_descriptions(names))
    b = bench.config_dict("suite", 2, bench.suite_descriptions(names, {n: "other text" for n in names}))
    assert a == b and set(a["fragments"]) == set(names)
