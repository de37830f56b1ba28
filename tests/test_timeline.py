"""The timeline measurement tool's record handling, on synthetic CTA records (no GPU),
and that the product library carries no timeline instrumentation."""
import ctypes
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "cuda-kernel_b200"))

from swiglu_b200 import _lib, timeline  # noqa: E402


def _records(launches=8, grid=296, period=22_000, tail_sm=(11, 12), seed=0):
    rng = np.random.default_rng(seed)
    rows, t = [], 1_000_000
    for _ in range(launches):
        for b in range(grid):
            sm = b % 148
            st = t + int(rng.integers(0, 150))
            end = st + 17_000 + (3_000 if sm in tail_sm else int(rng.integers(0, 500)))
            meta = b | (grid << 16) | (sm << 32) | (288 << 48)
            rows.append([st, st + 2_400, end - 300, end, st + 13_000, 0, 0, meta])
        t += period
    return np.array(rows, dtype=np.int64)


def test_launches_split_by_grid_and_steady_period():
    rec = _records()
    text, out = timeline.summarise("synthetic", rec, by_time=False)
    assert "8 launches" in text
    assert abs(out["steady"]["period_us"] - 22.0) < 0.2
    assert out["steady"]["tail_us"] > 2.0          # the two slow SMs end 3 us after the rest
    slow = {sm for sm, _ in out["sm"]["slowest"][-2:]}
    assert slow == {11, 12}


def test_work_stealing_records_split_by_start_pauses():
    rec = _records(launches=6)
    keep = np.ones(len(rec), bool)
    keep[::7] = False                               # cancelled CTAs leave no record
    text, out = timeline.summarise("stealing", rec[keep], by_time=True)
    assert "6 launches" in text
    assert "sm" not in out


def test_product_library_has_no_timeline_hooks():
    if not _lib.LIB_PATH.exists():
        import pytest
        pytest.skip("library not built")
    L = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in ("swb_timeline_reset", "swb_timeline_read", "swb_timeline_capacity"):
        assert not hasattr(L, name), name
