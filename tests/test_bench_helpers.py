"""Host-side pieces of bench.py that decide its workloads (no GPU).

* the prescribed exit-depth mix of the CDB workload (15/25/30/30% at loop steps 1-4);
* the CDB capacity rule: the outputs a request finishes within the run, counted from its
  prescribed exit depths, against a step-by-step simulation of the device routing
  (a row exits when its depth reaches the prescribed one, cdb_scheduler.py:207-213);
* the radix workload's page tables, built through the native radix prefix cache: rows of
  a group share one copy of the prefix pages, every other page belongs to one row, and the
  cache reports the shared prefix tokens it served;
* the clock-sample summary (median SM clock, throttle reasons) and request admission.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


B = _bench()


def test_cdb_exit_mix_is_prescribed() -> None:
    d = B.cdb_depths(200_000, 7)
    assert d.min() == 1 and d.max() == 4
    frac = np.bincount(d, minlength=5)[1:] / d.size
    assert np.allclose(frac, B.CDB_EXIT_P, atol=0.005), frac
    assert np.array_equal(B.cdb_depths(1000, 7), B.cdb_depths(1000, 7))


def test_cdb_capacity_counts_the_outputs_the_run_finishes() -> None:
    steps = 45
    future = B.cdb_depths(64 * (steps + 8), 3).reshape(64, steps + 8)
    exits = (np.cumsum(future, axis=1) <= steps).sum(1)
    for r in range(64):  # the device routing, step by step
        depth, k, done = 0, 0, 0
        for _ in range(steps):
            depth += 1
            if depth >= future[r, k]:
                done, k, depth = done + 1, k + 1, 0
        assert done == exits[r], r


class _Engine:
    def __init__(self) -> None:
        self.rows: dict[int, np.ndarray] = {}

    def assign_pages(self, row: int, pages: torch.Tensor) -> None:
        self.rows[row] = pages.numpy().copy()


def test_radix_page_tables_share_each_groups_prefix() -> None:
    from __graft_entry__ import load_package

    load_package()  # the page tables come from the package's native radix cache
    bs = 11
    prefix_pages = B.RADIX_PREFIX // B.PAGE
    own = (B.RADIX_SUFFIX + B.RADIX_OUT) // B.PAGE
    need = B.RADIX_GROUPS * prefix_pages + bs * own
    free = np.random.default_rng(1).permutation(need) + 1
    eng = _Engine()
    hits = B.radix_page_tables(eng, free, bs, 49152, "cpu")
    groups = min(bs, B.RADIX_GROUPS)
    assert hits == (bs - groups) * B.RADIX_PREFIX
    for r in range(1, bs + 1):
        pages = eng.rows[r]
        assert pages.size == prefix_pages + own
        first = eng.rows[(r - 1) % B.RADIX_GROUPS + 1]
        assert np.array_equal(pages[:prefix_pages], first[:prefix_pages])
    used = np.concatenate([eng.rows[g + 1][:prefix_pages] for g in range(groups)]
                          + [eng.rows[r][prefix_pages:] for r in eng.rows])
    assert np.unique(used).size == used.size == need  # no page owned twice, none unused
    prefixes = [set(eng.rows[g + 1][:prefix_pages]) for g in range(groups)]
    assert all(not (a & b) for i, a in enumerate(prefixes) for b in prefixes[i + 1:])


def test_clock_summary_reads_samples() -> None:
    got = B.ClockSampler.parse(
        "1965, 1965, 700.1, Not Active, Not Active, Not Active, Not Active\n"
        "1900, 1965, 990.0, Not Active, Not Active, Not Active, Active\n"
        "1965, 1965, 800.0, Not Active, Not Active, Not Active, Not Active\n")
    assert got == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                   "samples": 3}
    assert B.ClockSampler.parse("")["reasons"] == ["unsampled"]


def test_admission_counts_whole_pages() -> None:
    prompts = np.array([16, 17, 100])
    per = (prompts + B.OUT_TOKENS + B.PAGE - 1) // B.PAGE
    assert B.admit(prompts, int(per[:2].sum())) == 2
    assert B.admit(prompts, int(per.sum())) == 3
    assert B.admit(prompts, int(per[0]) - 1) == 0
