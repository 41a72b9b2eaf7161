"""The benchmark's workload definitions: interval
generation keeps the reference's interval rules and the exact row budgets."""

import argparse
import math

import pytest

import bench
from budgeted_kv_cache_repair_b200.validate import validate_intervals


def _check(intervals, length, rows, suffix_start):
    assert sum(b - a for a, b in intervals) == rows
    assert all(suffix_start <= a < b <= length for a, b in intervals)
    # sorted, disjoint and non-adjacent (kernels/executor.py:66-67)
    assert all(intervals[i][1] < intervals[i + 1][0] for i in range(len(intervals) - 1))
    assert list(validate_intervals(intervals, length)) == [tuple(i) for i in intervals]


@pytest.mark.parametrize("name", ["config1", "config2", "config3"])
def test_workload_intervals_hold_the_budget(name):
    cfg = bench.workload_config(argparse.Namespace(workload=name, intervals=None))
    length = cfg["context"] - cfg["delete"]
    intervals = bench.budget_intervals(1, cfg["delete_at"], length, cfg["intervals"], cfg["rows"])
    assert len(intervals) == cfg["intervals"]
    _check(intervals, length, cfg["rows"], cfg["delete_at"])


def test_config3_budget_is_five_percent_of_the_suffix():
    cfg = bench.CONFIG3
    suffix = cfg["context"] - cfg["delete"] - cfg["delete_at"]
    assert cfg["rows"] == math.ceil(0.05 * suffix) == 1383


@pytest.mark.parametrize("count", [1, 4, 16])
def test_config2_interval_sweep(count):
    cfg = bench.workload_config(argparse.Namespace(workload="config2", intervals=count))
    assert cfg["intervals"] == count and f"{count} interval" in cfg["metric"]
    length = cfg["context"] - cfg["delete"]
    _check(bench.budget_intervals(1, cfg["delete_at"], length, count, cfg["rows"]), length, cfg["rows"],
           cfg["delete_at"])


def test_even_split_matches_plain_intervals():
    assert bench.budget_intervals(1, 1024, 7936, 16, 64) == bench.make_intervals(1, 1024, 7936, 16, 4)


@pytest.mark.parametrize("name", ["ref2048", "ref8192"])
@pytest.mark.parametrize("count", [1, 4, 16])
def test_reference_benchmark_geometry(name, count):
    """The reference benchmark's placement (benchmarks/benchmark_refresh.py:35-61):
    8 tokens deleted at L // 8, 64 rows in `count` intervals about the middle,
    every interval after the deletion."""
    cfg = bench.workload_config(argparse.Namespace(workload=name, intervals=count))
    length = cfg["context"] - cfg["delete"]
    assert length in (2048, 8192) and cfg["delete_at"] == length // 8 and cfg["delete"] == 8
    intervals = bench.workload_intervals(cfg, 1, length)
    assert len(intervals) == count
    _check(intervals, length, 64, cfg["delete_at"])
    if count == 1:
        assert intervals == [((length - 64) // 2, (length - 64) // 2 + 64)]
    else:
        width = 64 // count
        assert intervals[0][0] == round(length / 4 - width / 2)
        assert intervals[-1][1] == round(3 * length / 4 - width / 2) + width
