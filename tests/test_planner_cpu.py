"""The K2 split planner's cost model (``plan_pages_per_split``) on CPU, with
the occupancies the kernel reports on B200 (148 SMs): it must reproduce the
plans that ran fastest there in the bench's config-1, -2 and -4 runs (10, 14
and 22 pages per item).  A same-box sweep of the whole decode step at config 2
(28 layers): 12 and 13 pages per item 71-73 us per layer, 14: 58.8, 15: 59.9,
16: 60.0, 17-22: 62-63; at config 1, 8: 38.2, 9: 39.6, 10: 34.2, 11: 35.5."""
from __future__ import annotations

from logitfill_b200.packed.attention import plan_pages_per_split

SMS = 148
RESID_PER_PAIR = 4  # 32-row residual chunks of a 128-token page: ceil((128 - 1 + 1) / 32)


def test_config1_three_page_items_per_sm():
    # 16 sequences x 4 KV heads, 64 pages: 256 residual items keep a slot each.
    pairs = 16 * 4
    assert plan_pages_per_split(64, pairs, pairs * RESID_PER_PAIR, SMS, lambda pps: 4) == 10


def test_config2_fills_every_slot_when_the_residual_items_are_few():
    # 8 sequences x 4 KV heads, 256 pages: 128 residual items fit in a quarter wave.
    # 14 pages per item: 576 full items and 16 of the 32 short last items (4
    # pages) fill the 592 slots; the other 16 start in the slots those free.
    pairs = 8 * 4
    assert plan_pages_per_split(256, pairs, pairs * RESID_PER_PAIR, SMS, lambda pps: 4) == 14
    # The same history where only three CTAs fit (31-word rows).
    assert plan_pages_per_split(256, pairs, pairs * RESID_PER_PAIR, SMS, lambda pps: 3) == 19


def test_config4_many_pairs():
    pairs = 64 * 8
    assert plan_pages_per_split(128, pairs, pairs * RESID_PER_PAIR, SMS, lambda pps: 4) == 22


def test_edge_cases():
    assert plan_pages_per_split(0, 4, 16, SMS, lambda pps: 4) == 1
    assert plan_pages_per_split(1, 4, 16, SMS, lambda pps: 4) == 1
    # No launchable pps above 8: the plan stays within what fits.
    assert plan_pages_per_split(100, 4, 16, SMS, lambda pps: 4 if pps <= 8 else 0) <= 8
    # A single pair: the largest item that keeps one wave.
    assert plan_pages_per_split(64, 1, 4, SMS, lambda pps: 4) == 1
