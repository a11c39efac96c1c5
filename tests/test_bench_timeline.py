"""bench.py --timeline: the per-round arithmetic over a kernel list, on the CPU.

Kernels launched with programmatic dependent launch start while their
predecessor still runs, so raw durations overlap; a kernel's live time counts
from the later of its own start and the end of every kernel before it, and the
live times of a round plus its idle gaps make up the round's span.
"""

from __future__ import annotations

import pytest

GEMM = "void ms::(anonymous namespace)::gemm_tc_kernel<256, 1, float>(CUtensorMap_st, int)"
ATTN = "void ms::(anonymous namespace)::attn_tma_kernel<64, 64, 3, 2, 4, 64>(ms::AttnArgs)"
ACC = "void ms::(anonymous namespace)::spec_accept_kernel(ms::AcceptArgs, int)"

# round 0: the attention kernel starts 2 us before the GEMM ends, then 5 us idle
# before the accept kernel; round 1: 1 us idle
EVENTS = [(0.0, 10.0, GEMM), (8.0, 20.0, ATTN), (25.0, 30.0, ACC),
          (30.0, 40.0, GEMM), (41.0, 50.0, ACC)]


def test_live_time_idle_and_span_per_round() -> None:
    import bench

    s = bench.timeline_summary(list(reversed(EVENTS)), 0, 2)
    assert s["rounds"] == 2
    assert s["round_us_each"] == [30.0, 20.0]
    assert s["idle_us_each"] == [5.0, 1.0]
    k = s["kernels"]
    assert set(k) == {"gemm_tc_kernel<256, 1, float>", "attn_tma_kernel<64, 64, 3, 2, 4, 64>",
                      "spec_accept_kernel"}
    assert k["gemm_tc_kernel<256, 1, float>"]["us"] == pytest.approx(10.0)  # (10 + 10) / 2
    assert k["attn_tma_kernel<64, 64, 3, 2, 4, 64>"]["us"] == pytest.approx(5.0)  # (20 - 10) / 2
    assert k["spec_accept_kernel"]["us"] == pytest.approx(7.0)  # (5 + 9) / 2
    assert k["gemm_tc_kernel<256, 1, float>"]["launches"] == pytest.approx(1.0)
    # live time and idle time add up to the span
    live = sum(v["us"] for v in k.values()) * s["rounds"]
    assert live + sum(s["idle_us_each"]) == pytest.approx(sum(s["round_us_each"]))
    assert sum(v["share"] for v in k.values()) == pytest.approx(1.0 - 6.0 / 50.0)


def test_rounds_before_first_are_left_out() -> None:
    import bench

    s = bench.timeline_summary(EVENTS, 1, 5)
    assert s["rounds"] == 1
    assert s["round_us_each"] == [20.0]
    assert s["kernels"]["spec_accept_kernel"]["us"] == pytest.approx(9.0)
