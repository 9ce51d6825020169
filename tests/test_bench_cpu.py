"""bench.py's measurement bookkeeping on the CPU: the cache positions its timed steps sample, the algorithmic bytes
per step that the roofline divides by, and the parsing of the clock record whose throttle reasons reject a run."""

from __future__ import annotations

import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import bench  # noqa: E402
from owsm_trt_b200.synthetic import MEDIUM_1B  # noqa: E402


def test_timed_positions_cover_the_decode_positions():
    # whole passes over the 200 decode positions 4 .. 203 when there are enough steps, else an even sample
    assert bench.positions(200) == list(range(4, 204))
    assert bench.positions(400) == list(range(4, 204)) * 2
    p = bench.positions(20)
    assert len(p) == 20 and len(set(p)) == 20 and p == sorted(p)
    assert p[0] == 4 and p[-1] >= 190


def test_step_bytes_counts_each_term_once():
    d = MEDIUM_1B
    L, D = d.L, d.D
    # fp16 weights once per call: the 631 MB the step streams
    weights = 2 * (L * (6 * D * D + 2 * D * d.F) + d.V * D)
    assert 630e6 < weights < 632e6
    assert bench.step_bytes(d, 1, 0, []) > weights
    # one more cached position: every row's keys and values of it in every layer (fp16)
    assert bench.step_bytes(d, 16, 101, []) - bench.step_bytes(d, 16, 100, []) == 16 * 2 * L * 2 * D
    # an utterance's cross K/V frames once, however many rows read them (the beam hypotheses share them)
    assert bench.step_bytes(d, 15, 100, [750] * 3) - bench.step_bytes(d, 15, 100, []) == 3 * 2 * L * 2 * 750 * D
    # per-row terms (cache, new K/V, logits, embedding and positional rows) grow with the rows
    assert bench.step_bytes(d, 16, 100, []) - bench.step_bytes(d, 15, 100, []) == (
        2 * L * 2 * D * 100 + 2 * L * 2 * D + 4 * d.V + 2 * D + 4 * D
    )


def _clocks(out: str, bus: int | None):
    c = bench.Clocks.__new__(bench.Clocks)  # (no GPU here: the record is given)
    c.bus, c.out = bus, out
    return c


ROWS = [
    "1965, 1965, 700.5, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active, 00000000:1B:00.0",
    "1965, 1965, 710.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active, 00000000:1B:00.0",
    "1950, 1965, 705.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active, 00000000:1B:00.0",
    "1200, 1965, 90.0, 0x0000000000000040, Not Active, Active, Not Active, Not Active, 00000000:2C:00.0",
]


def test_clock_record_of_this_gpu():
    s = _clocks("\n".join(ROWS), 0x1B).summary()
    assert s == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    # the other GPU's thermal slowdown is not this run's
    s = _clocks("\n".join(ROWS), 0x2C).summary()
    assert s["reasons"] == ["hw_thermal_slowdown"] and s["sm_mhz"] == 1200.0


def test_clock_record_without_a_bus_takes_the_busiest_gpu():
    assert _clocks("\n".join(ROWS), None).summary()["samples"] == 3
    assert _clocks("", 0x1B).summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
