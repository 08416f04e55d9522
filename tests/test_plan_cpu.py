"""The tiled GEMV's planner (qg_gemv_plan_sms, host-side, no device): on a B200's 148 SMs
the rows of every sweep, slice, decode and config-4 shape spread evenly -- the busiest SM
carries at most ~11% more rows than the average (tiles may end inside a shared-memory
stage, so medium matrices are not rounded to whole stages) -- and every plan is a valid
launch (grid no larger than its tiles, at most 544 threads, at least two stages)."""

import math

import pytest

from qgemv_b200 import ops, packs

SMS = 148
SHAPES = [
    # config 2 sweep
    *[(f, r, c) for f in (packs.Q4K_RAW, packs.Q5K, packs.IQ2S, packs.IQ3S)
      for r, c in ((14336, 4096), (128256, 8192))],
    # decode step (70B widths, TP1): Q/K/V fused, Wo, gate/up fused, Wd, vocab head
    (packs.IQ3S, 10240, 8192), (packs.IQ3S, 8192, 8192), (packs.IQ2S, 57344, 8192),
    (packs.Q5K, 8192, 28672), (packs.Q4K_RAW, 128256, 8192),
    # config 4 at batch 1
    (packs.Q4K_RAW, 28672, 8192), (packs.Q4K_RAW, 8192, 28672),
    (packs.IQ2S, 28672, 8192), (packs.IQ2S, 8192, 28672),
]


@pytest.mark.parametrize("fmt,rows,cols", SHAPES)
def test_plan_spreads_rows_over_the_sms(fmt, rows, cols):
    p = ops.gemv_plan(fmt, rows, cols, sms=SMS)
    tiles = math.ceil(rows / p["rows_per_tile"])
    assert 1 <= p["grid"] <= tiles
    assert p["threads"] <= 544 and p["stages"] >= 2
    per_sm = 2 if p["grid"] > SMS else 1          # CTAs that share an SM
    busiest = per_sm * math.ceil(tiles / p["grid"]) * p["rows_per_tile"]
    assert (rows / SMS) / busiest >= 0.9, (p, busiest, rows / SMS)


def test_plan_query_rejects_bad_shapes():
    with pytest.raises(RuntimeError):
        ops.gemv_plan(packs.Q4K_RAW, 16, 300, sms=SMS)
    with pytest.raises(RuntimeError):
        ops.gemv_plan(packs.Q4K_RAW, 0, 4096, sms=SMS)
