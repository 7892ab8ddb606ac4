"""bench.py's byte models and workload settings (no GPU): the per-agent byte
model of a whole tick (CARLB-v1), the per-stage algorithmic bytes used by the
roofline line, and the sizes each named workload runs at."""

from __future__ import annotations

import sys

import pytest

import bench


def test_whole_tick_byte_model():
    # 620 B per car-tick and 504 B per sim-tick: 3v3 704 B, 1v1 872 B, 2v2 746 B per agent-tick.
    assert bench.bytes_per_agent_tick(6) == pytest.approx(704.0)
    assert bench.bytes_per_agent_tick(2) == pytest.approx(872.0)
    assert bench.bytes_per_agent_tick(4) == pytest.approx(746.0)


def test_stage_bytes_cover_every_stage_kernel():
    from carl_b200 import capi

    assert set(bench.STAGE_BYTES) == set(capi.Env.STAGES)
    cars, sims = 98304.0, 16384.0
    work = {"plane_cars": 4600.0, "sat_cars": 1000.0, "moving_balls": 600.0, "car_car_sims": 200.0}
    assert bench.stage_bytes("flat", cars, sims, work) == 140 * cars + 8 * sims
    assert bench.stage_bytes("contact", cars, sims, work) == 232 * (4600 + 1000)
    # car-car: the gates of every car, plus every car of each sim with a pair in reach.
    assert bench.stage_bytes("carCar", cars, sims, work) == pytest.approx(16 * cars + 192 * 200 * 6)
    assert bench.stage_bytes("ball", cars, sims, work) == 144 * 600


@pytest.mark.parametrize("argv, blue, orange, n_sim, workload", [
    ([], 3, 3, 32768, "c3"),
    (["--workload", "c1"], 1, 1, 1024, "c1"),
    (["--workload", "c4"], 2, 2, 32768, "c4"),
    (["--workload", "reset"], 3, 3, 32768, "c5"),
])
def test_workload_sizes(monkeypatch, argv, blue, orange, n_sim, workload):
    monkeypatch.setattr(sys, "argv", ["bench.py", *argv])
    args = bench.parse_args()
    assert (args.blue, args.orange, args.n_sim, args.workload) == (blue, orange, n_sim, workload)
    assert args.reset_n_sim == 131072  # C5: 1,048,576 sims over 8 GPUs


def test_profiles_give_traffic_and_flops_for_every_stage():
    """The roofline's per-launch DRAM traffic and FP32 work come from the committed
    ncu summaries: every stage kernel has both, and traffic scales with the sims."""
    import re

    text = "\n".join(p.read_text() for p in sorted(bench.ROOT.joinpath("profiles").glob("*.md")))
    for stage in bench.STAGE_BYTES:
        t = bench.traffic_per_launch(stage, 32768)
        assert t is not None and t > 0, stage
        assert bench.traffic_per_launch(stage, 16384) == pytest.approx(t / 2), stage
        assert re.search(rf"fp32_flops_per_car_tick\[{stage}\]: \d", text), stage
    total = bench.fp32_flops_per_car_tick()
    assert total is not None and 3000 < total < 5000
