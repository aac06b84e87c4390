"""Tracer, routing statistics, expert placement and memory census (CPU)."""
import json
import time

import torch

from arcagi2_flashnext_dots3_b200.utils.observe import RouteStats, Tracer, memory_census, place_experts


def test_tracer_cpu(tmp_path):
    t = Tracer()
    for _ in range(3):
        with t.region("a", device="cpu"):
            time.sleep(0.002)
    s = t.summary()
    assert s["a"]["count"] == 3 and s["a"]["total_ms"] >= 6
    t.chrome(str(tmp_path / "t.json"))
    assert len(json.load(open(tmp_path / "t.json"))["traceEvents"]) == 3


def test_route_stats_and_placement():
    rs = RouteStats(2, 8, "cpu")
    rs.add(0, torch.tensor([[0, 1], [0, 2]]))
    rs.end_step()
    rs.add(0, torch.tensor([[0, 0]]))
    rs.end_step()
    assert rs.counts[0, 0] == 4 and rs.load()[0, 0] == 2
    load = torch.tensor([10.0, 1, 1, 1, 9, 1, 1, 8])
    owner = place_experts(load, 2)
    per = [sum(float(load[e]) for e in range(8) if owner[e] == r) for r in range(2)]
    assert sorted(owner.count(r) for r in range(2)) == [4, 4] and max(per) <= 19  # optimum with 4 per rank


def test_memory_census():
    w = {"a": torch.zeros(10), "b": {"c": torch.zeros(5, dtype=torch.int64)}}
    c = memory_census(w)
    assert c["weights"] == {"a": 40, "b": 40}
