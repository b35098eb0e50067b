"""CPU tests of the host-side schedule logic exported by libwx (PAB refresh /
plan, sigma schedule, sparse policy, row->modRow map) against the golden
fixtures restated from the reference."""
import json
import math
from pathlib import Path

import numpy as np

from wuxianhuabu_b200 import h3

GOLD = Path(__file__).resolve().parent / "golden"


def test_pab_refresh_matches_golden():
    g = json.load(open(GOLD / "pab_schedule.json"))
    for c in g["refresh"]:
        got = [h3.attn_broadcast_refresh(i, c["steps"], c["k"]) for i in range(c["steps"])]
        assert got == c["refresh"], c


def test_pab_plan_matches_golden():
    g = json.load(open(GOLD / "pab_schedule.json"))
    for p in g["plans"]:
        s = h3.sigma_schedule(p["steps"], p["shift"])
        assert np.allclose(s, p["sigmas"], rtol=0, atol=1e-15)
        assert h3.attn_broadcast_plan(s, p["k"], p["max_stale"]) == p["plan"]


def test_pab_reference_comment_examples():
    # PAB:68-69: 6 steps, k=2 -> refresh {0,1,3,5}, reuse {2,4}
    assert [h3.attn_broadcast_refresh(i, 6, 2) for i in range(6)] == [True, True, False, True, False, True]
    # PAB:106-110: shift 12, maxStale 0.04 -> N=6: 1 reuse, N=12: 4, N=30: 10
    for n, want in ((6, 1), (12, 4), (30, 10)):
        plan = h3.attn_broadcast_plan(h3.sigma_schedule(n, 12.0), 2, h3.attn_broadcast_default_max_stale())
        assert plan.count(False) == want
    # the benchmark window: 4 steps -> reuse {2} needs maxStale >= 0.05
    s4 = h3.sigma_schedule(4, 12.0)
    assert h3.attn_broadcast_plan(s4, 2, 0.06) == [True, True, False, True]
    assert h3.attn_broadcast_plan(s4, 2, 0.04) == [True, True, True, True]


def test_must_refresh():
    g = json.load(open(GOLD / "pab_schedule.json"))
    for d in g["must_refresh"]:
        cached = math.inf if d["cached"] == "inf" else d["cached"]
        assert h3.attn_broadcast_must_refresh(cached, d["sigma"], d["max_stale"]) == d["out"]


def test_sparse_mode_for_layer_mix():
    g = json.load(open(GOLD / "pab_schedule.json"))["dense_layers_mix"]
    for n, dense in g.items():
        n = int(n)
        got = [l for l in range(n) if h3.sparse_mode_for_layer(l, n, h3.SparsePolicy.MIX) == 0]
        assert got == dense
        assert all(h3.sparse_mode_for_layer(l, n, h3.SparsePolicy.OFF) == 0 for l in range(n))
        assert h3.sparse_mode_for_layer(3, n, h3.SparsePolicy.MIX) == 2
        assert h3.sparse_mode_for_layer(4, n, h3.SparsePolicy.MIX) == 1


def test_build_row_mod_map_fixture():
    g = json.load(open(GOLD / "modrun.json"))
    runs = [h3.ModRun(s, e, r) for s, e, r in g["runs"]]
    assert h3.H3FusedKernels.build_row_mod_map(g["count"], runs).tolist() == g["map"]
    # clamping of runs that overhang the sequence (fused:242-249)
    m = h3.H3FusedKernels.build_row_mod_map(4, [h3.ModRun(2, 10, 7)])
    assert m.tolist() == [0, 0, 7, 7]
