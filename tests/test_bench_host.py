"""CPU tests of bench.py's host-side arithmetic (no GPU): the config-5 geometry and PAB window,
the algorithmic FLOP counts the roofline divides by (GEMM 1.375 PFLOP per refresh step; the
attention of the mix policy), the phase summary of a trace, the memory-bound and peer-store
summaries, and the config-2 point and CTA-shape parsing, so that a refactor cannot break a GPU
run's final JSON line unnoticed."""
import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_config5_geometry_and_window(bench):
    c = bench.geometry("c5")
    assert (c["S"], c["g"], c["video"], c["inner"]) == (126512, 14912, 111600, 3072)
    assert bench.window_plan() == [True, True, False, True]


def test_step_flops_match_the_survey(bench):
    """The survey's 3.93 PFLOP of attention assumes top-k on all 48 layers (strip q-rows 1.11,
    video -> strip keys 0.98, video -> video 25 % 1.84 PF); the mix policy's 6 dense anchor
    layers attend every video key instead, which adds 6 x 111600 x (111600 - 219 x 128) pairs."""
    c = bench.geometry("c5")
    f = bench.step_flops(c, True)
    assert abs(f["gemm"] / 1.375e15 - 1) < 0.01, f
    per_pair = 4 * 128 * 24
    dense_extra = 6 * 111600 * (111600 - 219 * 128) * per_pair
    assert abs(f["attn"] / (3.93e15 + dense_extra) - 1) < 0.01, f
    r = bench.step_flops(c, False)
    assert r["attn"] == 0 and abs(r["gemm"] / 0.92e15 - 1) < 0.02, r


def test_phase_summary(bench):
    rec = lambda layer, mode, ms: dict(layer=layer, mode=mode, total_ms=sum(ms), norm1_ms=ms[0], qkv_ms=ms[1],
                                       rope_ms=ms[2], attn_ms=ms[3], out_ms=ms[4], mlp_ms=ms[5])
    trace = [rec(0, "dense", [1, 2, 0, 10, 1, 6]), rec(1, "sparse", [1, 2, 0, 5, 1, 6]),
             rec(2, "reuse", [0, 0, 0, 0, 1, 6])]
    p = bench.phase_summary(trace, 2)
    assert p["blocks"] == 3
    assert p["ms_per_step"]["attn"] == 7.5 and p["ms_per_step"]["mlp"] == 9.0
    assert p["dense_block_ms"] == dict(mean=20.0, count=1)
    assert p["reuse_block_ms"] == dict(mean=7.0, count=1)


def test_memory_and_peer_summaries(bench):
    c = bench.geometry("c5")
    kinds = ["qgemm", "attention", "routing", "row_kernels", "dequant", "collectives", "qk_norm_rope",
             "norm_modscale", "qkv_to_peers", "peer_wait"]
    prof = {k: dict(ms=0.0, launches=0) for k in kinds}
    prof["norm_modscale"] = dict(ms=2.0, launches=8)
    prof["peer_wait"] = dict(ms=1.0, launches=4)
    peaks = dict(hbm_gbs=6461.5)
    m = bench.memory_bound_kernels(c, prof, 2, peaks, "measured")
    nm = m["row_kernels"]["norm_modscale"]
    rows = c["S"] // 2
    assert nm["bytes_per_launch"] == 2 * rows * c["hidden"] * 2 + rows * 4
    assert abs(nm["gbs"] - nm["bytes_per_launch"] / 0.25e-3 / 1e9) < 1e-6
    assert m["row_kernels"]["qk_norm_rope"] is None and m["exchange"]["qkv_to_peers"] is None
    trace = [dict(mode="dense")] * 2 + [dict(mode="reuse")]
    phases = dict(ms_per_step=dict(qkv=100.0, attn=1000.0))
    ps = bench.peer_store_summary(trace, phases, c, 2, 1, m["exchange"]["attention_out_peer_bytes_per_launch"])
    qkv_b = rows * 3 * c["inner"] * 2 / 2 * 2
    assert ps["peer_bytes_per_step"]["qkv_from_projection_epilogue"] == qkv_b
    assert abs(ps["peer_gbs_lower_bound"]["qkv_phase"] - qkv_b / 0.1 / 1e9) < 1e-6


def test_c2_plan_points_and_cta_shapes(bench):
    plan, rows = bench.c2_plan("", "")
    assert [kn for kn, _ in plan] == [(3072, 3072), (3072, 9216), (3072, 12288), (12288, 3072)]
    assert all(ms == (256, 4096, 28520, 111600) for _, ms in plan) and rows == [None]
    plan, rows = bench.c2_plan("256,3072,3072;512,3072,3072;8,3072,9216;256,3072,3072", "128/2,128/4,256,0")
    assert plan == [((3072, 3072), (256, 512)), ((3072, 9216), (8,)), ((3072, 3072), (256,))]
    assert rows == ["128/2", "128/4", "256", "0"]
    for bad in ("64", "128/3", "128/2/4", "x"):
        with pytest.raises(ValueError):
            bench.c2_plan("", bad)
