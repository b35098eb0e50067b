"""Generate the committed golden fixtures under tests/golden/.

The reference (Swift + MLX + Metal) cannot run here, so the fixtures are
known answers taken from the reference's own source, restated in numpy:

* pab_schedule.json — attnBroadcastRefresh / attnBroadcastPlan / sigmaSchedule
  (网络算子-注意力跨步缓存-通用.swift:57-112, model/minimax h3/H3Layout.swift:156-182)
  restated in plain Python, cross-checked against the examples the reference
  writes in its comments (PAB:68-69 "6 步 + k=2 → refresh {0,1,3,5}"; PAB:106-110
  "N=6 只剩 1 个复用步（跨度 0.024）, N=12 剩 4 个, N=30 剩 10 个").
* dequant4.npz — MfLinear.dequantizedWeight (H3Common.swift:379-401), the
  reference's only in-tree unpacker (4-bit words), restated in numpy on seeded
  packed words: pins the packed bit layout and the fp32 q*scale+bias -> bf16 rule.
* modrun.json — the 3-run ModRun fixture of the fused self-test
  (网络算子-融合-RMSNormRoPE-通用.swift:417-421) and buildRowModMap's (:238-250) map.
* sol_selftest.json — geometries and tolerances of the SOL self-test
  (网络算子-稀疏注意力-SOL通用.swift:686-761, 888-915) and the fused self-test (fused:404-407).

Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


# ---------------------------------------------------------------- PAB restatement
def scaled_gate(steps: int, at30: int) -> int:
    return max(1, min(at30, steps * at30 // 30))


def pab_refresh(i: int, steps: int, k: int) -> bool:
    if k <= 1:
        return True
    warm = scaled_gate(steps, 4)
    if i < warm:
        return True
    if i + scaled_gate(steps, 2) >= steps:
        return True
    return (i - warm) % k == 0


def must_refresh(cached: float, sigma: float, max_stale: float) -> bool:
    return not (abs(sigma - cached) <= max_stale)


def pab_plan(sigmas, k, max_stale):
    nfe = max(0, len(sigmas) - 1)
    cached = math.inf
    out = []
    for i in range(nfe):
        r = pab_refresh(i, nfe, k) or must_refresh(cached, sigmas[i], max_stale)
        if r:
            cached = sigmas[i]
        out.append(r)
    return out


def time_shift_sigma(sigma, from_shift, to_shift):
    base = sigma / (from_shift + sigma * (1.0 - from_shift))
    return to_shift * base / (1.0 + (to_shift - 1.0) * base)


def sigma_schedule(steps, shift):
    return [time_shift_sigma(1.0 - i / steps, 1.0, shift) for i in range(steps + 1)]


def make_pab():
    cases = []
    for steps in (1, 2, 4, 6, 12, 30):
        for k in (0, 1, 2, 3):
            cases.append(dict(i_range=steps, steps=steps, k=k,
                              refresh=[pab_refresh(i, steps, k) for i in range(steps)]))
    plans = []
    for steps in (4, 6, 12, 30):
        s = sigma_schedule(steps, 12.0)
        for ms in (0.04, 0.06, 1e9):
            plans.append(dict(steps=steps, shift=12.0, k=2, max_stale=ms, sigmas=s, plan=pab_plan(s, 2, ms)))
    # cross-checks against the reference's own comments
    assert [pab_refresh(i, 6, 2) for i in range(6)] == [True, True, False, True, False, True]
    reuse = {n: sum(1 for r in pab_plan(sigma_schedule(n, 12.0), 2, 0.04) if not r) for n in (6, 12, 30)}
    assert reuse == {6: 1, 12: 4, 30: 10}, reuse
    s6 = sigma_schedule(6, 12.0)
    assert abs(abs(s6[2] - s6[1]) - 0.024) < 0.001
    assert [round(x, 5) for x in sigma_schedule(4, 12.0)] == [1.0, 0.97297, 0.92308, 0.8, 0.0]
    must = [dict(cached=c, sigma=s, max_stale=m, out=must_refresh(c, s, m))
            for c, s, m in [(math.inf, 1.0, 0.04), (1.0, 0.97, 0.04), (1.0, 0.95, 0.04), (0.5, 0.46, 0.04)]]
    for d in must:
        if d["cached"] == math.inf:
            d["cached"] = "inf"
    sparse = {str(n): [lay for lay in range(n) if _sparse_mode(lay, n, 1) == 0] for n in (48, 50)}
    json.dump(dict(refresh=cases, plans=plans, must_refresh=must, dense_layers_mix=sparse,
                   source="restated from 网络算子-注意力跨步缓存-通用.swift:57-112 and H3Layout.swift:156-182,896-906"),
              open(HERE / "pab_schedule.json", "w"), indent=1)


def _sparse_mode(layer, n, policy):
    if policy == 0:
        return 0
    mid = n // 2
    if layer < 2 or layer + 2 >= n or layer == mid or layer == mid + 1:
        return 0
    return 1 if layer % 2 == 0 else 2


# ------------------------------------------------------------ 4-bit dequant pin
def bf16_round_bits(x: np.ndarray) -> np.ndarray:
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = u + 0x7FFF + ((u >> 16) & 1)
    return (u >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def make_dequant4():
    rng = np.random.default_rng(20261201)
    out_dim, in_dim, group, bits = 8, 128, 64, 4
    words = rng.integers(0, 2**32, size=(out_dim, in_dim * bits // 32), dtype=np.uint64).astype(np.uint32)
    scales = bf16_round_bits(rng.normal(0, 0.01, size=(out_dim, in_dim // group)).astype(np.float32))
    biases = bf16_round_bits(rng.normal(0, 0.1, size=(out_dim, in_dim // group)).astype(np.float32))
    # H3Common.swift:385-398: words [out, groups, gs/npw, 1] >> shifts[npw] & 0xF; q*s + b in fp32; -> bf16
    n_per_word = 32 // bits
    w4 = words.reshape(out_dim, in_dim // group, group // n_per_word, 1)
    shifts = (np.arange(n_per_word, dtype=np.uint32) * bits).reshape(1, 1, 1, n_per_word)
    nib = (w4 >> shifts) & 0xF
    s = bf16_to_f32(scales).reshape(out_dim, in_dim // group, 1, 1)
    b = bf16_to_f32(biases).reshape(out_dim, in_dim // group, 1, 1)
    dq = nib.astype(np.float32) * s + b
    expect = bf16_round_bits(dq.reshape(out_dim, in_dim))
    np.savez(HERE / "dequant4.npz", words=words, scales=scales, biases=biases, expect=expect,
             bits=bits, group=group, in_dim=in_dim)


def make_modrun():
    runs = [(0, 5, 0), (5, 11, 3), (11, 16, 5)]
    m = [0] * 16
    for s, e, r in runs:
        for i in range(s, e):
            m[i] = r
    json.dump(dict(runs=runs, count=16, map=m, hidden=64, num_mod_rows=6,
                   source="网络算子-融合-RMSNormRoPE-通用.swift:408-421 (fixture), :238-250 (map)"),
              open(HERE / "modrun.json", "w"), indent=1)


def make_sol_selftest():
    json.dump(dict(
        case1=dict(h=2, g=17, L=160, hd=128, tau=-100.0, tol_video=0.03, tol_strip=0.005,
                   source="SOL:686-730"),
        case3=dict(h=2, g=128, L=192, hd=128, tau=-100.0, tol=0.03, source="SOL:748-761"),
        case2=dict(h=2, g=17, L=160, hd=128, tau=0.4, source="SOL:732-746 (report only)"),
        case4=dict(h=2, g=17, L=160, hd=128, tau=0.4, sink=[0, 1], source="SOL:763-769 (report only)"),
        caseR=dict(h=56, g=934, L=9324, hd=128, source="SOL:874-886 production geometry"),
        caseS=dict(tol=0.02, source="SOL:888-915 chunked == whole"),
        fused=dict(S=8, H=4, hd=128, rot=96, eps=1e-5, tol=0.25, source="fused:391-407"),
    ), open(HERE / "sol_selftest.json", "w"), indent=1)


if __name__ == "__main__":
    make_pab()
    make_dequant4()
    make_modrun()
    make_sol_selftest()
    print("golden fixtures written to", HERE)
