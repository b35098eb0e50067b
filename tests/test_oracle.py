"""CPU tests of the oracle: its pins against the reference's own fixtures and
known answers, and its internal consistency (quantize/dequantize, routing,
SOL semantics vs dense attention at the self-test geometries)."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, f32

GOLD = Path(__file__).resolve().parent / "golden"


def test_bf16_round_trip_and_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, 1e-40, 0.0], dtype=np.float32)
    b = O.f32_to_bf16(x)
    # 1 + 2^-8 is a tie between 1 and 1+2^-7 -> even (1.0); 1+3*2^-8 -> 1+2^-6
    assert O.bf16_to_f32(b)[0] == 1.0 and O.bf16_to_f32(b)[1] == 1.0
    assert O.bf16_to_f32(b)[2] == np.float32(1.015625)
    assert O.bf16_to_f32(b)[3] == -2.5


def test_rng_is_counter_based():
    a = O.normal_f32((1000,), seed=7, stream=3)
    b = O.normal_f32((2000,), seed=7, stream=3)
    assert np.array_equal(a, b[:1000])
    c = O.normal_f32((1000,), seed=7, stream=4)
    assert not np.array_equal(a, c)
    assert abs(b.mean()) < 0.1 and abs(b.std() - 1) < 0.1


def test_dequant_pinned_to_reference_4bit_unpacker():
    """The only unpacker in the reference (H3Common.swift:379-401, 4-bit) pins the
    word layout and the fp32 q*scale+bias -> bf16 rule; the oracle's general
    unpacker must reproduce it bit for bit."""
    d = np.load(GOLD / "dequant4.npz")
    got = O.dequantize(d["words"], d["scales"], d["biases"], int(d["in_dim"]), bits=int(d["bits"]),
                       group=int(d["group"]))
    assert np.array_equal(got, d["expect"])


@pytest.mark.parametrize("bits", [4, 6, 8])
def test_quantize_dequantize_error_bound(bits):
    w = O.normal_f32((64, 256), seed=1, stream=bits, std=0.02)
    wq, sc, bi = O.quantize(w, bits=bits)
    dq = f32(O.dequantize(wq, sc, bi, 256, bits=bits))
    s = f32(sc).repeat(64, axis=1)
    # error within half a quantization step plus bf16 rounding of the result
    err = np.abs(dq - w)
    assert (err <= 0.5 * s + np.abs(w) * 2 ** -7 + 2 * np.abs(s) * 2 ** -7 + 1e-6).all()


def test_six_bit_stream_layout_16_values_per_3_words():
    # one row with q = 0..63 placed in order: word stream must be the LE bit stream
    k = 64
    q = np.arange(k, dtype=np.uint64)
    bits = np.zeros(k * 6, dtype=np.uint8)
    for i in range(k):
        for b in range(6):
            bits[i * 6 + b] = (q[i] >> b) & 1
    words = np.zeros(k * 6 // 32, dtype=np.uint32)
    for j in range(len(words)):
        words[j] = sum(int(bits[j * 32 + b]) << b for b in range(32))
    sc = O.f32_to_bf16(np.ones((1, 1), np.float32))
    bi = O.f32_to_bf16(np.zeros((1, 1), np.float32))
    dq = f32(O.dequantize(words.reshape(1, -1), sc, bi, k, bits=6))
    assert np.array_equal(dq.ravel(), np.arange(k, dtype=np.float32))


def test_qlinear_matches_float64_reference():
    x = O.normal_bf16((17, 128), 3, 1)
    w = O.normal_f32((96, 128), 3, 2, std=0.02)
    wq, sc, bi = O.quantize(w)
    bias = O.normal_bf16((96,), 3, 3, std=0.1)
    y = O.qlinear(x, wq, sc, bi, bias=bias)
    wd = f32(O.dequantize(wq, sc, bi, 128)).astype(np.float64)
    ref = f32(x).astype(np.float64) @ wd.T
    ref = f32(O.f32_to_bf16(f32(O.f32_to_bf16(ref.astype(np.float32))) + f32(bias)))
    assert np.array_equal(y, O.f32_to_bf16(ref))


def _unfused_norm_rope(x, w, cos, sin, rot, eps):
    # rmsNormLast (H3Common.swift:502-508) then applyRopePub (:555-569), MLX rounding per op in bf16
    xf = f32(x).astype(np.float32)
    var = (xf * xf).mean(-1, keepdims=True)
    nv = f32(O.f32_to_bf16(xf / np.sqrt(var + eps) * f32(w)))
    rh = rot // 2
    c = f32(cos)[:, None, :]
    s = f32(sin)[:, None, :]
    r = lambda a: f32(O.f32_to_bf16(a))
    x1, x2 = nv[..., :rh], nv[..., rh:rot]
    o1 = r(r(x1 * c) - r(x2 * s))
    o2 = r(r(x2 * c) + r(x1 * s))
    return np.concatenate([o1, o2, nv[..., rot:]], -1)


def test_qk_norm_rope_vs_unfused_reference_semantics():
    g = json.load(open(GOLD / "sol_selftest.json"))["fused"]
    S, H, hd, rot, eps = g["S"], g["H"], g["hd"], g["rot"], g["eps"]
    x = O.normal_bf16((S, H, hd), 5, 1)
    w = O.normal_bf16((hd,), 5, 2)
    cos = O.normal_bf16((S, rot // 2), 5, 3)
    sin = O.normal_bf16((S, rot // 2), 5, 4)
    got = f32(O.qk_norm_rope(x, w, cos, sin, rot, eps))
    ref = _unfused_norm_rope(x, w, cos, sin, rot, eps)
    assert np.abs(got - ref).max() < g["tol"]


def test_norm_modscale_and_mod_gate_modrun_fixture():
    g = json.load(open(GOLD / "modrun.json"))
    S, hidden, R = g["count"], g["hidden"], g["num_mod_rows"]
    rowmap = np.array(g["map"], dtype=np.uint32)
    x = O.normal_bf16((S, hidden), 6, 1)
    w = O.normal_bf16((hidden,), 6, 2)
    sh = O.normal_bf16((R, hidden), 6, 3)
    sc = O.normal_bf16((R, hidden), 6, 4)
    got = f32(O.norm_modscale(x, w, sh, sc, rowmap, 1e-5))
    xf = f32(x)
    nv = f32(O.f32_to_bf16(xf / np.sqrt((xf * xf).mean(-1, keepdims=True) + 1e-5) * f32(w)))
    ref = nv * (f32(sc)[rowmap] + 1) + f32(sh)[rowmap]
    assert np.abs(got - ref).max() < 0.25
    other = O.normal_bf16((S, hidden), 6, 5)
    gate = O.normal_bf16((R, hidden), 6, 6)
    got2 = f32(O.mod_gate(x, other, gate, rowmap))
    ref2 = xf + f32(other) * f32(gate)[rowmap]
    assert np.abs(got2 - ref2).max() < 0.25


def _qkv(S, H, hd, seed):
    return (O.normal_bf16((S, H, hd), seed, 1), O.normal_bf16((S, H, hd), seed, 2),
            O.normal_bf16((S, H, hd), seed, 3))


@pytest.mark.parametrize("case", ["case1", "case3"])
def test_sol_all_exact_equals_dense(case):
    g = json.load(open(GOLD / "sol_selftest.json"))[case]
    h, gg, L, hd = g["h"], g["g"], g["L"], g["hd"]
    S = gg + L
    q, k, v = _qkv(S, h, hd, 11)
    scale = 1.0 / np.sqrt(hd)
    route = O.sol_route(q, k, v, gg, scale, g["tau"])
    assert route["sel"].all()
    route.update(g=gg, block=64, tail=True)
    sol = f32(O.sparse_attention(q, k, v, gg, scale, route=route))
    dense = f32(O.sparse_attention(q, k, v, 0, scale))
    tol = g.get("tol_video", g.get("tol"))
    assert np.abs(sol[gg:] - dense[gg:]).max() < tol
    assert np.abs(sol[:gg] - dense[:gg]).max() < g.get("tol_strip", tol)


def test_sol_tail_reduces_error_vs_dropping():
    g = json.load(open(GOLD / "sol_selftest.json"))["case2"]
    h, gg, L, hd = g["h"], g["g"], g["L"], g["hd"]
    S = gg + L
    q, k, v = _qkv(S, h, hd, 12)
    scale = 1.0 / np.sqrt(hd)
    route = O.sol_route(q, k, v, gg, scale, g["tau"])
    route.update(g=gg, block=64)
    dense = f32(O.sparse_attention(q, k, v, 0, scale))
    on = f32(O.sparse_attention(q, k, v, gg, scale, route=route, tail=True))
    off = f32(O.sparse_attention(q, k, v, gg, scale, route=route, tail=False))
    # the pooled tail keeps the softmax denominator close to the full sequence
    assert np.abs(on[gg:] - dense[gg:]).mean() <= np.abs(off[gg:] - dense[gg:]).mean() * 1.05


def test_sol_route_forces_diagonal_and_sink():
    S, H, hd, g = 17 + 400, 2, 128, 17
    q, k, v = _qkv(S, H, hd, 13)
    r = O.sol_route(q, k, v, g, 1 / np.sqrt(hd), 100.0, sink=(2, 4))
    nb = r["sel"].shape[1]
    for i in range(nb):
        for j in range(nb):
            forced = abs(i - j) <= 1 or 2 <= j < 4
            assert r["sel"][:, i, j].all() if forced else not r["sel"][:, i, j].any()
    assert r["lens"][-1] == (S - g) - 64 * (nb - 1)


def test_topk_route_counts_and_ties():
    S, H, hd = 128 * 9 + 40, 2, 128
    q, k, v = _qkv(S, H, hd, 14)
    r = O.topk_route(q, k, v, 0, 1 / np.sqrt(hd), 0.25)
    nb = r["sel"].shape[1]
    keep = int(np.ceil(0.25 * nb))
    assert (r["sel"].sum(-1) == keep + 1).all()
    for h in range(H):
        for i in range(nb):
            assert r["sel"][h, i, i] == 1
            sc = r["scores"][h, i].copy()
            sc[i] = -np.inf
            order = sorted(range(nb), key=lambda j: (-sc[j], j))[:keep]
            assert set(np.nonzero(r["sel"][h, i])[0]) == set(order) | {i}
