"""GPU parity of the SOL / top-k routers (bit-exact decisions and tables) and
of the tcgen05 flash-attention kernel against the CPU oracle, at the
reference self-test geometries and at ragged / aligned / strip-heavy shapes."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
HD = 128


def _qkv(S, H, seed):
    return (O.normal_bf16((S, H, HD), seed, 1), O.normal_bf16((S, H, HD), seed, 2),
            O.normal_bf16((S, H, HD), seed, 3))


def _dev(*arrs):
    return [to_torch_bf16(a) for a in arrs]


def _h3():
    from wuxianhuabu_b200 import h3
    return h3


GEOMS = [(2, 17, 160), (2, 128, 192), (3, 0, 640), (2, 100, 1000), (2, 700, 300), (1, 1, 64)]


@pytest.mark.parametrize("H,g,L", GEOMS)
@pytest.mark.parametrize("tau", [0.4, 1.3, -100.0])
def test_sol_route_bit_exact(H, g, L, tau):
    h3 = _h3()
    S = g + L
    q, k, v = _qkv(S, H, 100 + g + L)
    scale = float(1 / np.sqrt(HD))
    ref = O.sol_route(q, k, v, g, scale, tau, sink=(1, 2))
    cfg = h3.H3SolAttnConfig(tau=tau, sink_blocks=range(1, 2))
    got = h3.H3SolAttn.route(*_dev(q, k, v), g, scale, cfg)
    assert np.array_equal(got["sel"].cpu().numpy(), ref["sel"])
    assert np.array_equal(got["thr"].cpu().numpy().view(np.uint32), ref["thr"].view(np.uint32))
    assert np.array_equal(to_np_bf16(got["cm"]), ref["cm"])
    assert np.array_equal(to_np_bf16(got["vsum"]), ref["vsum"])
    assert np.array_equal(got["lens"].cpu().numpy(), ref["lens"])


@pytest.mark.parametrize("H,g,S", [(2, 0, 128 * 9 + 40), (2, 300, 3000), (3, 0, 128 * 40)])
def test_topk_route_bit_exact(H, g, S):
    h3 = _h3()
    q, k, v = _qkv(S, H, 200 + S)
    scale = float(1 / np.sqrt(HD))
    ref = O.topk_route(q, k, v, g, scale, 0.25)
    cfg = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False)
    got = h3.H3SolAttn.route(*_dev(q, k, v), g, scale, cfg)
    assert np.array_equal(got["scores"].cpu().numpy().view(np.uint32), ref["scores"].view(np.uint32))
    assert np.array_equal(got["sel"].cpu().numpy(), ref["sel"])


@pytest.mark.parametrize("pattern", ["all_equal", "two_levels", "signed_zero"])
def test_topk_route_ties_bit_exact(pattern):
    """Many equal block scores: the selection must break ties by the lower block index."""
    h3 = _h3()
    H, g, S = 2, 0, 128 * 23 + 17
    q, k, v = _qkv(S, H, 900)
    kf = O.bf16_to_f32(k)
    if pattern == "all_equal":
        kf[:] = kf[0:1]
    elif pattern == "two_levels":
        kf[:] = np.where((np.arange(S) // 128 % 3 == 0)[:, None, None], kf[0:1], kf[1:2])
    else:  # zero keys give +0 / -0 scores that must compare equal
        kf[:] = 0.0
    k = O.f32_to_bf16(kf)
    scale = float(1 / np.sqrt(HD))
    ref = O.topk_route(q, k, v, g, scale, 0.25)
    cfg = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False)
    got = h3.H3SolAttn.route(*_dev(q, k, v), g, scale, cfg)
    assert np.array_equal(got["scores"].cpu().numpy().view(np.uint32), ref["scores"].view(np.uint32))
    assert np.array_equal(got["sel"].cpu().numpy(), ref["sel"])


@pytest.mark.parametrize("S,H", [(64, 1), (300, 2), (1000, 3), (129, 2)])
def test_dense_attention(S, H):
    h3 = _h3()
    q, k, v = _qkv(S, H, 300 + S)
    scale = float(1 / np.sqrt(HD))
    ref = f32(O.sparse_attention(q, k, v, 0, scale))
    got = f32(to_np_bf16(h3.H3SolAttn.forward(*_dev(q, k, v), 0, scale, None)))
    assert_close(got, ref, rel=2e-2, cos=0.9995, what=f"dense S={S}")


@pytest.mark.parametrize("case", ["case1", "case3"])
def test_sol_all_exact_matches_dense_reference_tolerances(case):
    """SOL self-test cases 1/3 (SOL:715-761): tau=-100 selects every block, so the
    output equals dense SDPA within 0.03 (video rows) / 0.005 (strip rows)."""
    h3 = _h3()
    gd = json.load(open(GOLD / "sol_selftest.json"))[case]
    H, g, L = gd["h"], gd["g"], gd["L"]
    S = g + L
    q, k, v = _qkv(S, H, 11)
    scale = float(1 / np.sqrt(HD))
    dense = f32(O.sparse_attention(q, k, v, 0, scale))
    got = f32(to_np_bf16(h3.H3SolAttn.forward(*_dev(q, k, v), g, scale, h3.H3SolAttnConfig(tau=gd["tau"]))))
    tol_v = gd.get("tol_video", gd.get("tol"))
    assert np.abs(got[g:] - dense[g:]).max() < tol_v
    assert np.abs(got[:g] - dense[:g]).max() < gd.get("tol_strip", tol_v) + 0.01  # bf16 P on tensor cores


@pytest.mark.parametrize("H,g,L", GEOMS)
@pytest.mark.parametrize("tail", [True, False])
def test_sol_attention_vs_oracle(H, g, L, tail):
    h3 = _h3()
    S = g + L
    q, k, v = _qkv(S, H, 400 + g + L)
    scale = float(1 / np.sqrt(HD))
    route = O.sol_route(q, k, v, g, scale, 0.4)
    route.update(g=g, block=64)
    ref = f32(O.sparse_attention(q, k, v, g, scale, route=route, tail=tail))
    got = f32(to_np_bf16(h3.H3SolAttn.forward(*_dev(q, k, v), g, scale, h3.H3SolAttnConfig(tau=0.4, tail=tail))))
    assert_close(got, ref, rel=2e-2, cos=0.9995, what=f"sol H={H} g={g} L={L} tail={tail}")


@pytest.mark.parametrize("H,g,S", [(2, 0, 128 * 9 + 40), (2, 300, 3000)])
@pytest.mark.parametrize("tail", [False, True])
def test_topk_attention_vs_oracle(H, g, S, tail):
    h3 = _h3()
    q, k, v = _qkv(S, H, 500 + S)
    scale = float(1 / np.sqrt(HD))
    route = O.topk_route(q, k, v, g, scale, 0.25)
    route.update(g=g, block=128)
    ref = f32(O.sparse_attention(q, k, v, g, scale, block=128, route=route, tail=tail))
    cfg = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=tail)
    got = f32(to_np_bf16(h3.H3SolAttn.forward(*_dev(q, k, v), g, scale, cfg)))
    assert_close(got, ref, rel=2e-2, cos=0.9995, what=f"topk S={S} g={g}")


def test_attention_from_given_selection_random_masks():
    """The flash kernel alone on random selections (exercises odd union counts)."""
    h3 = _h3()
    import torch
    H, g, L = 2, 33, 64 * 13 + 5
    S = g + L
    q, k, v = _qkv(S, H, 600)
    scale = float(1 / np.sqrt(HD))
    route = O.sol_route(q, k, v, g, scale, 0.4)
    rng = np.random.default_rng(1)
    sel = (rng.random(route["sel"].shape) < 0.3).astype(np.uint8)
    nb = sel.shape[1]
    for i in range(nb):
        sel[:, i, i] = 1
    route["sel"] = sel
    route.update(g=g, block=64)
    ref = f32(O.sparse_attention(q, k, v, g, scale, route=route, tail=True))
    cfg = h3.H3SolAttnConfig(tau=0.4, tail=True)
    got = h3.H3SolAttn.attend_with_selection(*_dev(q, k, v), g, scale, cfg, torch.from_numpy(sel).cuda(),
                                             to_torch_bf16(route["cm"]), to_torch_bf16(route["vsum"]),
                                             torch.from_numpy(route["lens"]).cuda())
    assert_close(f32(to_np_bf16(got)), ref, rel=2e-2, cos=0.9995, what="given selection")


def test_dense_attention_large_vs_torch_fp32():
    import torch
    h3 = _h3()
    S, H = 8192 + 77, 2
    gen = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = [torch.randn((S, H, HD), device="cuda", generator=gen).to(torch.bfloat16) for _ in range(3)]
    scale = float(1 / np.sqrt(HD))
    got = h3.H3SolAttn.forward(q, k, v, 0, scale, None).float()
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float().transpose(0, 1), k.float().transpose(0, 1), v.float().transpose(0, 1), scale=scale).transpose(0, 1)
    err = ((got - ref).abs().max() / ref.abs().max()).item()
    cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
    assert err < 2e-2 and cos > 0.9995, (err, cos)


def test_topk_full_size_selection_properties():
    """Config-3 geometry (S=28520, 128-blocks): every (head, q-block) keeps the
    diagonal plus exactly ceil(0.25*nb) other blocks."""
    import torch
    h3 = _h3()
    S, H = 28520, 4
    gen = torch.Generator(device="cuda").manual_seed(4)
    q, k, v = [torch.randn((S, H, HD), device="cuda", generator=gen).to(torch.bfloat16) for _ in range(3)]
    cfg = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False)
    r = h3.H3SolAttn.route(q, k, v, 0, float(1 / np.sqrt(HD)), cfg)
    sel = r["sel"].cpu().numpy()
    nb = sel.shape[1]
    assert nb == 223
    assert (sel.sum(-1) == int(np.ceil(0.25 * nb)) + 1).all()
    assert all(sel[:, i, i].all() for i in range(nb))
    h3.context().check_device()
