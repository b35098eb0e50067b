"""GPU parity at the BASELINE geometries (configs 3-5 of the benchmark), against the oracle:

* routing tables bit-exact at full size: the top-k router of config 3 (S = 28520 and 111600,
  24 heads, 128-row blocks, g = 0) and the SOL-tau router (tau 1.3, 64-row blocks, a sink block,
  tail statistics) at the config-4 and config-5 packed geometries (S = 29032, g = 512;
  S = 126512, g = 14912) — SOL:455-497 for SOL, the benchmark's top-k for config 3;
* attention on row slabs of the config-5 sequence (S = 126512, g = 14912, 24 heads): strip rows,
  video rows and the ragged last video block, top-k and SOL-tau, against the oracle's row-range
  attention (SOL:110-231 semantics; the reference's chunked path for S > 35000,
  H3Transformer.swift:488-544, is numerically the same computation, SOL:888-915);
* one DiT block at the configs' width (hidden 3072, 24 x 128 heads, FFN 12288 GELU, rot 96) with
  top-k and SOL attention, the oracle taking the GPU block's own block selection;
* the sampler step under the mix policy (dense anchor layers + sparse layers) against the
  oracle composition, again with the GPU's selections per sparse layer;
* the SOL self-test's production geometry (Case R: 56 heads, g = 934, L = 9324) with the
  production router: tables bit-exact, attention of four heads over every row.

Tolerances: routing tables bit-exact; attention and block outputs max rel err <= 2e-2 and
cosine >= 0.999; the step's velocity the same.
Inputs are seeded synthetic tensors with the configs' shapes and distributions (no dataset).
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16
from tests.test_gpu_block import (gpu_block, gpu_block_routing, make_block, oracle_route,
                                  route_with_selection)

pytestmark = pytest.mark.gpu
HD = 128
SCALE = float(1 / np.sqrt(np.float32(HD)))


def _qkv_device(S, H, seed):
    """q, k, v [S, H, 128] bf16 ~ N(0, 1) generated on the device (seeded)."""
    import torch
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn((S, H, HD), device="cuda", generator=gen).to(torch.bfloat16) for _ in range(3)]


def _host(t):
    return np.ascontiguousarray(to_np_bf16(t))


def _check_tables(got, ref, score_key):
    import torch
    torch.cuda.synchronize()
    assert np.array_equal(got["sel"].cpu().numpy(), ref["sel"]), "sel"
    assert np.array_equal(got[score_key].cpu().numpy().view(np.uint32), ref[score_key].view(np.uint32)), score_key
    assert np.array_equal(to_np_bf16(got["cm"]), ref["cm"]), "cm"
    assert np.array_equal(to_np_bf16(got["vsum"]), ref["vsum"]), "vsum"
    assert np.array_equal(got["lens"].cpu().numpy(), ref["lens"]), "lens"


@pytest.mark.parametrize("S", [28520, 111600])
def test_topk_route_bit_exact_config3(S):
    """Config 3: diagonal + ceil(0.25 nb) best blocks over mean-pooled Q.K block scores."""
    from wuxianhuabu_b200 import h3
    H = 24
    q, k, v = _qkv_device(S, H, 1000 + S)
    cfg = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False)
    got = h3.H3SolAttn.route(q, k, v, 0, SCALE, cfg)
    ref = O.topk_route(_host(q), _host(k), _host(v), 0, SCALE, 0.25)
    nb = ref["sel"].shape[1]
    assert nb == (S + 127) // 128
    assert (ref["sel"].sum(-1) == int(np.ceil(0.25 * nb)) + 1).all()
    _check_tables(got, ref, "scores")
    h3.context().check_device()


@pytest.mark.parametrize("S,g", [(29032, 512), (126512, 14912)])
def test_sol_route_bit_exact_packed_geometry(S, g):
    """The production router (tau 1.3, 64-row blocks) at the config-4/5 packed sequences,
    with a sink block forced exact."""
    from wuxianhuabu_b200 import h3
    H = 24
    q, k, v = _qkv_device(S, H, 2000 + S)
    cfg = h3.H3SolAttnConfig(tau=1.3, sink_blocks=range(0, 1), tail=True)
    got = h3.H3SolAttn.route(q, k, v, g, SCALE, cfg)
    ref = O.sol_route(_host(q), _host(k), _host(v), g, SCALE, 1.3, sink=(0, 1))
    _check_tables(got, ref, "thr")
    h3.context().check_device()


def _slabs(S, g):
    """Row ranges of the config-5 sequence compared with the oracle: the first strip rows
    (text), the last strip rows (reference images, up to the strip end), a slab of video rows
    straddling a block boundary, and the ragged last video block."""
    last = g + ((S - g) // 128) * 128  # first row of the last (partial) 128-row block
    return [(0, 128), (g - 128, g), (g + 40000 - 64, g + 40000 + 192), (last, S)]


@pytest.mark.parametrize("mode", ["topk", "sol"])
def test_attention_row_slabs_config5(mode):
    """Config-5 geometry (S = 126512: 512 text + 4 x 3600 reference-image rows in the strip,
    111600 video rows). The GPU attends all 24 heads; the oracle recomputes three of them on the
    row slabs, with the same routing tables (bit-exact with the GPU's, checked above)."""
    import torch
    from wuxianhuabu_b200 import h3
    S, g, H = 126512, 14912, 24
    q, k, v = _qkv_device(S, H, 3000 + (mode == "sol"))
    if mode == "topk":
        sparse = dict(block=128, topk_ratio=0.25, tail=False)
    else:
        sparse = dict(tau=1.3, tail=True)
    cfg = h3.H3SolAttnConfig(**sparse)
    out = h3.H3SolAttn.forward(q, k, v, g, SCALE, cfg)
    h3.context().check_device()
    heads = [0, 11, 23]
    qs, ks, vs = (np.ascontiguousarray(_host(t[:, heads, :])) for t in (q, k, v))
    route = oracle_route(qs, ks, vs, g, SCALE, sparse)
    got_all = _host(out[:, heads, :])
    torch.cuda.synchronize()
    for r0, r1 in _slabs(S, g):
        ref = O.attention_rows(qs, ks, vs, g, SCALE, r0, r1, block=route["block"], route=route, tail=route["tail"])
        assert_close(f32(got_all[r0:r1]), f32(ref), rel=2e-2, cos=0.999, what=f"{mode} rows [{r0}, {r1})")


@pytest.mark.parametrize("name,sparse", [("topk", dict(block=128, topk_ratio=0.25, tail=False)),
                                         ("sol", dict(tau=1.3, tail=True))])
def test_block_config_width_vs_oracle(name, sparse):
    """One block at the width of configs 3-5 (hidden 3072, 24 heads of 128, FFN 12288 GELU,
    rot 96, eps 1e-6) over 512 strip rows + 1536 video rows."""
    import torch
    from wuxianhuabu_b200 import h3
    hidden, heads, ffn, rot, eps = 3072, 24, 12288, 96, 1e-6
    g, S = 512, 2048
    w, mods, h, cos, sin, rowmap = make_block(41, hidden, heads, ffn, 0, S, rot)
    blk = gpu_block(w, hidden, heads, ffn, 0, rot, eps)
    md = [to_torch_bf16(m) for m in mods]
    rm = torch.from_numpy(rowmap.view(np.int32)).cuda()
    ct, st = to_torch_bf16(cos), to_torch_bf16(sin)
    sel = gpu_block_routing(blk, 0, to_torch_bf16(h), md, rm, ct, st, sparse, g)
    cfgd = dict(heads=heads, head_dim=HD, eps=eps, rot=rot, mlp_kind=0)
    ref, ref_at = O.block_forward(h, w, mods, rowmap, cos, sin, cfgd,
                                  route_fn=route_with_selection(sel, g, SCALE, sparse))
    ht = to_torch_bf16(h)
    slot = torch.empty((S, hidden), dtype=torch.bfloat16, device="cuda")
    blk.block_forward(0, ht, md, rm, ct, st, h3.H3SolAttnConfig(**sparse).spec(g), pab_slot=slot, refresh=True)
    h3.context().check_device()
    assert_close(f32(to_np_bf16(slot)), f32(ref_at), rel=2e-2, cos=0.999, what=f"{name} at (config width)")
    assert_close(f32(to_np_bf16(ht)), f32(ref), rel=2e-2, cos=0.999, what=f"{name} h (config width)")


HIDDEN, HEADS, FFN, ROT, EPS, PATCH = 256, 2, 512, 96, 1e-6, 96


@pytest.mark.parametrize("name,sparse", [("topk", dict(block=128, topk_ratio=0.25, tail=False)),
                                         ("sol", dict(tau=0.4, tail=True))])
def test_step_mix_policy_vs_oracle(name, sparse):
    """wx_dit_step with the mix policy over 8 blocks (sparseModeForLayer, H3Layout.swift:896-906:
    layers 0, 1, 4, 5, 6, 7 dense, 2 and 3 sparse) against the oracle composition of the step.
    The GPU's selections of the sparse layers come from running its blocks one by one through the
    same kernels; the step's own latent update must equal that block-by-block run bit for bit,
    so the oracle is given exactly the selections the step used."""
    import torch
    from wuxianhuabu_b200 import h3
    nblk, S, text, video_start, dsigma = 8, 640, 40, 128, -0.05
    g = video_start
    blocks = [make_block(51 + b, HIDDEN, HEADS, FFN, 0, S, ROT) for b in range(nblk)]
    _, _, _, cos, sin, rowmap = blocks[0]
    lat = O.normal_f32((S - text, PATCH), 51, 90)
    ew, eb = O.normal_f32((PATCH, HIDDEN), 51, 91, std=0.1), O.normal_f32((HIDDEN,), 51, 92, std=0.1)
    ow, ob = O.normal_f32((HIDDEN, PATCH), 51, 93, std=0.05), O.normal_f32((PATCH,), 51, 94, std=0.05)
    fn = O.normal_bf16((HIDDEN,), 51, 95, mean=1.0, std=0.02)
    fsh, fsc = O.normal_bf16((HIDDEN,), 51, 96, std=0.1), O.normal_bf16((HIDDEN,), 51, 97, std=0.1)
    ts = O.normal_bf16((text, HIDDEN), 51, 98)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    ew_t, eb_t, ow_t, ob_t, fn_t = t(ew), t(eb), t(ow), t(ob), to_torch_bf16(fn)
    fsh_t, fsc_t, ts_t = to_torch_bf16(fsh), to_torch_bf16(fsc), to_torch_bf16(ts)
    dits = [gpu_block(w, HIDDEN, HEADS, FFN, 0, ROT, EPS) for (w, *_r) in blocks]
    allb = h3.H3DiTBlocks(dits[0].cfg, [d.blocks[0] for d in dits])
    mods_t = [[to_torch_bf16(m) for m in b[1]] for b in blocks]
    dit = h3.H3DiT(allb, mods_t, ew_t, eb_t, fn_t, ow_t, ob_t)
    rm, ct, st = torch.from_numpy(rowmap.view(np.int32)).cuda(), to_torch_bf16(cos), to_torch_bf16(sin)
    cfg = h3.H3SolAttnConfig(**sparse)
    modes = [h3.sparse_mode_for_layer(b, nblk, h3.SparsePolicy.MIX) for b in range(nblk)]
    assert [b for b in range(nblk) if modes[b] != 0] == [2, 3]

    # block-by-block run on the GPU: patch embed, each block (recording the sparse layers'
    # selections), final head and Euler update, with the kernels the step uses
    ctx = h3.context()
    emb32 = torch.empty((S - text, HIDDEN), dtype=torch.float32, device="cuda")
    lat_d = t(lat.copy())
    ctx.call("wx_dense_f32", lat_d.data_ptr(), S - text, PATCH, ew_t.data_ptr(), HIDDEN, eb_t.data_ptr(),
             emb32.data_ptr())
    hb = torch.empty((S, HIDDEN), dtype=torch.bfloat16, device="cuda")
    hb[:text] = ts_t
    ctx.call("wx_f32_to_bf16", emb32.data_ptr(), (S - text) * HIDDEN, hb[text:].data_ptr())
    sels = {}
    for b in range(nblk):
        spec = None
        if modes[b] != 0:
            sels[b] = gpu_block_routing(allb, b, hb.clone(), mods_t[b], rm, ct, st, sparse, g)
            spec = cfg.spec(g)
        allb.block_forward(b, hb, mods_t[b], rm, ct, st, spec)
    hv = h3.H3FusedKernels.fused_norm_modscale(hb[video_start:].contiguous(), fn_t, fsh_t[None], fsc_t[None], None,
                                               EPS)
    v32 = torch.empty((S - video_start, PATCH), dtype=torch.float32, device="cuda")
    hv32 = hv.float()
    ctx.call("wx_dense_f32", hv32.data_ptr(), S - video_start, HIDDEN, ow_t.data_ptr(), PATCH, ob_t.data_ptr(),
             v32.data_ptr())
    manual = lat_d.clone()
    ctx.call("wx_euler_update", manual[video_start - text:].data_ptr(), v32.data_ptr(), v32.numel(), float(dsigma))

    # the step itself
    lat_s = t(lat.copy())
    dit.step(S, text, video_start, ts_t, lat_s, rm, ct, st, fsh_t, fsc_t, cfg, h3.SparsePolicy.MIX, None, True,
             dsigma)
    ctx.check_device()
    torch.cuda.synchronize()
    assert torch.equal(lat_s, manual), "the step and its block-by-block run differ"

    # oracle composition with the GPU's selections on layers 2 and 3
    emb = O.f32_to_bf16(O.dense_f32(lat, ew, eb))
    h = np.concatenate([ts, emb], 0)
    cfgd = dict(heads=HEADS, head_dim=HD, eps=EPS, rot=ROT, mlp_kind=0)
    for b, (w, mods, _h, _c, _s, _r) in enumerate(blocks):
        route_fn = route_with_selection(sels[b], g, SCALE, sparse) if b in sels else None
        h, _ = O.block_forward(h, w, mods, rowmap, cos, sin, cfgd, route_fn=route_fn)
    m = O.norm_modscale(h[video_start:], fn, fsh[None], fsc[None], None, EPS)
    ref_v = O.dense_f32(f32(m), ow, ob)
    got = lat_s.cpu().numpy()
    assert np.array_equal(got[:video_start - text], lat[:video_start - text])
    v_got = (got[video_start - text:] - lat[video_start - text:]) / -dsigma
    assert_close(v_got, ref_v, rel=2e-2, cos=0.999, what=f"mix-policy step velocity ({name})")


def test_sol_case_r_production_geometry():
    """The SOL self-test's production geometry (Case R, SOL:874-886: 56 heads, g = 934 strip rows,
    L = 9324 video rows, head_dim 128; neither g nor L a multiple of 64) with the production router
    (tau 1.3, 64-row blocks, tail): routing tables bit-exact over all 56 heads, and the attention
    of four heads over every row against the oracle."""
    import json
    from pathlib import Path
    from wuxianhuabu_b200 import h3
    gd = json.load(open(Path(__file__).resolve().parent / "golden" / "sol_selftest.json"))["caseR"]
    H, g, L = gd["h"], gd["g"], gd["L"]
    S = g + L
    q, k, v = _qkv_device(S, H, 4000)
    cfg = h3.H3SolAttnConfig(tau=1.3, tail=True)
    got = h3.H3SolAttn.route(q, k, v, g, SCALE, cfg)
    qh, kh, vh = _host(q), _host(k), _host(v)
    ref = O.sol_route(qh, kh, vh, g, SCALE, 1.3)
    _check_tables(got, ref, "thr")
    out = h3.H3SolAttn.forward(q, k, v, g, SCALE, cfg)
    h3.context().check_device()
    heads = [0, 17, 38, 55]
    qs, ks, vs = (np.ascontiguousarray(a[:, heads, :]) for a in (qh, kh, vh))
    route = O.sol_route(qs, ks, vs, g, SCALE, 1.3)
    route.update(g=g, block=64)
    want = O.sparse_attention(qs, ks, vs, g, SCALE, route=route, tail=True)
    assert_close(f32(_host(out[:, heads, :])), f32(want), rel=2e-2, cos=0.999, what="case R attention")
