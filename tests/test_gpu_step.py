"""GPU parity of the whole sampler step (wx_dit_step: patch embed, blocks,
final head, Euler; H3Pipeline.swift:1398-1445 around H3DiT.forward) against the
oracle composition of the same step, plus the PAB refresh/reuse pair."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, cosine, f32, to_np_bf16, to_torch_bf16
from tests.test_gpu_block import gpu_block, make_block

pytestmark = pytest.mark.gpu

HIDDEN, HEADS, FFN, ROT, EPS, PATCH = 256, 2, 512, 96, 1e-6, 96


def _setup(n_blocks, S, text, seed=21):
    blocks = [make_block(seed + b, HIDDEN, HEADS, FFN, 0, S, ROT) for b in range(n_blocks)]
    _, _, _, cos, sin, rowmap = blocks[0]
    rng_lat = O.normal_f32((S - text, PATCH), seed, 90)
    embed_w = O.normal_f32((PATCH, HIDDEN), seed, 91, std=0.1)
    embed_b = O.normal_f32((HIDDEN,), seed, 92, std=0.1)
    out_w = O.normal_f32((HIDDEN, PATCH), seed, 93, std=0.05)
    out_b = O.normal_f32((PATCH,), seed, 94, std=0.05)
    final_norm = O.normal_bf16((HIDDEN,), seed, 95, mean=1.0, std=0.02)
    fshift = O.normal_bf16((HIDDEN,), seed, 96, std=0.1)
    fscale = O.normal_bf16((HIDDEN,), seed, 97, std=0.1)
    text_states = O.normal_bf16((text, HIDDEN), seed, 98)
    return blocks, cos, sin, rowmap, rng_lat, embed_w, embed_b, out_w, out_b, final_norm, fshift, fscale, text_states


def _oracle_step(blocks, cos, sin, rowmap, lat, embed_w, embed_b, out_w, out_b, final_norm, fshift, fscale,
                 text_states, text, video_start, dsigma):
    emb = O.f32_to_bf16(O.dense_f32(lat, embed_w, embed_b))
    h = np.concatenate([text_states, emb], 0)
    cfgd = dict(heads=HEADS, head_dim=128, eps=EPS, rot=ROT, mlp_kind=0)
    for (w, mods, _h, _c, _s, _r) in blocks:
        h, _ = O.block_forward(h, w, mods, rowmap, cos, sin, cfgd)
    m = O.norm_modscale(h[video_start:], final_norm, fshift[None], fscale[None], None, EPS)
    v = O.dense_f32(f32(m), out_w, out_b)
    out = lat.copy()
    out[video_start - text:] += -v * np.float32(dsigma)
    return out, v


def _gpu_model(blocks, embed_w, embed_b, out_w, out_b, final_norm):
    import torch
    from wuxianhuabu_b200 import h3
    dits = [gpu_block(w, HIDDEN, HEADS, FFN, 0, ROT, EPS) for (w, *_rest) in blocks]
    allb = h3.H3DiTBlocks(dits[0].cfg, [d.blocks[0] for d in dits])
    mods = [[to_torch_bf16(m) for m in b[1]] for b in blocks]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return h3.H3DiT(allb, mods, t(embed_w), t(embed_b), to_torch_bf16(final_norm), t(out_w), t(out_b)), mods


def test_step_matches_oracle_dense():
    import torch
    from wuxianhuabu_b200 import h3
    S, text, video_start, dsigma = 344, 40, 104, -0.05
    (blocks, cos, sin, rowmap, lat, ew, eb, ow, ob, fn, fsh, fsc, ts) = _setup(3, S, text)
    ref, ref_v = _oracle_step(blocks, cos, sin, rowmap, lat, ew, eb, ow, ob, fn, fsh, fsc, ts, text, video_start,
                              dsigma)
    dit, _ = _gpu_model(blocks, ew, eb, ow, ob, fn)
    lat_d = torch.from_numpy(lat.copy()).cuda()
    dit.step(S, text, video_start, to_torch_bf16(ts), lat_d, torch.from_numpy(rowmap.view(np.int32)).cuda(),
             to_torch_bf16(cos), to_torch_bf16(sin), to_torch_bf16(fsh), to_torch_bf16(fsc), None, 0, None, True,
             dsigma)
    h3.context().check_device()
    got = lat_d.cpu().numpy()
    assert np.array_equal(got[:video_start - text], lat[:video_start - text])  # cond rows untouched
    v_got = (got[video_start - text:] - lat[video_start - text:]) / -dsigma
    assert_close(v_got, ref_v, rel=2e-2, cos=0.999, what="step velocity")


def test_step_pab_window_and_sparse_policy():
    """Refresh then reuse on the same state reproduces the refresh output bit for bit;
    the mix policy with top-k layers stays close to the all-dense step."""
    import torch
    from wuxianhuabu_b200 import h3
    S, text, video_start, dsigma = 512, 40, 104, -0.05
    (blocks, cos, sin, rowmap, lat, ew, eb, ow, ob, fn, fsh, fsc, ts) = _setup(6, S, text, seed=31)
    dit, _ = _gpu_model(blocks, ew, eb, ow, ob, fn)
    args = lambda: (S, text, video_start, to_torch_bf16(ts))
    common = dict(rowmap=torch.from_numpy(rowmap.view(np.int32)).cuda(), cos=to_torch_bf16(cos),
                  sin=to_torch_bf16(sin), final_shift=to_torch_bf16(fsh), final_scale=to_torch_bf16(fsc))
    cfg = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False)
    pab = h3.H3AttnBroadcast(6)
    l1 = torch.from_numpy(lat.copy()).cuda()
    dit.step(*args(), l1, sparse_cfg=cfg, policy=h3.SparsePolicy.MIX, attn_bcast=pab, attn_refresh=True,
             dsigma=dsigma, sigma=1.0, **common)
    l2 = torch.from_numpy(lat.copy()).cuda()
    dit.step(*args(), l2, sparse_cfg=cfg, policy=h3.SparsePolicy.MIX, attn_bcast=pab, attn_refresh=False,
             dsigma=dsigma, sigma=1.0, **common)
    l3 = torch.from_numpy(lat.copy()).cuda()
    dit.step(*args(), l3, sparse_cfg=None, policy=h3.SparsePolicy.OFF, attn_bcast=None, attn_refresh=True,
             dsigma=dsigma, **common)
    torch.cuda.synchronize()
    h3.context().check_device()
    assert torch.equal(l1, l2)
    assert pab.cached_sigma == 1.0
    v1 = (l1.cpu().numpy() - lat)[video_start - text:]
    v3 = (l3.cpu().numpy() - lat)[video_start - text:]
    assert cosine(v1, v3) > 0.99


def test_step_with_audio_rows():
    """Audio segments of the packed layout (refAudio, then the target audio; H3Transformer.swift
    :1036-1062 embeds them with audioPatchW, :1176-1188 runs the audio head) inside a step:
    cond video rows on both sides of them come from the video latents in order."""
    import torch
    from wuxianhuabu_b200 import h3
    S, text, video_start, dsigma = 344, 40, 200, -0.05
    segs = [(104, 114), (114, 134)]  # refAudio (never denoised), target audio
    AD, vscale, da = 32, -1.25, 0.03
    (blocks, cos, sin, rowmap, _lat, ew, eb, ow, ob, fn, fsh, fsc, ts) = _setup(2, S, text, seed=31)
    n_audio = sum(e - s for s, e in segs)
    lat = O.normal_f32((S - text - n_audio, PATCH), 31, 80)
    alat = O.normal_f32((n_audio, AD), 31, 81)
    aew, aeb = O.normal_f32((AD, HIDDEN), 31, 82, std=0.1), O.normal_f32((HIDDEN,), 31, 83, std=0.1)
    aow, aob = O.normal_f32((HIDDEN, AD), 31, 84, std=0.05), O.normal_f32((AD,), 31, 85, std=0.05)
    afsh, afsc = O.normal_bf16((HIDDEN,), 31, 86, std=0.1), O.normal_bf16((HIDDEN,), 31, 87, std=0.1)
    # oracle: embed the runs in order, blocks, both heads
    rows, vi, ai, p = [], 0, 0, text
    for s0, s1 in segs + [(S, S)]:
        if s0 > p:
            rows.append(O.f32_to_bf16(O.dense_f32(lat[vi:vi + s0 - p], ew, eb)))
            vi += s0 - p
        if s1 > s0:
            rows.append(O.f32_to_bf16(O.dense_f32(alat[ai:ai + s1 - s0], aew, aeb)))
            ai += s1 - s0
        p = s1
    h = np.concatenate([ts] + rows, 0)
    cfgd = dict(heads=HEADS, head_dim=128, eps=EPS, rot=ROT, mlp_kind=0)
    for (w, mods, _h, _c, _s, _r) in blocks:
        h, _ = O.block_forward(h, w, mods, rowmap, cos, sin, cfgd)
    mv = O.norm_modscale(h[video_start:], fn, fsh[None], fsc[None], None, EPS)
    ref_v = O.dense_f32(f32(mv), ow, ob)
    ma = O.norm_modscale(h[segs[1][0]:segs[1][1]], fn, afsh[None], afsc[None], None, EPS)
    ref_a = O.dense_f32(f32(ma), aow, aob)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dit, _ = _gpu_model(blocks, ew, eb, ow, ob, fn)
    dit = h3.H3DiT(dit.blocks, dit.mods, t(ew), t(eb), to_torch_bf16(fn), t(ow), t(ob), t(aew), t(aeb), t(aow), t(aob))
    lat_d, alat_d = t(lat.copy()), t(alat.copy())
    audio = h3.H3AudioRows(segs, alat_d, 1, to_torch_bf16(afsh), to_torch_bf16(afsc), vscale, da)
    dit.step(S, text, video_start, to_torch_bf16(ts), lat_d, torch.from_numpy(rowmap.view(np.int32)).cuda(),
             to_torch_bf16(cos), to_torch_bf16(sin), to_torch_bf16(fsh), to_torch_bf16(fsc), None, 0, None, True,
             dsigma, audio=audio)
    h3.context().check_device()
    got, agot = lat_d.cpu().numpy(), alat_d.cpu().numpy()
    nv = S - video_start
    assert np.array_equal(got[:-nv], lat[:-nv])          # cond video rows untouched
    assert np.array_equal(agot[:10], alat[:10])          # refAudio rows untouched
    v_got = (got[-nv:] - lat[-nv:]) / -dsigma
    assert_close(v_got, ref_v, rel=2e-2, cos=0.999, what="step velocity with audio rows")
    a_got = (agot[10:] - alat[10:]) / np.float32(vscale * da)
    assert_close(a_got, ref_a, rel=2e-2, cos=0.999, what="audio head")


def test_step_cfg_guidance():
    """The SelfLift CFG step (SelfLiftH3-(h3专属).swift:826-845) through wx_dit_step_guided:
    each branch's video output matches the oracle composition of the step; the guided output is
    exactly v_neg + cfg*(v_pos - v_neg) of the two single-branch outputs; the negative branch
    neither reads nor writes the PAB slots; update=1 without CFG equals wx_dit_step."""
    import torch
    from wuxianhuabu_b200 import h3
    S, text, video_start, dsigma, cfg = 344, 40, 104, -0.05, 4.0
    (blocks, cos, sin, rowmap, lat, ew, eb, ow, ob, fn, fsh, fsc, ts) = _setup(3, S, text, seed=41)
    ts_neg = O.normal_bf16((text, HIDDEN), 41, 99)
    dit, _ = _gpu_model(blocks, ew, eb, ow, ob, fn)
    common = dict(rowmap=torch.from_numpy(rowmap.view(np.int32)).cuda(), cos=to_torch_bf16(cos),
                  sin=to_torch_bf16(sin), final_shift=to_torch_bf16(fsh), final_scale=to_torch_bf16(fsc))
    pos_t, neg_t = to_torch_bf16(ts), to_torch_bf16(ts_neg)
    nv = S - video_start
    lat_d = torch.from_numpy(lat.copy()).cuda()

    def run(text_states, **kw):
        v = torch.full((nv, PATCH), float("nan"), dtype=torch.float32, device="cuda")
        dit.step(S, text, video_start, text_states, lat_d, sparse_cfg=None, policy=0, attn_refresh=True,
                 dsigma=dsigma, update=False, velocity_out=v, **dict(dict(attn_bcast=None), **kw), **common)
        return v

    vp = run(pos_t)
    vn = run(neg_t)
    vc = run(pos_t, text_states_neg=neg_t, cfg_scale=cfg)
    h3.context().check_device()
    assert torch.equal(lat_d, torch.from_numpy(lat).cuda()), "update=0 must leave the latents untouched"
    vp_, vn_, vc_ = (t.cpu().numpy() for t in (vp, vn, vc))
    assert np.array_equal(vc_, vn_ + (vp_ - vn_) * np.float32(cfg)), "guided output is not the CFG combination"
    # each branch against the oracle composition (its velocity is minus the video output)
    _, ref_pos = _oracle_step(blocks, cos, sin, rowmap, lat, ew, eb, ow, ob, fn, fsh, fsc, ts, text, video_start,
                              dsigma)
    _, ref_neg = _oracle_step(blocks, cos, sin, rowmap, lat, ew, eb, ow, ob, fn, fsh, fsc, ts_neg, text,
                              video_start, dsigma)
    assert_close(-vp_, ref_pos, rel=2e-2, cos=0.999, what="positive branch")
    assert_close(-vn_, ref_neg, rel=2e-2, cos=0.999, what="negative branch")
    # PAB: a guided refresh writes the positive branch's attention outputs only, so a
    # positive-only reuse step on the same state reproduces the positive output exactly
    pab = h3.H3AttnBroadcast(3)
    vc2 = run(pos_t, text_states_neg=neg_t, cfg_scale=cfg, attn_bcast=pab)
    v_reuse = torch.full((nv, PATCH), float("nan"), dtype=torch.float32, device="cuda")
    dit.step(S, text, video_start, pos_t, lat_d, sparse_cfg=None, policy=0, attn_bcast=pab, attn_refresh=False,
             dsigma=dsigma, update=False, velocity_out=v_reuse, **common)
    torch.cuda.synchronize()
    assert torch.equal(vc2, vc)
    assert torch.equal(v_reuse, vp)
    # update=1 without guidance is wx_dit_step
    l1, l2 = torch.from_numpy(lat.copy()).cuda(), torch.from_numpy(lat.copy()).cuda()
    dit.step(S, text, video_start, pos_t, l1, sparse_cfg=None, policy=0, attn_bcast=None, attn_refresh=True,
             dsigma=dsigma, **common)
    vo = torch.empty((nv, PATCH), dtype=torch.float32, device="cuda")
    dit.step(S, text, video_start, pos_t, l2, sparse_cfg=None, policy=0, attn_bcast=None, attn_refresh=True,
             dsigma=dsigma, velocity_out=vo, **common)
    h3.context().check_device()
    assert torch.equal(l1, l2)
    assert torch.equal(vo, vp)
