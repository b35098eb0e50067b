"""The per-layer phase trace (wx_ctx_trace_enable / _read), the counterpart of the reference's
NA_H3PROF timers (H3Transformer.swift:445-450, 575-597: qkv, ropeN, attn(mode), out, tot per layer).

* one record per block forward, layers counted from 0 since enable/read, in call order;
* the mode (dense / sparse / PAB reuse) and which phases ran: a refresh runs all phases (rope
  takes no time of its own where QK-norm + RoPE run in the q|k|v GEMM's epilogue), a reuse only
  the cached gated residual (out) and the MLP;
* the phases add up to the block's total (they tile it: each phase ends where the next begins);
* a read clears the record, and disabling stops recording;
* the sampler step records one block per layer (two forwards per layer for the CFG step);
* tracing changes no result (outputs bit-identical with and without it)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import to_torch_bf16
from tests.test_gpu_block import gpu_block, make_block

pytestmark = pytest.mark.gpu
PHASES = ("norm1", "qkv", "rope", "attn", "out", "mlp")


def _check_tiles(r):
    parts = sum(r[p + "_ms"] for p in PHASES)
    assert r["total_ms"] > 0
    assert abs(parts - r["total_ms"]) <= 1e-3 * r["total_ms"] + 2e-3, r


def test_block_trace_records_modes_and_phases():
    import torch
    from wuxianhuabu_b200 import h3
    hidden, heads, ffn, rot, eps, S = 256, 2, 512, 96, 1e-6, 700
    w, mods, h, cos, sin, rowmap = make_block(12, hidden, heads, ffn, 0, S, rot)
    blk = gpu_block(w, hidden, heads, ffn, 0, rot, eps)
    md = [to_torch_bf16(m) for m in mods]
    rm = torch.from_numpy(rowmap.view(np.int32)).cuda()
    c, s = to_torch_bf16(cos), to_torch_bf16(sin)
    slot = torch.empty((S, hidden), dtype=torch.bfloat16, device="cuda")
    topk = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False).spec(200)
    ctx = h3.context()

    def run(trace):
        outs = []
        if trace:
            ctx.trace(True)
        for spec, refresh in ((None, True), (topk, True), (topk, False)):
            x = to_torch_bf16(h)
            blk.block_forward(0, x, md, rm, c, s, spec, pab_slot=slot, refresh=refresh)
            outs.append(x)
        torch.cuda.synchronize()
        recs = ctx.trace_read() if trace else []
        if trace:
            ctx.trace(False)
        return outs, recs

    plain, _ = run(False)
    traced, recs = run(True)
    ctx.check_device()
    for a, b in zip(plain, traced):
        assert torch.equal(a, b)
    assert [r["layer"] for r in recs] == [0, 1, 2]
    assert [r["mode"] for r in recs] == ["dense", "sparse", "reuse"]
    for r in recs[:2]:  # rope is 0 where QK-norm + RoPE run in the q|k|v GEMM's epilogue
        assert all(r[p + "_ms"] > 0 for p in PHASES if p != "rope") and r["rope_ms"] >= 0, r
    assert recs[2]["out_ms"] > 0 and recs[2]["mlp_ms"] > 0
    assert all(recs[2][p + "_ms"] == 0 for p in ("norm1", "qkv", "rope", "attn")), recs[2]
    for r in recs:
        _check_tiles(r)
    # read cleared the record; with tracing off nothing is recorded
    assert ctx.trace_read() == []
    x = to_torch_bf16(h)
    blk.block_forward(0, x, md, rm, c, s, None, pab_slot=slot, refresh=True)
    assert ctx.trace_read() == []
    lines = h3.Context.format_trace(recs).splitlines()
    assert len(lines) == 3 and lines[1].startswith("[PROF] L02 ") and "attn(sol)=" in lines[1]


def test_step_trace_one_record_per_layer():
    import torch
    from wuxianhuabu_b200 import h3
    from tests.test_gpu_step import _gpu_model, _setup
    S, text, video_start, dsigma, nb = 344, 40, 104, -0.05, 4
    (blocks, cos, sin, rowmap, lat, ew, eb, ow, ob, fn, fsh, fsc, ts) = _setup(nb, S, text, seed=41)
    dit, _ = _gpu_model(blocks, ew, eb, ow, ob, fn)
    common = dict(rowmap=torch.from_numpy(rowmap.view(np.int32)).cuda(), cos=to_torch_bf16(cos),
                  sin=to_torch_bf16(sin), final_shift=to_torch_bf16(fsh), final_scale=to_torch_bf16(fsc))
    cfg = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False)
    ctx = h3.context()
    ctx.trace(True)
    lat_d = torch.from_numpy(lat.copy()).cuda()
    dit.step(S, text, video_start, to_torch_bf16(ts), lat_d, sparse_cfg=cfg, policy=h3.SparsePolicy.MIX,
             attn_bcast=None, attn_refresh=True, dsigma=dsigma, **common)
    recs = ctx.trace_read()
    assert [r["layer"] for r in recs] == list(range(nb))
    modes = [h3.sparse_mode_for_layer(i, nb, h3.SparsePolicy.MIX) for i in range(nb)]
    assert [r["mode"] for r in recs] == ["dense" if m == 0 else "sparse" for m in modes]
    for r in recs:
        _check_tiles(r)
    # CFG step: the positive and the negative forward, each over every layer
    neg = to_torch_bf16(O.normal_bf16((text, 256), 41, 7))
    lat_g = torch.from_numpy(lat.copy()).cuda()
    dit.step(S, text, video_start, to_torch_bf16(ts), lat_g, sparse_cfg=None, policy=h3.SparsePolicy.OFF,
             attn_bcast=None, attn_refresh=True, dsigma=dsigma, text_states_neg=neg, cfg_scale=3.0, **common)
    recs = ctx.trace_read()
    ctx.trace(False)
    ctx.check_device()
    assert [r["layer"] for r in recs] == list(range(2 * nb))
    assert all(r["mode"] == "dense" for r in recs)
