"""GPU parity of one DiT block (H3Transformer.swift:1078-1159) through
wx_dit_block_forward against the oracle composition, in dense, SOL and top-k
attention modes, GELU and SwiGLU MLPs, and the PAB refresh/reuse paths."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


def make_block(seed, hidden, heads, ffn, mlp_kind, S, rot=96, hd=128):
    inner = heads * hd
    fc1_n = 2 * ffn if mlp_kind == 1 else ffn
    w = {}
    for i, (name, n, k) in enumerate([("qkv", 3 * inner, hidden), ("out", hidden, inner), ("fc1", fc1_n, hidden),
                                      ("fc2", hidden, ffn)]):
        wq, sc, bi = O.quantize(O.normal_f32((n, k), seed, 10 + i, std=0.02))
        w[name] = (wq, sc, bi, O.normal_bf16((n,), seed, 20 + i, std=0.02))
    w["q_norm"] = O.normal_bf16((hd,), seed, 30, mean=1.0, std=0.02)
    w["k_norm"] = O.normal_bf16((hd,), seed, 31, mean=1.0, std=0.02)
    w["norm1"] = O.normal_bf16((hidden,), seed, 32, mean=1.0, std=0.02)
    w["norm2"] = O.normal_bf16((hidden,), seed, 33, mean=1.0, std=0.02)
    mods = [O.normal_bf16((6, hidden), seed, 40 + j, std=0.1) for j in range(6)]
    h = O.normal_bf16((S, hidden), seed, 50)
    cos = O.normal_bf16((S, rot // 2), seed, 51)
    sin = O.normal_bf16((S, rot // 2), seed, 52)
    g = json.load(open(GOLD / "modrun.json"))
    rowmap = np.array((g["map"] * (S // 16 + 1))[:S], dtype=np.uint32)
    return w, mods, h, cos, sin, rowmap


def gpu_block(w, hidden, heads, ffn, mlp_kind, rot, eps, hd=128):
    import torch
    from wuxianhuabu_b200 import h3

    def lin(t, k):
        wq, sc, bi, b = t
        return h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                           to_torch_bf16(b) if b is not None else None)
    inner = heads * hd
    bw = h3.H3BlockWeights(lin(w["qkv"], hidden), lin(w["out"], inner), lin(w["fc1"], hidden), lin(w["fc2"], ffn),
                           to_torch_bf16(w["q_norm"]), to_torch_bf16(w["k_norm"]), to_torch_bf16(w["norm1"]),
                           to_torch_bf16(w["norm2"]))
    cfg = h3.H3DiTConfig(hidden=hidden, heads=heads, head_dim=hd, ffn=ffn, mlp_kind=mlp_kind, rot=rot, eps=eps,
                         layers=1)
    return h3.H3DiTBlocks(cfg, [bw])


def oracle_route(q, k, v, g, scale, sparse):
    """The oracle router of a sparse spec dict (topk_ratio -> top-k over 128-blocks, else SOL tau
    over 64-blocks with the tail term), as the oracle block composition takes it."""
    if sparse.get("topk_ratio"):
        r = O.topk_route(q, k, v, g, scale, sparse["topk_ratio"])
        r.update(g=g, block=128, tail=bool(sparse.get("tail", False)))
    else:
        sink = sparse.get("sink_blocks") or range(0, 0)
        r = O.sol_route(q, k, v, g, scale, sparse["tau"], sink=(sink.start, sink.stop))
        r.update(g=g, block=64, tail=bool(sparse.get("tail", True)))
    return r


def gpu_block_qkv(blk, bi, h, mods, rowmap):
    """The GPU block's qkv projection of h (norm1 + modulation, then the qkv linear with its
    LoRA adapters when attached: the kernels wx_dit_block_forward runs), before the per-head
    norm; [S, 3*inner] bf16 on the device."""
    from wuxianhuabu_b200 import h3
    w = blk.blocks[bi]
    m1 = h3.H3FusedKernels.fused_norm_modscale(h, w.norm1, mods[0], mods[1], rowmap, blk.cfg.eps)
    return w.qkv(m1)


def gpu_block_routing(blk, bi, h, mods, rowmap, cos, sin, sparse, g):
    """The block-selection decisions the GPU block will take on h: its own q/k/v (norm1 +
    modulation, the qkv projection, per-head RMSNorm + RoPE in place, the same kernels as
    wx_dit_block_forward) routed on the GPU. The oracle router on the same q/k/v must give the
    same tables bit for bit (asserted). Returns the selection [H, nb, nb] (host uint8)."""
    import torch
    from wuxianhuabu_b200 import h3
    cfg = blk.cfg
    w = blk.blocks[bi]
    S = h.shape[0]
    H, hd = cfg.heads, cfg.head_dim
    inner = H * hd
    qkv = gpu_block_qkv(blk, bi, h, mods, rowmap)
    h3.context().call("wx_qk_norm_rope_qkv", qkv.data_ptr(), S, H, hd, w.q_norm.data_ptr(), w.k_norm.data_ptr(),
                      cos.data_ptr(), sin.data_ptr(), cfg.rot, float(cfg.eps))
    q, k, v = (qkv[:, i * inner:(i + 1) * inner].view(S, H, hd) for i in range(3))
    scale = float(1 / np.sqrt(np.float32(hd)))
    hcfg = h3.H3SolAttnConfig(**sparse)
    got = h3.H3SolAttn.route(q, k, v, g, scale, hcfg)
    qn, kn, vn = (np.ascontiguousarray(to_np_bf16(t.contiguous())) for t in (q, k, v))
    ref = oracle_route(qn, kn, vn, g, scale, sparse)
    torch.cuda.synchronize()
    assert np.array_equal(got["sel"].cpu().numpy(), ref["sel"]), "GPU and oracle routers disagree on the same q/k"
    assert np.array_equal(to_np_bf16(got["cm"]), ref["cm"])
    assert np.array_equal(to_np_bf16(got["vsum"]), ref["vsum"])
    assert np.array_equal(got["lens"].cpu().numpy(), ref["lens"])
    if "thr" in got:
        assert np.array_equal(got["thr"].cpu().numpy().view(np.uint32), ref["thr"].view(np.uint32))
    else:
        assert np.array_equal(got["scores"].cpu().numpy().view(np.uint32), ref["scores"].view(np.uint32))
    return ref["sel"]


def route_with_selection(sel, g, scale, sparse):
    """An oracle route_fn that routes the oracle's own q/k/v (tail statistics) but takes the
    block selection the GPU block takes, so that a near-tie in the block scores cannot pick
    different blocks on the two sides."""
    def fn(q, k, v):
        r = oracle_route(q, k, v, g, scale, sparse)
        r["sel"] = sel
        return r
    return fn


CASES = [
    ("dense", 0, None),
    ("sol_all", 0, dict(tau=-100.0)),
    ("sol", 0, dict(tau=0.4)),
    ("topk", 0, dict(block=128, topk_ratio=0.25, tail=False)),
    ("dense_swiglu", 1, None),
]


@pytest.mark.parametrize("name,mlp_kind,sparse", CASES)
def test_block_vs_oracle(name, mlp_kind, sparse):
    import torch
    from wuxianhuabu_b200 import h3
    hidden, heads, ffn, rot, eps = 256, 2, 512, 96, 1e-6
    g, L = 44, 300
    S = g + L
    w, mods, h, cos, sin, rowmap = make_block(7, hidden, heads, ffn, mlp_kind, S, rot)
    cfgd = dict(heads=heads, head_dim=128, eps=eps, rot=rot, mlp_kind=mlp_kind)
    scale = float(1 / np.sqrt(np.float32(128)))
    blk = gpu_block(w, hidden, heads, ffn, mlp_kind, rot, eps)
    md = [to_torch_bf16(m) for m in mods]
    rm = torch.from_numpy(rowmap.view(np.int32)).cuda()
    ct, st = to_torch_bf16(cos), to_torch_bf16(sin)
    route_fn = None
    if sparse is not None:
        sel = gpu_block_routing(blk, 0, to_torch_bf16(h), md, rm, ct, st, sparse, g)
        route_fn = route_with_selection(sel, g, scale, sparse)
    ref, ref_at = O.block_forward(h, w, mods, rowmap, cos, sin, cfgd, route_fn=route_fn)
    ht = to_torch_bf16(h)
    spec = None if sparse is None else h3.H3SolAttnConfig(**sparse).spec(g)
    slot = torch.empty((S, hidden), dtype=torch.bfloat16, device="cuda")
    blk.block_forward(0, ht, md, rm, ct, st, spec, pab_slot=slot, refresh=True)
    h3.context().check_device()
    assert_close(f32(to_np_bf16(slot)), f32(ref_at), rel=2e-2, cos=0.999, what=f"{name} at")
    assert_close(f32(to_np_bf16(ht)), f32(ref), rel=2e-2, cos=0.999, what=f"{name} h")


def test_pab_reuse_equals_refresh_with_same_inputs():
    """A reuse step with the slot written by a refresh step on the same h and mods
    gives bit-identical output (PAB skips only the attention branch)."""
    import torch
    from wuxianhuabu_b200 import h3
    hidden, heads, ffn, rot, eps = 256, 2, 512, 96, 1e-6
    S = 300
    w, mods, h, cos, sin, rowmap = make_block(8, hidden, heads, ffn, 0, S, rot)
    blk = gpu_block(w, hidden, heads, ffn, 0, rot, eps)
    md = [to_torch_bf16(m) for m in mods]
    rm = torch.from_numpy(rowmap.view(np.int32)).cuda()
    c, s = to_torch_bf16(cos), to_torch_bf16(sin)
    slot = torch.empty((S, hidden), dtype=torch.bfloat16, device="cuda")
    h1 = to_torch_bf16(h)
    blk.block_forward(0, h1, md, rm, c, s, None, pab_slot=slot, refresh=True)
    h2 = to_torch_bf16(h)
    blk.block_forward(0, h2, md, rm, c, s, None, pab_slot=slot, refresh=False)
    torch.cuda.synchronize()
    assert torch.equal(h1, h2)
    # reuse with a different gate uses the current step's gate (PAB:19-21)
    md2 = list(md)
    md2[2] = md[2] * 2
    h3_ = to_torch_bf16(h)
    blk.block_forward(0, h3_, md2, rm, c, s, None, pab_slot=slot, refresh=False)
    assert not torch.equal(h1, h3_)
    h3.context().check_device()


@pytest.mark.parametrize("sparse", [None, dict(block=128, topk_ratio=0.25, tail=False)])
def test_block_real_h3_geometry_swiglu(sparse):
    """The production H3 geometry (H3Config, H3Common.swift:78-89): hidden 5376, 56 heads of
    128 (inner 7168 != hidden), SwiGLU FFN 14336 (fc1 N = 28672), eps 1e-5, rot 96."""
    import torch
    from wuxianhuabu_b200 import h3
    hidden, heads, ffn, rot, eps = 5376, 56, 14336, 96, 1e-5
    g, S = 128, 512
    w, mods, h, cos, sin, rowmap = make_block(12, hidden, heads, ffn, 1, S, rot)
    cfgd = dict(heads=heads, head_dim=128, eps=eps, rot=rot, mlp_kind=1)
    scale = float(1 / np.sqrt(np.float32(128)))

    def route_fn(q, k, v):
        if sparse is None:
            return None
        r = O.topk_route(q, k, v, g, scale, sparse["topk_ratio"])
        r.update(g=g, block=128, tail=False)
        return r

    ref, ref_at = O.block_forward(h, w, mods, rowmap, cos, sin, cfgd, route_fn=route_fn)
    blk = gpu_block(w, hidden, heads, ffn, 1, rot, eps)
    ht = to_torch_bf16(h)
    spec = None if sparse is None else h3.H3SolAttnConfig(**sparse).spec(g)
    slot = torch.empty((S, hidden), dtype=torch.bfloat16, device="cuda")
    blk.block_forward(0, ht, [to_torch_bf16(m) for m in mods], torch.from_numpy(rowmap.view(np.int32)).cuda(),
                      to_torch_bf16(cos), to_torch_bf16(sin), spec, pab_slot=slot, refresh=True)
    h3.context().check_device()
    assert_close(f32(to_np_bf16(slot)), f32(ref_at), rel=2e-2, cos=0.999, what="real geometry at")
    assert_close(f32(to_np_bf16(ht)), f32(ref), rel=2e-2, cos=0.999, what="real geometry h")
