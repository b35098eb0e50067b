"""A block forward captured as a CUDA graph (wx_dit_block_graph_create) and replayed
(wx_graph_launch) against the direct call: bit-identical outputs for dense, top-k (whose duo
attention kernel runs on the side stream, joined inside the graph) and SOL blocks, on new
input contents written into the same buffers between replays, head_dim 128 and 64; nothing
runs at capture time; the launch counter advances by the graph's kernels per replay."""
import numpy as np
import pytest

from tests._util import to_torch_bf16
from tests.test_gpu_block import gpu_block, make_block

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,hd", [("dense", 128), ("topk", 128), ("sol", 128), ("dense", 64)])
def test_block_graph_replays_the_block(mode, hd):
    import torch
    from wuxianhuabu_b200 import h3
    S, heads, g = (1000, 2, 200) if hd == 128 else (777, 4, 0)
    rot = 96 if hd == 128 else 64
    w, mods, h0, cos, sin, rowmap = make_block(31, 256, heads, 512, 0, S, rot, hd=hd)
    _, _, h1, _, _, _ = make_block(32, 256, heads, 512, 0, S, rot, hd=hd)
    blk = gpu_block(w, 256, heads, 512, 0, rot, 1e-6, hd=hd)
    spec = None
    if mode == "topk":
        spec = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False).spec(g)
    elif mode == "sol":
        spec = h3.H3SolAttnConfig(tau=0.4, tail=True).spec(g)
    md = [to_torch_bf16(m) for m in mods]
    rm = torch.from_numpy(rowmap.view(np.int32)).cuda()
    c, s = to_torch_bf16(cos), to_torch_bf16(sin)
    ctx = h3.context()
    # direct calls
    want = []
    for hin in (h0, h1):
        x = to_torch_bf16(hin)
        slot = torch.empty((S, 256), dtype=torch.bfloat16, device="cuda")
        blk.block_forward(0, x, md, rm, c, s, spec, pab_slot=slot, refresh=True)
        want.append((x.clone(), slot.clone()))
    # one graph over fixed buffers
    hbuf = to_torch_bf16(h0)
    slot = torch.zeros((S, 256), dtype=torch.bfloat16, device="cuda")
    n0 = ctx.lib.wx_ctx_launch_count(ctx.h)
    graph = blk.block_graph(0, hbuf, md, rm, c, s, spec, pab_slot=slot, refresh=True)
    torch.cuda.synchronize()
    assert ctx.lib.wx_ctx_launch_count(ctx.h) == n0          # capture runs nothing
    assert torch.equal(hbuf, to_torch_bf16(h0)) and not slot.any()
    k = graph.kernels()
    assert k >= 8
    for hin, (wh, ws) in zip((h0, h1), want):
        hbuf.copy_(to_torch_bf16(hin))
        graph.launch()
        torch.cuda.synchronize()
        assert torch.equal(hbuf, wh) and torch.equal(slot, ws)
    assert ctx.lib.wx_ctx_launch_count(ctx.h) == n0 + 2 * k
    graph.close()
    ctx.check_device()
