"""Benchmark config 1 on the GPU: head_dim 64 (16 heads x 64, hidden 1024).

* attention with head_dim 64 against the oracle: dense at the config-1 size (S = 4096, 16 heads),
  and routed (top-k over 128-row blocks, SOL tau with the tail term) with strip rows and ragged
  tails — the reference's fused norm/RoPE and its SDPA take any head_dim
  (网络算子-融合-RMSNormRoPE-通用.swift:41-94, H3Transformer.swift:551);
* the config-1 DiT block exactly: S = 4096 (16 x 16 x 16 latent grid), hidden 1024, FFN 4096
  GELU, QK-RMSNorm eps 1e-6, 3-D RoPE over 32 frequency pairs (8/12/12 over t/h/w, theta 10000),
  dense attention, six-bit group-64 weights, against the oracle composition of the block.
Bound: max rel err <= 2e-2 and cosine >= 0.999."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16
from tests.test_gpu_block import gpu_block, make_block

pytestmark = pytest.mark.gpu
HD = 64
SCALE = float(1 / np.sqrt(np.float32(HD)))


@pytest.mark.parametrize("S,H,g,mode", [(4096, 16, 0, "dense"), (1000, 2, 100, "topk"), (1000, 2, 130, "sol"),
                                        (4096 + 37, 3, 300, "topk"), (260, 2, 17, "sol"), (77, 1, 0, "dense")])
def test_attention_head_dim_64_vs_oracle(S, H, g, mode):
    from wuxianhuabu_b200 import h3
    q, k, v = (O.normal_bf16((S, H, HD), 70 + S + H, i) for i in (1, 2, 3))
    if mode == "dense":
        cfg, ref = None, O.sparse_attention(q, k, v, 0, SCALE)
    elif mode == "sol":
        cfg = h3.H3SolAttnConfig(tau=0.4, tail=True)
        route = O.sol_route(q, k, v, g, SCALE, 0.4)
        route.update(g=g, block=64)
        ref = O.sparse_attention(q, k, v, g, SCALE, route=route, tail=True)
    else:
        cfg = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False)
        route = O.topk_route(q, k, v, g, SCALE, 0.25)
        route.update(g=g, block=128)
        ref = O.sparse_attention(q, k, v, g, SCALE, block=128, route=route, tail=False)
    tq, tk, tv = (to_torch_bf16(a) for a in (q, k, v))
    if cfg is not None:  # the routers at head_dim 64 are bit-exact with the oracle too
        got_r = h3.H3SolAttn.route(tq, tk, tv, g, SCALE, cfg)
        assert np.array_equal(got_r["sel"].cpu().numpy(), route["sel"])
        assert np.array_equal(to_np_bf16(got_r["vsum"]), route["vsum"])
    got = h3.H3SolAttn.forward(tq, tk, tv, g, SCALE, cfg)
    h3.context().check_device()
    assert_close(f32(to_np_bf16(got)), f32(ref), rel=2e-2, cos=0.999, what=f"hd64 {mode} S={S} g={g}")


def rope_tables_grid16(S=4096):
    """cos/sin [S, 32] of the config-1 latent grid (t, h, w each 0..15; 8/12/12 frequency
    pairs of theta 10000 per axis), as buildRope forms them (H3Layout.swift:725-740)."""
    t, hh, ww = np.meshgrid(np.arange(16), np.arange(16), np.arange(16), indexing="ij")
    pos = np.stack([t.ravel(), hh.ravel(), ww.ravel()], 1).astype(np.float32)[:S]
    ang = []
    for axis, nf in enumerate((8, 12, 12)):
        inv = (1.0 / 10000.0 ** (np.arange(nf, dtype=np.float64) * 2 / (2 * nf))).astype(np.float32)
        ang.append((pos[:, axis:axis + 1] * inv[None, :]).astype(np.float32))
    a = np.concatenate(ang, 1).astype(np.float64)
    return O.f32_to_bf16(np.cos(a).astype(np.float32)), O.f32_to_bf16(np.sin(a).astype(np.float32))


def test_config1_block_vs_oracle():
    import torch
    from wuxianhuabu_b200 import h3
    hidden, heads, ffn, rot, eps, S = 1024, 16, 4096, 64, 1e-6, 4096
    w, mods, h, _c, _s, rowmap = make_block(61, hidden, heads, ffn, 0, S, rot, hd=HD)
    cos, sin = rope_tables_grid16(S)
    cfgd = dict(heads=heads, head_dim=HD, eps=eps, rot=rot, mlp_kind=0)
    ref, ref_at = O.block_forward(h, w, mods, rowmap, cos, sin, cfgd)
    blk = gpu_block(w, hidden, heads, ffn, 0, rot, eps, hd=HD)
    ht = to_torch_bf16(h)
    slot = torch.empty((S, hidden), dtype=torch.bfloat16, device="cuda")
    blk.block_forward(0, ht, [to_torch_bf16(m) for m in mods], torch.from_numpy(rowmap.view(np.int32)).cuda(),
                      to_torch_bf16(cos), to_torch_bf16(sin), None, pab_slot=slot, refresh=True)
    h3.context().check_device()
    assert_close(f32(to_np_bf16(slot)), f32(ref_at), rel=2e-2, cos=0.999, what="config-1 block at")
    assert_close(f32(to_np_bf16(ht)), f32(ref), rel=2e-2, cos=0.999, what="config-1 block h")
