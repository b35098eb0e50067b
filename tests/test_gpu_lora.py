"""LoRA adapters of the quantized linears (LoraRef / loraDelta, H3Common.swift:407-433,
applied in MfLinear.forward :369-375) against the CPU oracle: the packed operands
bit-exact, the linear with one and several adapters under each epilogue, and a DiT
block with adapters on all four linears."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16
from tests.test_gpu_block import gpu_block, make_block

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


def _adapters(seed, k, n, ranks, scales):
    return [(O.normal_bf16((k, r), seed, 100 + i, std=0.05), O.normal_bf16((r, n), seed, 200 + i, std=0.05), s)
            for i, (r, s) in enumerate(zip(ranks, scales))]


def _refs(ad):
    from wuxianhuabu_b200 import h3
    return [h3.LoraRef(to_torch_bf16(a), to_torch_bf16(b), s) for a, b, s in ad]


def _linear(seed, n, k, bias=True):
    import torch
    from wuxianhuabu_b200 import h3
    wq, sc, bi = O.quantize(O.normal_f32((n, k), seed, 1, std=0.02))
    b = O.normal_bf16((n,), seed, 2, std=0.02) if bias else None
    lin = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                      to_torch_bf16(b) if bias else None)
    return lin, (wq, sc, bi, b)


def test_lora_pack_bit_exact():
    """at = bf16(scale_i * A_i^T) stacked, bt = B_i^T side by side, zero padding to R."""
    from wuxianhuabu_b200 import h3
    k, n = 192, 128
    ad = _adapters(3, k, n, [8, 40], [0.5, 1.75])
    lin, _ = _linear(3, n, k)
    lin.set_lora(_refs(ad))
    pack = lin.lora_pack()
    assert pack.R == 64 and pack.n == n and pack.k == k
    at = to_np_bf16(lin._pack[1]).reshape(64, k)
    bt = to_np_bf16(lin._pack[2]).reshape(n, 64)
    off = 0
    for a, b, s in ad:
        r = a.shape[1]
        want = O.f32_to_bf16(np.float32(s) * O.bf16_to_f32(a).T)
        assert np.array_equal(at[off:off + r], want)
        assert np.array_equal(bt[:, off:off + r], b.T)
        off += r
    assert not at[off:].any() and not bt[:, off:].any()
    h3.context().check_device()


@pytest.mark.parametrize("m", [300, 1000])
@pytest.mark.parametrize("ranks,scales", [([16], [1.0]), ([8, 40], [0.5, 1.5]), ([100], [0.8])])
@pytest.mark.parametrize("epi", ["none", "gelu", "gate_resid"])
def test_qlinear_lora_vs_oracle(m, ranks, scales, epi):
    import torch
    from wuxianhuabu_b200 import h3
    k, n = 512, 768
    lin, (wq, sc, bi, b) = _linear(11 + m, n, k)
    ad = _adapters(11 + m, k, n, ranks, scales)
    lin.set_lora(_refs(ad))
    x = O.normal_bf16((m, k), 11 + m, 3)
    kw, tkw = {}, {}
    e = {"none": O.EPI_NONE, "gelu": O.EPI_GELU, "gate_resid": O.EPI_GATE_RESID}[epi]
    if epi == "gate_resid":
        gate = O.normal_bf16((6, n), 11 + m, 4, std=0.5)
        resid = O.normal_bf16((m, n), 11 + m, 5)
        g = json.load(open(GOLD / "modrun.json"))
        rowmap = np.array((g["map"] * (m // 16 + 1))[:m], dtype=np.uint32)
        kw = dict(gate=gate, resid=resid, rowmap=rowmap)
        tkw = dict(gate=to_torch_bf16(gate), resid=to_torch_bf16(resid),
                   rowmap=torch.from_numpy(rowmap.view(np.int32)).cuda())
    ref = O.qlinear_lora(x, wq, sc, bi, ad, bias=b, epilogue=e, **kw)
    got = lin.forward(to_torch_bf16(x), e, **tkw)
    h3.context().check_device()
    # the reference rounds the base product, x A, (x A) B, the scaled delta and the sum to bf16;
    # the GPU accumulates base and delta in one fp32 accumulator and rounds once: results can
    # sit a couple of bf16 steps apart, so the bar is the north-star 2e-2 (cosine 0.9999)
    assert_close(f32(to_np_bf16(got)), f32(ref), rel=2e-2, cos=0.9999, what=f"lora m={m} r={ranks} {epi}")
    # the delta is not negligible in these cases: the result differs from the base linear
    base = O.qlinear(x, wq, sc, bi, bias=b, epilogue=e, **kw)
    assert np.abs(f32(ref) - f32(base)).max() > 1e-2


def test_zero_scale_lora_is_bit_identical_to_base():
    """An adapter of scale 0 packs to zeros: the K extension adds exact zeros."""
    from wuxianhuabu_b200 import h3
    k, n, m = 512, 768, 700
    lin, _ = _linear(21, n, k)
    x = to_torch_bf16(O.normal_bf16((m, k), 21, 3))
    base = lin.forward(x).clone()
    lin.set_lora(_refs(_adapters(21, k, n, [32], [0.0])))
    with_zero = lin.forward(x)
    h3.context().check_device()
    assert np.array_equal(to_np_bf16(base), to_np_bf16(with_zero))


def test_block_with_lora_vs_oracle():
    """A block with two adapters on each of its four linears. The qkv projection with its
    adapters is checked on its own first (GPU vs oracle at the linear tolerance); the oracle
    block is then fed that same projection, so that the projection's rounding differences
    (one fp32 accumulator here, the reference's bf16 intermediates in loraDelta) are not
    amplified by the softmax into the block comparison, which keeps the north-star bound."""
    import torch
    from tests.test_gpu_block import gpu_block_qkv
    from wuxianhuabu_b200 import h3
    hidden, heads, ffn, rot, eps = 256, 2, 512, 96, 1e-6
    S = 344
    w, mods, h, cos, sin, rowmap = make_block(9, hidden, heads, ffn, 0, S, rot)
    inner = heads * 128
    dims = {"qkv": (hidden, 3 * inner), "out": (inner, hidden), "fc1": (hidden, ffn), "fc2": (ffn, hidden)}
    w["lora"] = {name: _adapters(30 + i, k, n, [16, 8], [0.7, 1.3]) for i, (name, (k, n)) in enumerate(dims.items())}
    cfgd = dict(heads=heads, head_dim=128, eps=eps, rot=rot, mlp_kind=0)
    blk = gpu_block(w, hidden, heads, ffn, 0, rot, eps)
    for name, lin in zip(dims, blk.blocks[0].linears()):
        lin.set_lora(_refs(w["lora"][name]))
    blk = h3.H3DiTBlocks(blk.cfg, blk.blocks)  # re-read the packs and the LoRA rank
    md = [to_torch_bf16(m) for m in mods]
    rm = torch.from_numpy(rowmap.view(np.int32)).cuda()
    qkv_gpu = to_np_bf16(gpu_block_qkv(blk, 0, to_torch_bf16(h), md, rm))
    m1 = O.norm_modscale(h, w["norm1"], mods[0], mods[1], rowmap, eps)
    qkv_ref = O.qlinear_lora(m1, *w["qkv"][:3], w["lora"]["qkv"], bias=w["qkv"][3])
    assert_close(f32(qkv_gpu), f32(qkv_ref), rel=1e-2, cos=0.9999, what="qkv projection with adapters")
    ref, ref_at = O.block_forward(h, w, mods, rowmap, cos, sin, cfgd, qkv_override=qkv_gpu)
    ht = to_torch_bf16(h)
    slot = torch.empty((S, hidden), dtype=torch.bfloat16, device="cuda")
    blk.block_forward(0, ht, md, rm, to_torch_bf16(cos), to_torch_bf16(sin), None, pab_slot=slot, refresh=True)
    h3.context().check_device()
    assert_close(f32(to_np_bf16(slot)), f32(ref_at), rel=2e-2, cos=0.999, what="lora block at")
    assert_close(f32(to_np_bf16(ht)), f32(ref), rel=2e-2, cos=0.999, what="lora block h")
