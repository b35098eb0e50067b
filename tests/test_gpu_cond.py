"""Conditioning around the DiT blocks against the CPU oracle: the timestep embedder
(H3TimeEmbedder, H3Transformer.swift:255-302), the AdaLN tables (precomputeAdaln
:957-988, H3AdalnW :353-404, the LUT variant :319-350), RMSNorm (H3Common.swift:502-508)
and the text refiner (refineText :993-1016, H3RefinerBlockW :676-700)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16

pytestmark = pytest.mark.gpu


def _cuda_f32(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def _qlinear(seed, n, k, bias=True):
    import torch
    from wuxianhuabu_b200 import h3
    wq, sc, bi = O.quantize(O.normal_f32((n, k), seed, 1, std=0.02))
    b = O.normal_bf16((n,), seed, 2, std=0.02) if bias else None
    lin = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                      to_torch_bf16(b) if bias else None)
    return lin, (wq, sc, bi, b)


def _bf16_ulps(a, b):
    """largest distance in bf16 steps between two bf16 arrays of the same sign pattern"""
    ia = a.astype(np.int32)
    ib = b.astype(np.int32)
    ia = np.where(ia & 0x8000, -(ia & 0x7FFF), ia)
    ib = np.where(ib & 0x8000, -(ib & 0x7FFF), ib)
    return int(np.abs(ia - ib).max())


@pytest.mark.parametrize("dim", [384, 2688])
def test_time_embed_vs_oracle(dim):
    from wuxianhuabu_b200 import h3
    ts = [0.0, 0.5, 27.03, 972.97, 999.0]
    w_in = O.normal_f32((256, dim), 5, 1, std=0.05)
    b_in = O.normal_f32((dim,), 5, 2, std=0.05)
    w_out = O.normal_f32((dim, dim), 5, 3, std=0.02)
    b_out = O.normal_f32((dim,), 5, 4, std=0.02)
    emb = h3.H3TimeEmbedder(256, dim, _cuda_f32(w_in), _cuda_f32(b_in), _cuda_f32(w_out), _cuda_f32(b_out))
    got = emb(ts).cpu().numpy()
    h3.context().check_device()
    ref = O.time_embed(ts, w_in, b_in, w_out, b_out)
    # fp32 throughout; only the summation order of the two dense products differs
    assert_close(got, ref, rel=1e-4, cos=0.9999999, what=f"time_embed dim={dim}")


def test_silu_bf16_within_one_step():
    import torch
    from wuxianhuabu_b200 import h3
    x = O.normal_bf16((4096,), 6, 1, std=4.0)
    y = torch.empty(4096, dtype=torch.bfloat16, device="cuda")
    h3.context().call("wx_silu_bf16", to_torch_bf16(x).data_ptr(), 4096, y.data_ptr())
    h3.context().check_device()
    ref = O.silu_bf16(x)
    got = to_np_bf16(y)
    # expf on the GPU and in libm may differ in the last fp32 bit; after the bf16
    # rounding of sigmoid and of the product that is at most one bf16 step
    assert _bf16_ulps(got, ref) <= 1
    assert (got == ref).mean() > 0.99


@pytest.mark.parametrize("S,hidden", [(5, 256), (300, 3072), (64, 5376)])
def test_rms_norm_vs_oracle(S, hidden):
    from wuxianhuabu_b200 import h3
    x = O.normal_bf16((S, hidden), 7, 1, std=2.0)
    w = O.normal_bf16((hidden,), 7, 2, mean=1.0, std=0.1)
    got = to_np_bf16(h3.rms_norm(to_torch_bf16(x), to_torch_bf16(w), 1e-5))
    h3.context().check_device()
    ref = O.rms_norm(x, w, 1e-5)
    assert _bf16_ulps(got, ref) <= 1
    assert_close(f32(got), f32(ref), rel=1e-2, cos=0.99999, what="rms_norm")


@pytest.mark.parametrize("m", [1, 3])
@pytest.mark.parametrize("expand,modalities", [(6, 3), (2, 1)])
@pytest.mark.parametrize("lora", [False, True])
def test_adaln_tables_quantized(m, expand, modalities, lora):
    from wuxianhuabu_b200 import h3
    hidden, k = 256, 384
    n = expand * modalities * hidden
    lin, (wq, sc, bi, b) = _qlinear(31 + m, n, k)
    ad = None
    if lora:
        ad = [(O.normal_bf16((k, 16), 31, 100, std=0.05), O.normal_bf16((16, n), 31, 101, std=0.05), 0.9)]
        lin.set_lora([h3.LoraRef(to_torch_bf16(a), to_torch_bf16(bb), s) for a, bb, s in ad])
    t_emb = O.normal_bf16((m, k), 31 + m, 3, std=1.5)
    tabs = h3.H3AdalnW(lin, expand, modalities)(to_torch_bf16(t_emb), apply_silu=True)
    h3.context().check_device()
    refs = O.adaln_tables(t_emb, expand, modalities, True, q=(wq, sc, bi, b), lora=ad)
    assert len(tabs) == expand
    for e, (got, ref) in enumerate(zip(tabs, refs)):
        assert tuple(got.shape) == (m * modalities, hidden)
        assert_close(f32(to_np_bf16(got)), f32(ref), rel=2e-2, cos=0.9999, what=f"adaln table {e}")


def test_adaln_lut_dense_path():
    """Pruned / fused checkpoints: LUT coefficients (no SiLU) through a dense folded adaln_proj."""
    import torch
    from wuxianhuabu_b200 import h3
    rank, hidden, m = 8, 128, 3
    n = 6 * 3 * hidden
    table = O.normal_f32((1025, rank), 41, 1)
    lut = h3.H3AdalnLUT(None, None, _cuda_f32(table))
    ts = [0.0, 0.97297, 0.5004882812]
    coeffs = lut.coeffs(ts)
    h3.context().check_device()
    assert np.array_equal(to_np_bf16(coeffs), O.lut_coeffs(ts, table))
    w = O.normal_bf16((rank, n), 41, 2, std=0.1)
    bias = O.normal_bf16((n,), 41, 3, std=0.1)
    dense = h3.DenseLinear(to_torch_bf16(w), to_torch_bf16(bias))
    tabs = h3.H3AdalnW(dense, 6, 3)(coeffs, apply_silu=False)
    h3.context().check_device()
    refs = O.adaln_tables(O.lut_coeffs(ts, table), 6, 3, False, dense=(w, bias))
    for got, ref in zip(tabs, refs):
        g = to_np_bf16(got)
        assert _bf16_ulps(g, ref) <= 1
        assert (g == ref).mean() > 0.99
    assert tabs[0].shape == torch.Size([m * 3, hidden])


def test_precompute_adaln_chain():
    """precomputeAdaln with the time embedder: fp32 embedding -> bf16 -> SiLU -> each
    block's adaln_proj -> six tables; an absent block gets zero tables; final -> two."""
    from wuxianhuabu_b200 import h3
    hidden, ted = 256, 384
    ts = [1000.0, 972.97]
    w_in, b_in = O.normal_f32((256, ted), 8, 1, std=0.05), O.normal_f32((ted,), 8, 2, std=0.05)
    w_out, b_out = O.normal_f32((ted, ted), 8, 3, std=0.02), O.normal_f32((ted,), 8, 4, std=0.02)
    emb = h3.H3TimeEmbedder(256, ted, _cuda_f32(w_in), _cuda_f32(b_in), _cuda_f32(w_out), _cuda_f32(b_out))
    lin0, q0 = _qlinear(51, 18 * hidden, ted)
    linf, qf = _qlinear(52, 2 * hidden, ted)
    tables = h3.precompute_adaln(ts, [h3.H3AdalnW(lin0, 6, 3), None], h3.H3AdalnW(linf, 2, 1), hidden,
                                 embedder=emb)
    h3.context().check_device()
    temb = O.f32_to_bf16(O.time_embed(ts, w_in, b_in, w_out, b_out))
    ref0 = O.adaln_tables(temb, 6, 3, True, q=q0)
    reff = O.adaln_tables(temb, 2, 1, True, q=qf)
    for got, ref in zip(tables.blocks[0], ref0):
        assert_close(f32(to_np_bf16(got)), f32(ref), rel=2e-2, cos=0.9999, what="block table")
    assert all(not to_np_bf16(t).any() for t in tables.blocks[1])
    for got, ref in zip(tables.final, reff):
        assert_close(f32(to_np_bf16(got)), f32(ref), rel=2e-2, cos=0.9999, what="final table")


def _refiner_weights(seed, hidden, heads, ffn, mlp_kind):
    from tests.test_gpu_block import make_block
    w, _, _, _, _, _ = make_block(seed, hidden, heads, ffn, mlp_kind, 16)
    return w


def _gpu_refiner_block(w, hidden, heads, ffn):
    import torch
    from wuxianhuabu_b200 import h3

    def lin(t, k):
        wq, sc, bi, b = t
        return h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                           to_torch_bf16(b))
    inner = heads * 128
    return h3.H3BlockWeights(lin(w["qkv"], hidden), lin(w["out"], inner), lin(w["fc1"], hidden),
                             lin(w["fc2"], ffn), to_torch_bf16(w["q_norm"]), to_torch_bf16(w["k_norm"]),
                             to_torch_bf16(w["norm1"]), to_torch_bf16(w["norm2"]))


@pytest.mark.parametrize("L", [77, 300])
@pytest.mark.parametrize("mlp_kind", [0, 1])
def test_refiner_block_vs_oracle(L, mlp_kind):
    from wuxianhuabu_b200 import h3
    hidden, heads, ffn, eps = 256, 2, 512, 1e-5
    w = _refiner_weights(61 + mlp_kind, hidden, heads, ffn, mlp_kind)
    h = O.normal_bf16((L, hidden), 61, 9)
    cfg = h3.H3DiTConfig(hidden=hidden, heads=heads, head_dim=128, ffn=ffn, mlp_kind=mlp_kind, rot=0, eps=eps)
    ref = h3.H3TextRefiner(cfg, None, [_gpu_refiner_block(w, hidden, heads, ffn)], None)
    ht = to_torch_bf16(h)
    ref.block_forward(0, ht)
    h3.context().check_device()
    want = O.refiner_block_forward(h, w, dict(heads=heads, head_dim=128, eps=eps, mlp_kind=mlp_kind))
    assert_close(f32(to_np_bf16(ht)), f32(want), rel=2e-2, cos=0.999, what=f"refiner block L={L}")


def test_refine_text_vs_oracle():
    from wuxianhuabu_b200 import h3
    hidden, heads, ffn, eps, text_dim, L = 256, 2, 512, 1e-5, 384, 150
    cfg = h3.H3DiTConfig(hidden=hidden, heads=heads, head_dim=128, ffn=ffn, mlp_kind=1, rot=0, eps=eps)
    ws = [_refiner_weights(70 + i, hidden, heads, ffn, 1) for i in range(2)]
    cp, cpq = _qlinear(72, hidden, text_dim)
    fnorm = O.normal_bf16((hidden,), 72, 5, mean=1.0, std=0.05)
    text = O.normal_bf16((L, text_dim), 72, 6)
    refiner = h3.H3TextRefiner(cfg, cp, [_gpu_refiner_block(w, hidden, heads, ffn) for w in ws],
                               to_torch_bf16(fnorm))
    got = refiner(to_torch_bf16(text))
    h3.context().check_device()
    want = O.refine_text(text, dict(hidden=hidden, heads=heads, head_dim=128, eps=eps, mlp_kind=1), cpq, ws, fnorm)
    assert_close(f32(to_np_bf16(got)), f32(want), rel=2e-2, cos=0.999, what="refine_text")
    # states already `hidden` wide come back unchanged (refineText :996)
    same = O.normal_bf16((L, hidden), 72, 7)
    assert np.array_equal(to_np_bf16(refiner(to_torch_bf16(same))), same)
