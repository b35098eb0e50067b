"""GPU parity of the quantizer, dequantizer, quantized linear (all epilogues)
and the fused row kernels against the CPU oracle, through the C ABI."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    return torch


def _mf(torch, wq, sc, bi, k, bias=None):
    from wuxianhuabu_b200 import h3
    return h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                       None if bias is None else to_torch_bf16(bias))


@pytest.mark.parametrize("bits", [4, 6, 8])
def test_quantize_bit_exact(torch_mod, bits):
    from wuxianhuabu_b200 import h3
    torch = torch_mod
    w = O.normal_f32((96, 512), 21, bits, std=0.02)
    wq, sc, bi = O.quantize(w, bits=bits)
    m = h3.MfLinear.quantize(torch.from_numpy(w).cuda(), bits=bits)
    torch.cuda.synchronize()
    assert np.array_equal(m.w.cpu().numpy().view(np.uint32), wq)
    assert np.array_equal(to_np_bf16(m.scales), sc)
    assert np.array_equal(to_np_bf16(m.biases), bi)


@pytest.mark.parametrize("bits", [4, 6, 8])
def test_dequant_bit_exact(torch_mod, bits):
    w = O.normal_f32((64, 384), 22, bits, std=0.02)
    wq, sc, bi = O.quantize(w, bits=bits)
    ref = O.dequantize(wq, sc, bi, 384, bits=bits)
    got = to_np_bf16(_mf(torch_mod, wq, sc, bi, 384).dequantized_weight())
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("n,k", [(1000, 3072), (9216, 3072), (130, 704)])
def test_dequant_6bit_bundles_bit_exact(torch_mod, n, k):
    """The 6-bit expansion (one thread per 16-value bundle) at projection sizes: 9216 x 3072
    has more bundles than the grid's threads (the grid-stride loop), 704 = 11 groups per row."""
    wq, sc, bi = O.quantize(O.normal_f32((n, k), 23, 6, std=0.02))
    got = to_np_bf16(_mf(torch_mod, wq, sc, bi, k).dequantized_weight())
    assert np.array_equal(got, O.dequantize(wq, sc, bi, k))


def test_dequant_reference_4bit_fixture(torch_mod):
    d = np.load(GOLD / "dequant4.npz")
    m = _mf(torch_mod, d["words"], d["scales"], d["biases"], int(d["in_dim"]))
    assert np.array_equal(to_np_bf16(m.dequantized_weight()), d["expect"])


SHAPES = [(1, 128, 192), (77, 256, 384), (128, 512, 512), (300, 1024, 3072), (256, 3072, 256),
          # M <= 512 and N % 128 == 0 take the fused path (weights expanded in shared memory,
          # K split over a thread-block cluster): one row, a few rows, K blocks not divisible
          # by the split count, K = 12288 (the fc2 shape), two token tiles
          (256, 3072, 3072), (257, 1024, 1024), (512, 1024, 3072), (600, 512, 256),
          (1, 256, 128), (8, 3072, 9216), (100, 704, 640), (33, 12288, 3072), (256, 12288, 3072)]


@pytest.mark.parametrize("m,k,n", SHAPES)
@pytest.mark.parametrize("with_bias", [False, True])
def test_qlinear_none(torch_mod, m, k, n, with_bias):
    x = O.normal_bf16((m, k), 31, 1)
    w = O.normal_f32((n, k), 31, 2, std=0.02)
    wq, sc, bi = O.quantize(w)
    bias = O.normal_bf16((n,), 31, 3, std=0.1) if with_bias else None
    ref = O.qlinear(x, wq, sc, bi, bias=bias)
    got = to_np_bf16(_mf(torch_mod, wq, sc, bi, k, bias)(to_torch_bf16(x)))
    assert_close(f32(got), f32(ref), rel=1e-2, cos=0.9999, what=f"qlinear {m}x{k}x{n}")


@pytest.mark.parametrize("m,k,n", [(256, 3072, 3072), (33, 12288, 3072), (256, 12288, 3072)])
def test_qlinear_fused_is_deterministic(torch_mod, m, k, n):
    """The split-K sums of the small-M path are reduced in a fixed order, and no stage of its
    shared-memory rings is reused before every reader is done with it: bit-identical runs,
    also with many K blocks per CTA (the rings wrap many times)."""
    x = to_torch_bf16(O.normal_bf16((m, k), 35, 1))
    wq, sc, bi = O.quantize(O.normal_f32((n, k), 35, 2, std=0.02))
    lin = _mf(torch_mod, wq, sc, bi, k)
    a = lin(x).clone()
    for _ in range(3):
        assert torch_mod.equal(a, lin(x))


ROWS_SHAPES = [(1, 256, 256), (8, 3072, 9216), (100, 704, 768), (256, 3072, 3072), (257, 1024, 1024),
               (512, 1024, 3072), (33, 12288, 3072), (256, 12288, 3072)]


@pytest.mark.parametrize("rows,tpr", [(128, 2), (128, 4), (256, 2)])
@pytest.mark.parametrize("m,k,n", ROWS_SHAPES)
def test_qlinear_small_m_rows_per_cta(torch_mod, monkeypatch, rows, tpr, m, k, n):
    """Every CTA shape of the small-M kernel, forced by WX_QGEMM_ROWS / WX_QGEMM_TPR: 128 weight
    rows (one TMEM accumulator) expanded by 2 or 4 threads per row, or 256 (two accumulators
    sharing each activation tile, the split-K reduction run once per accumulator), with bias,
    against the oracle, and deterministic."""
    monkeypatch.setenv("WX_QGEMM_ROWS", str(rows))
    monkeypatch.setenv("WX_QGEMM_TPR", str(tpr))
    x = O.normal_bf16((m, k), 36, 1)
    wq, sc, bi = O.quantize(O.normal_f32((n, k), 36, 2, std=0.02))
    bias = O.normal_bf16((n,), 36, 3, std=0.1)
    lin = _mf(torch_mod, wq, sc, bi, k, bias)
    xt = to_torch_bf16(x)
    got = lin(xt).clone()
    assert_close(f32(to_np_bf16(got)), f32(O.qlinear(x, wq, sc, bi, bias=bias)), rel=1e-2, cos=0.9999,
                 what=f"qlinear {m}x{k}x{n}, {rows} rows per CTA")
    assert torch_mod.equal(got, lin(xt))


@pytest.mark.parametrize("m,k,n", [(256, 3072, 3072), (33, 12288, 3072), (512, 1024, 3072)])
def test_qlinear_small_m_threads_per_row_bit_identical(torch_mod, monkeypatch, m, k, n):
    """Two or four expansion threads per weight row write the same expanded tiles and keep the
    same split plan: bit-identical outputs."""
    x = to_torch_bf16(O.normal_bf16((m, k), 38, 1))
    wq, sc, bi = O.quantize(O.normal_f32((n, k), 38, 2, std=0.02))
    lin = _mf(torch_mod, wq, sc, bi, k)
    monkeypatch.setenv("WX_QGEMM_ROWS", "128")
    outs = []
    for tpr in ("2", "4"):
        monkeypatch.setenv("WX_QGEMM_TPR", tpr)
        outs.append(lin(x).clone())
    assert torch_mod.equal(outs[0], outs[1])


@pytest.mark.parametrize("rows,tpr", [(128, 2), (128, 4), (256, 2)])
def test_qlinear_small_m_epilogues_rows_per_cta(torch_mod, monkeypatch, rows, tpr):
    """GELU and gate + residual (with y_raw and a row map) through every CTA shape."""
    from wuxianhuabu_b200 import h3
    torch = torch_mod
    monkeypatch.setenv("WX_QGEMM_ROWS", str(rows))
    monkeypatch.setenv("WX_QGEMM_TPR", str(tpr))
    m, k, n = 200, 1024, 768
    x = O.normal_bf16((m, k), 37, 1)
    wq, sc, bi = O.quantize(O.normal_f32((n, k), 37, 2, std=0.05))
    bias = O.normal_bf16((n,), 37, 3, std=0.1)
    lin = _mf(torch, wq, sc, bi, k, bias)
    got = to_np_bf16(lin(to_torch_bf16(x), epilogue=h3.EPI_GELU))
    assert_close(f32(got), f32(O.qlinear(x, wq, sc, bi, bias=bias, epilogue=O.EPI_GELU)), rel=1e-2, cos=0.9999,
                 what=f"gelu, {rows} rows per CTA")
    gate, resid = O.normal_bf16((3, n), 37, 4), O.normal_bf16((m, n), 37, 5)
    rowmap = (np.arange(m) % 3).astype(np.uint32)
    raw = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    got = to_np_bf16(lin(to_torch_bf16(x), epilogue=h3.EPI_GATE_RESID, gate=to_torch_bf16(gate),
                         resid=to_torch_bf16(resid), rowmap=torch.from_numpy(rowmap.view(np.int32)).cuda(),
                         y_raw=raw))
    want, want_raw = O.qlinear(x, wq, sc, bi, bias=bias, epilogue=O.EPI_GATE_RESID, gate=gate, resid=resid,
                               rowmap=rowmap, want_raw=True)
    assert_close(f32(got), f32(want), rel=1e-2, cos=0.9999, what=f"gate+resid, {rows} rows per CTA")
    assert_close(f32(to_np_bf16(raw)), f32(want_raw), rel=1e-2, cos=0.9999, what=f"raw, {rows} rows per CTA")


def test_qlinear_gelu(torch_mod):
    m, k, n = 200, 512, 768
    x = O.normal_bf16((m, k), 32, 1)
    wq, sc, bi = O.quantize(O.normal_f32((n, k), 32, 2, std=0.05))
    bias = O.normal_bf16((n,), 32, 3, std=0.1)
    ref = O.qlinear(x, wq, sc, bi, bias=bias, epilogue=O.EPI_GELU)
    from wuxianhuabu_b200 import h3
    got = to_np_bf16(_mf(torch_mod, wq, sc, bi, k, bias)(to_torch_bf16(x), epilogue=h3.EPI_GELU))
    assert_close(f32(got), f32(ref), rel=1e-2, cos=0.9999, what="gelu")


def test_qlinear_gate_resid(torch_mod):
    torch = torch_mod
    from wuxianhuabu_b200 import h3
    g = json.load(open(GOLD / "modrun.json"))
    m, k, n = 130, 256, 512
    rowmap = np.array((g["map"] * 20)[:m], dtype=np.uint32)
    x = O.normal_bf16((m, k), 33, 1)
    wq, sc, bi = O.quantize(O.normal_f32((n, k), 33, 2, std=0.05))
    bias = O.normal_bf16((n,), 33, 3, std=0.1)
    gate = O.normal_bf16((6, n), 33, 4)
    resid = O.normal_bf16((m, n), 33, 5)
    ref, ref_raw = O.qlinear(x, wq, sc, bi, bias=bias, epilogue=O.EPI_GATE_RESID, gate=gate, resid=resid,
                             rowmap=rowmap, want_raw=True)
    raw = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    got = _mf(torch, wq, sc, bi, k, bias)(to_torch_bf16(x), epilogue=h3.EPI_GATE_RESID, gate=to_torch_bf16(gate),
                                          resid=to_torch_bf16(resid),
                                          rowmap=torch.from_numpy(rowmap.view(np.int32)).cuda(), y_raw=raw)
    assert_close(f32(to_np_bf16(raw)), f32(ref_raw), rel=1e-2, cos=0.9999, what="gate_resid raw")
    assert_close(f32(to_np_bf16(got)), f32(ref), rel=1e-2, cos=0.9999, what="gate_resid")


def test_qlinear_swiglu(torch_mod):
    from wuxianhuabu_b200 import h3
    m, k, F = 90, 256, 256
    x = O.normal_bf16((m, k), 34, 1)
    wq, sc, bi = O.quantize(O.normal_f32((2 * F, k), 34, 2, std=0.05))
    ref = O.qlinear(x, wq, sc, bi, epilogue=O.EPI_SWIGLU)
    got = to_np_bf16(_mf(torch_mod, wq, sc, bi, k)(to_torch_bf16(x), epilogue=h3.EPI_SWIGLU))
    assert got.shape == (m, F)
    assert_close(f32(got), f32(ref), rel=1e-2, cos=0.9999, what="swiglu")


@pytest.mark.parametrize("epi", ["none", "gelu", "gate_resid", "lora"])
def test_qlinear_many_tiles_vs_oracle(torch_mod, epi):
    """A shape with several waves of 128x256 tiles of the persistent kernel and a ragged
    last M tile, each epilogue (and a LoRA extension) against the oracle."""
    torch = torch_mod
    from wuxianhuabu_b200 import h3
    m, k, n = 4000, 1024, 12288
    x = O.normal_bf16((m, k), 35, 1)
    wq, sc, bi = O.quantize(O.normal_f32((n, k), 35, 2, std=0.03))
    bias = O.normal_bf16((n,), 35, 3, std=0.1)
    lin = _mf(torch, wq, sc, bi, k, bias)
    kw, tkw = {}, {}
    if epi == "gate_resid":
        g = json.load(open(GOLD / "modrun.json"))
        rowmap = np.array((g["map"] * (m // 16 + 1))[:m], dtype=np.uint32)
        gate = O.normal_bf16((6, n), 35, 4)
        resid = O.normal_bf16((m, n), 35, 5)
        kw = dict(epilogue=O.EPI_GATE_RESID, gate=gate, resid=resid, rowmap=rowmap)
        tkw = dict(epilogue=h3.EPI_GATE_RESID, gate=to_torch_bf16(gate), resid=to_torch_bf16(resid),
                   rowmap=torch.from_numpy(rowmap.view(np.int32)).cuda())
    elif epi == "gelu":
        kw, tkw = dict(epilogue=O.EPI_GELU), dict(epilogue=h3.EPI_GELU)
    if epi == "lora":
        ad = [(O.normal_bf16((k, 32), 35, 6, std=0.05), O.normal_bf16((32, n), 35, 7, std=0.05), 0.7)]
        lin.set_lora([h3.LoraRef(to_torch_bf16(a), to_torch_bf16(b), sc_) for a, b, sc_ in ad])
        ref = O.qlinear_lora(x, wq, sc, bi, ad, bias=bias)
        rel = 2e-2  # one fp32 accumulator against the reference's bf16 intermediates
    else:
        ref = O.qlinear(x, wq, sc, bi, bias=bias, **kw)
        rel = 1e-2
    got = to_np_bf16(lin(to_torch_bf16(x), **tkw))
    h3.context().check_device()
    assert_close(f32(got), f32(ref), rel=rel, cos=0.9999, what=f"many tiles {epi}")


@pytest.mark.parametrize("m,k,n", [(4096, 3072, 3072), (1000, 12288, 3072), (2000, 3072, 12288)])
def test_qlinear_large_vs_torch_fp32(torch_mod, m, k, n):
    """Large shapes against a plain PyTorch fp32 matmul of the GPU-dequantized weight."""
    torch = torch_mod
    from wuxianhuabu_b200 import h3
    gen = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn((m, k), device="cuda", generator=gen).to(torch.bfloat16)
    lin = h3.MfLinear.quantize(torch.randn((n, k), device="cuda", generator=gen) * 0.02)
    y = lin(x).float()
    ref = x.float() @ lin.dequantized_weight().float().t()
    err = ((y - ref).abs().max() / ref.abs().max()).item()
    cos = torch.nn.functional.cosine_similarity(y.flatten(), ref.flatten(), dim=0).item()
    assert err < 1e-2 and cos > 0.9999, (err, cos)


# (128, *, *) with rot/2 % 4 == 0 takes the 8-heads-per-warp kernel (H=11: a ragged head group);
# rot 100 and head_dim 64 take the warp-per-row kernel
@pytest.mark.parametrize("hd,rot,eps,H", [(128, 96, 1e-5, 3), (64, 64, 1e-6, 3), (128, 128, 1e-6, 3),
                                          (128, 128, 1e-6, 11), (128, 100, 1e-6, 3), (128, 0, 1e-6, 3)])
def test_qk_norm_rope(torch_mod, hd, rot, eps, H):
    from wuxianhuabu_b200 import h3
    S = 333
    x = O.normal_bf16((S, H, hd), 41, hd)
    w = O.normal_bf16((hd,), 41, 2, mean=1.0, std=0.1)
    cos = O.normal_bf16((S, rot // 2), 41, 3)
    sin = O.normal_bf16((S, rot // 2), 41, 4)
    ref = O.qk_norm_rope(x, w, cos, sin, rot, eps)
    got = h3.H3FusedKernels.fused_rmsnorm_rope(to_torch_bf16(x), to_torch_bf16(w), to_torch_bf16(cos),
                                               to_torch_bf16(sin), rot, eps)
    g = f32(to_np_bf16(got))
    r = f32(ref)
    assert np.abs(g - r).max() < 0.25  # the reference self-test bound (fused:404-407)
    assert_close(g, r, rel=1e-2, cos=0.99999, what="qk_norm_rope")
    assert (to_np_bf16(got) == ref).mean() > 0.95


def test_qk_norm_rope_packed_qkv_in_place(torch_mod):
    torch = torch_mod
    import ctypes as C
    from wuxianhuabu_b200 import h3
    S, H, hd, rot, eps = 200, 2, 128, 96, 1e-6
    inner = H * hd
    qkv = O.normal_bf16((S, 3 * inner), 42, 1)
    qw = O.normal_bf16((hd,), 42, 2, mean=1.0, std=0.1)
    kw = O.normal_bf16((hd,), 42, 3, mean=1.0, std=0.1)
    cos = O.normal_bf16((S, rot // 2), 42, 4)
    sin = O.normal_bf16((S, rot // 2), 42, 5)
    rq = O.qk_norm_rope(np.ascontiguousarray(qkv[:, :inner].reshape(S, H, hd)), qw, cos, sin, rot, eps)
    rk = O.qk_norm_rope(np.ascontiguousarray(qkv[:, inner:2 * inner].reshape(S, H, hd)), kw, cos, sin, rot, eps)
    t = to_torch_bf16(qkv)
    keep = [to_torch_bf16(a) for a in (qw, kw, cos, sin)]  # alive until the kernel has run
    ctx = h3.context()
    ctx.call("wx_qk_norm_rope_qkv", t.data_ptr(), S, H, hd, *[a.data_ptr() for a in keep], rot, float(eps))
    torch.cuda.synchronize()
    out = to_np_bf16(t)
    assert_close(f32(out[:, :inner]), f32(rq.reshape(S, inner)), rel=1e-2, cos=0.99999, what="q")
    assert_close(f32(out[:, inner:2 * inner]), f32(rk.reshape(S, inner)), rel=1e-2, cos=0.99999, what="k")
    assert np.array_equal(out[:, 2 * inner:], qkv[:, 2 * inner:])  # v untouched


@pytest.mark.parametrize("hidden", [64, 3072])
def test_norm_modscale_and_mod_gate(torch_mod, hidden):
    torch = torch_mod
    from wuxianhuabu_b200 import h3
    g = json.load(open(GOLD / "modrun.json"))
    S = 16 if hidden == 64 else 1000
    rowmap = np.array((g["map"] * 100)[:S], dtype=np.uint32)
    rm = torch.from_numpy(rowmap.view(np.int32)).cuda()
    x = O.normal_bf16((S, hidden), 43, 1)
    w = O.normal_bf16((hidden,), 43, 2, mean=1.0, std=0.1)
    sh = O.normal_bf16((6, hidden), 43, 3)
    sc = O.normal_bf16((6, hidden), 43, 4)
    ref = O.norm_modscale(x, w, sh, sc, rowmap, 1e-6)
    got = h3.H3FusedKernels.fused_norm_modscale(to_torch_bf16(x), to_torch_bf16(w), to_torch_bf16(sh),
                                                to_torch_bf16(sc), rm, 1e-6)
    assert np.abs(f32(to_np_bf16(got)) - f32(ref)).max() < 0.25
    assert_close(f32(to_np_bf16(got)), f32(ref), rel=1e-2, cos=0.99999, what="norm_modscale")
    ref_row = O.norm_modscale(x, w, sh[:1], sc[:1], None, 1e-6)
    got_row = h3.H3FusedKernels.fused_norm_modscale_row(to_torch_bf16(x), to_torch_bf16(w), to_torch_bf16(sh[:1]),
                                                        to_torch_bf16(sc[:1]), 1e-6)
    assert_close(f32(to_np_bf16(got_row)), f32(ref_row), rel=1e-2, cos=0.99999, what="row variant")
    other = O.normal_bf16((S, hidden), 43, 5)
    gate = O.normal_bf16((6, hidden), 43, 6)
    ref2 = O.mod_gate(x, other, gate, rowmap)
    got2 = h3.H3FusedKernels.fused_mod_gate(to_torch_bf16(x), to_torch_bf16(gate), to_torch_bf16(other), rm)
    assert_close(f32(to_np_bf16(got2)), f32(ref2), rel=1e-2, cos=0.99999, what="mod_gate")


def test_invalid_arguments_return_errors(torch_mod):
    torch = torch_mod
    from wuxianhuabu_b200 import h3, _lib
    x = torch.zeros((4, 100), dtype=torch.bfloat16, device="cuda")
    lin = h3.MfLinear(torch.zeros((8, 100 * 6 // 32 + 1), dtype=torch.int32, device="cuda"),
                      torch.zeros((8, 1), dtype=torch.bfloat16, device="cuda"),
                      torch.zeros((8, 1), dtype=torch.bfloat16, device="cuda"), 100)
    with pytest.raises(_lib.WxError):
        lin(x)  # K not a multiple of the group / word geometry
    q = torch.zeros((10, 2, 96), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.WxError):
        h3.H3SolAttn.forward(q, q, q, 0, 0.125, None)  # the flash kernels take head_dim 128 or 64 only
    h3.context().check_device()
