"""Checkpoint reader (H3Weights over wx_st_*, H3Common.swift:180-261) on CPU: header
parsing, both naming variants of the quantized triple (getQuantized :243-258), the
MfLinear.load geometry (:311-338), and rejection of malformed files."""
import ctypes as C
import struct

import numpy as np
import pytest

from oracle import oracle as O
from tests.st_writer import write_safetensors
from wuxianhuabu_b200 import _lib


def _open(path):
    lib = _lib.load()
    h = C.c_void_p()
    st = lib.wx_st_open(str(path).encode(), C.byref(h))
    return lib, h, st


def _find(lib, h, name):
    inf = _lib.StInfo()
    return lib.wx_st_find(h, name.encode(), C.byref(inf)), inf


def test_header_and_bytes(tmp_path):
    rng = np.random.default_rng(0)
    t = {"a.weight": rng.integers(0, 2**32, (6, 9), dtype=np.uint32),
         "b": rng.standard_normal((3, 4, 5)).astype(np.float32),
         "c.norm": rng.integers(0, 2**16, (17,), dtype=np.uint16),
         "scalar": np.array(3.5, dtype=np.float32)}
    p = tmp_path / "x.safetensors"
    write_safetensors(p, t, metadata={"format": "mlx", "note": "quote \" and \\\\ escapes"})
    lib, h, st = _open(p)
    assert st == 0, lib.wx_st_last_error()
    try:
        assert lib.wx_st_count(h) == len(t)
        assert {lib.wx_st_name(h, i).decode() for i in range(len(t))} == set(t)
        for name, a in t.items():
            st, inf = _find(lib, h, name)
            assert st == 0
            assert [inf.shape[i] for i in range(inf.ndim)] == list(a.shape)
            assert inf.nbytes == a.nbytes
            got = np.frombuffer(C.string_at(inf.host, inf.nbytes), dtype=a.dtype).reshape(a.shape)
            assert np.array_equal(got, a)
        assert _find(lib, h, "missing")[0] == _lib.WX_ERR_INVALID
    finally:
        lib.wx_st_close(h)


@pytest.mark.parametrize("variant", ["mlx", "hf"])
@pytest.mark.parametrize("bits,group,k", [(6, 64, 3072), (4, 64, 512), (8, 128, 256)])
def test_quantized_triple_lookup(tmp_path, variant, bits, group, k):
    n = 40
    wq = np.zeros((n, k * bits // 32), dtype=np.uint32)
    sc = np.zeros((n, k // group), dtype=np.uint16)
    t = {"blk.fc.weight": wq, "blk.fc.bias": np.zeros((n,), dtype=np.uint16)}
    if variant == "mlx":
        t.update({"blk.fc.scales": sc, "blk.fc.biases": sc})
    else:
        t.update({"blk.fc.weight.scales": sc, "blk.fc.weight.biases": sc})
    p = tmp_path / "q.safetensors"
    write_safetensors(p, t)
    lib, h, st = _open(p)
    assert st == 0
    try:
        infos = [_lib.StInfo() for _ in range(4)]
        b, g = C.c_int32(), C.c_int32()
        st = lib.wx_st_find_qlinear(h, b"blk.fc", k, *[C.byref(i) for i in infos], C.byref(b), C.byref(g))
        assert st == 0, lib.wx_st_last_error()
        assert (b.value, g.value) == (bits, group)
        assert infos[0].nbytes == wq.nbytes and infos[1].nbytes == sc.nbytes and infos[3].nbytes == 2 * n
        # wrong in_features -> inconsistent geometry; absent prefix -> missing weight
        assert lib.wx_st_find_qlinear(h, b"blk.fc", k + 1, *[C.byref(i) for i in infos], C.byref(b),
                                      C.byref(g)) == _lib.WX_ERR_INVALID
        assert lib.wx_st_find_qlinear(h, b"blk.nope", k, *[C.byref(i) for i in infos], C.byref(b),
                                      C.byref(g)) == _lib.WX_ERR_INVALID
        assert b"missing weight" in lib.wx_st_last_error()
    finally:
        lib.wx_st_close(h)


def test_malformed_files_are_rejected(tmp_path):
    good = tmp_path / "g.safetensors"
    write_safetensors(good, {"x": np.arange(8, dtype=np.float32)})
    raw = good.read_bytes()
    cases = {
        "short": b"\x01\x00",
        "huge_header": struct.pack("<Q", 1 << 40) + raw[8:],
        "truncated_data": raw[:-4],
        "bad_json": struct.pack("<Q", 8) + b"{\"x\":[}" + b" ",
        "bad_offsets": None,
    }
    h = raw[8:8 + struct.unpack("<Q", raw[:8])[0]].decode().replace("[0, 32]", "[0, 64]")
    hb = h.encode()
    cases["bad_offsets"] = struct.pack("<Q", len(hb)) + hb + raw[8 + len(hb):]
    lib = _lib.load()
    for name, data in cases.items():
        p = tmp_path / f"{name}.safetensors"
        p.write_bytes(data)
        hd = C.c_void_p()
        assert lib.wx_st_open(str(p).encode(), C.byref(hd)) == _lib.WX_ERR_INVALID, name
        assert not hd.value
    assert lib.wx_st_open(str(tmp_path / "absent").encode(), C.byref(C.c_void_p())) == _lib.WX_ERR_INVALID


@pytest.mark.gpu
def test_load_block_runs_like_in_memory_weights(tmp_path):
    """A block written to safetensors (HF naming for qkv, mlx naming for the rest) and loaded
    through H3Weights gives the bit-identical linear outputs of the in-memory weights."""
    import torch
    from tests._util import to_np_bf16, to_torch_bf16
    from wuxianhuabu_b200 import h3
    hidden, heads, ffn = 256, 2, 512
    inner = heads * 128
    t = {}
    ref = {}
    for i, (name, n, k) in enumerate([("attn.qkv_proj", 3 * inner, hidden), ("attn.out_proj", hidden, inner),
                                      ("mlp.fc1", ffn, hidden), ("mlp.fc2", hidden, ffn)]):
        wq, sc, bi = O.quantize(O.normal_f32((n, k), 5, i, std=0.02))
        bias = O.normal_bf16((n,), 5, 10 + i, std=0.02)
        p = f"blocks.0.{name}"
        t[p + ".weight"] = wq
        if i == 0:
            t[p + ".weight.scales"], t[p + ".weight.biases"] = sc, bi
        else:
            t[p + ".scales"], t[p + ".biases"] = sc, bi
        t[p + ".bias"] = bias
        ref[name] = (wq, sc, bi, bias, k)
    for nm in ("attn.q_norm", "attn.k_norm"):
        t[f"blocks.0.{nm}.weight"] = O.normal_bf16((128,), 5, 20, mean=1.0, std=0.02)
    for nm in ("norm1", "norm2"):
        t[f"blocks.0.{nm}.weight"] = O.normal_bf16((hidden,), 5, 21, mean=1.0, std=0.02)
    path = tmp_path / "blk.safetensors"
    write_safetensors(path, t, metadata={"format": "mlx"})
    cfg = h3.H3DiTConfig(hidden=hidden, heads=heads, head_dim=128, ffn=ffn, layers=1)
    w = h3.H3Weights(path)
    bw = h3.load_block(w, 0, cfg)
    assert np.array_equal(to_np_bf16(bw.norm1), t["blocks.0.norm1.weight"])
    for lin, name in zip(bw.linears(), ["attn.qkv_proj", "attn.out_proj", "mlp.fc1", "mlp.fc2"]):
        wq, sc, bi, bias, k = ref[name]
        assert (lin.bits, lin.group_size, lin.in_dim) == (6, 64, k)
        mem = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                          to_torch_bf16(bias))
        x = to_torch_bf16(O.normal_bf16((300, k), 6, 1))
        assert torch.equal(lin(x), mem(x)), name
    w.close()


@pytest.mark.gpu
def test_load_conditioning_weights(tmp_path):
    """time_embedder, a quantized and a dense (folded) adaln_proj, condition_proj, one
    token-refiner block and its final norm, read through the H3DiT.load names
    (H3Transformer.swift:762-807) and run against the oracle."""
    from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16
    from wuxianhuabu_b200 import h3
    hidden, heads, ffn, ted, text_dim, rank = 256, 2, 512, 384, 384, 8
    inner = heads * 128
    t, qref = {}, {}
    t["time_embedder.proj_in.weight"] = O.normal_f32((256, ted), 9, 1, std=0.05)
    t["time_embedder.proj_in.bias"] = O.normal_f32((ted,), 9, 2, std=0.05)
    t["time_embedder.proj_out.weight"] = O.normal_f32((ted, ted), 9, 3, std=0.02)
    t["time_embedder.proj_out.bias"] = O.normal_f32((ted,), 9, 4, std=0.02)
    lins = [("blocks.0.adaln_proj.linear", 18 * hidden, ted), ("condition_proj", hidden, text_dim),
            ("token_refiner.blocks.0.attn.qkv_proj", 3 * inner, hidden),
            ("token_refiner.blocks.0.attn.out_proj", hidden, inner),
            ("token_refiner.blocks.0.mlp.fc1", 2 * ffn, hidden), ("token_refiner.blocks.0.mlp.fc2", hidden, ffn)]
    for i, (p, n, k) in enumerate(lins):
        wq, sc, bi = O.quantize(O.normal_f32((n, k), 9, 10 + i, std=0.02))
        bias = O.normal_bf16((n,), 9, 20 + i, std=0.02)
        t[p + ".weight"], t[p + ".scales"], t[p + ".biases"], t[p + ".bias"] = wq, sc, bi, bias
        qref[p] = (wq, sc, bi, bias)
    dense_w = O.normal_bf16((18 * hidden, rank), 9, 30, std=0.1)  # [out, in] as stored
    t["blocks.1.adaln_proj.linear.weight"] = dense_w
    for nm in ("attn.q_norm", "attn.k_norm"):
        t[f"token_refiner.blocks.0.{nm}.weight"] = O.normal_bf16((128,), 9, 31, mean=1.0, std=0.02)
    for nm in ("norm1", "norm2"):
        t[f"token_refiner.blocks.0.{nm}.weight"] = O.normal_bf16((hidden,), 9, 32, mean=1.0, std=0.02)
    t["token_refiner.final_norm.weight"] = O.normal_bf16((hidden,), 9, 33, mean=1.0, std=0.02)
    path = tmp_path / "cond.safetensors"
    write_safetensors(path, t, metadata={"format": "mlx"})
    w = h3.H3Weights(path)
    cfg = h3.H3DiTConfig(hidden=hidden, heads=heads, head_dim=128, ffn=ffn, mlp_kind=h3.MLP_SWIGLU, rot=0,
                         eps=1e-5, layers=2)
    ts = [1000.0, 500.0]
    emb = h3.load_time_embedder(w, 256, ted)
    temb = O.f32_to_bf16(O.time_embed(ts, *[t["time_embedder." + k] for k in
                                            ("proj_in.weight", "proj_in.bias", "proj_out.weight", "proj_out.bias")]))
    ad_q = h3.load_adaln(w, "blocks.0.adaln_proj", ted, 6, 3)
    assert isinstance(ad_q.linear, h3.MfLinear)
    tables = h3.precompute_adaln(ts, [ad_q], None, hidden, embedder=emb)
    for got, ref in zip(tables.blocks[0], O.adaln_tables(temb, 6, 3, True, q=qref["blocks.0.adaln_proj.linear"])):
        assert_close(f32(to_np_bf16(got)), f32(ref), rel=2e-2, cos=0.9999, what="loaded adaln table")
    ad_d = h3.load_adaln(w, "blocks.1.adaln_proj", ted, 6, 3)
    assert isinstance(ad_d.linear, h3.DenseLinear) and ad_d.linear.in_dim == rank
    c = O.normal_bf16((2, rank), 9, 40)
    for got, ref in zip(ad_d(to_torch_bf16(c), apply_silu=False),
                        O.adaln_tables(c, 6, 3, False, dense=(np.ascontiguousarray(dense_w.T), None))):
        assert_close(f32(to_np_bf16(got)), f32(ref), rel=1e-2, cos=0.9999, what="dense adaln table")
    refiner = h3.load_text_refiner(w, cfg, text_dim)
    assert refiner.condition_proj is not None and len(refiner.blocks) == 1 and refiner.final_norm is not None
    text = O.normal_bf16((96, text_dim), 9, 41)
    got = refiner(to_torch_bf16(text))
    h3.context().check_device()
    blk = {"qkv": qref["token_refiner.blocks.0.attn.qkv_proj"], "out": qref["token_refiner.blocks.0.attn.out_proj"],
           "fc1": qref["token_refiner.blocks.0.mlp.fc1"], "fc2": qref["token_refiner.blocks.0.mlp.fc2"],
           "q_norm": t["token_refiner.blocks.0.attn.q_norm.weight"],
           "k_norm": t["token_refiner.blocks.0.attn.k_norm.weight"],
           "norm1": t["token_refiner.blocks.0.norm1.weight"], "norm2": t["token_refiner.blocks.0.norm2.weight"]}
    want = O.refine_text(text, dict(hidden=hidden, heads=heads, head_dim=128, eps=1e-5, mlp_kind=1),
                         qref["condition_proj"], [blk], t["token_refiner.final_norm.weight"])
    assert_close(f32(to_np_bf16(got)), f32(want), rel=2e-2, cos=0.999, what="loaded refiner")
    w.close()
