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
