"""numpy front end of the C oracle (oracle/wx_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference legs of bench.py, never by the product package.
bf16 arrays are numpy uint16 bit patterns. Parity status: see wx_oracle.h.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libwxoracle.so"

EPI_NONE, EPI_GELU, EPI_GATE_RESID, EPI_SWIGLU = 0, 1, 2, 3

_vp, _i64, _i32, _f32, _u64 = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_uint64
_SIGS = {
    "wxo_f32_to_bf16": (None, [_vp, _vp, _i64]),
    "wxo_bf16_to_f32": (None, [_vp, _vp, _i64]),
    "wxo_fill_normal_f32": (None, [_vp, _i64, _u64, _u64, _f32, _f32]),
    "wxo_fill_normal_bf16": (None, [_vp, _i64, _u64, _u64, _f32, _f32]),
    "wxo_quantize_affine": (_i32, [_vp, _i64, _i64, _i32, _i32, _vp, _vp, _vp]),
    "wxo_dequantize_affine": (_i32, [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _vp]),
    "wxo_qlinear": (_i32, [_vp, _i64, _i64, _vp, _vp, _vp, _i64, _i32, _i32, _vp, _i32, _vp, _vp, _vp, _vp, _vp]),
    "wxo_qk_norm_rope": (_i32, [_vp, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _i32, _f32, _vp, _i64]),
    "wxo_norm_modscale": (_i32, [_vp, _i64, _i64, _vp, _vp, _vp, _vp, _f32, _vp]),
    "wxo_mod_gate": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "wxo_sol_route": (_i32, [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i64, _i32, _f32, _f32, _i32, _i32,
                             _vp, _vp, _vp, _vp, _vp]),
    "wxo_topk_route": (_i32, [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i64, _i32, _f32, _f32,
                              _vp, _vp, _vp, _vp, _vp]),
    "wxo_sparse_attention": (_i32, [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i64, _i32, _f32, _vp, _vp, _vp, _vp,
                                    _i32, _vp, _i64]),
    "wxo_sparse_attention_rows": (_i32, [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i64, _i32, _f32, _vp, _vp, _vp,
                                         _vp, _i32, _i64, _i64, _vp, _i64]),
    "wxo_dense_f32": (_i32, [_vp, _i64, _i64, _vp, _i64, _vp, _vp]),
    "wxo_num_threads": (_i32, []),
    "wxo_set_num_threads": (_i32, [_i32]),
}

_lib = None


def build() -> Path:
    src, hdr = HERE / "wx_oracle.c", HERE / "wx_oracle.h"
    LIB.parent.mkdir(exist_ok=True)
    if not LIB.exists() or LIB.stat().st_mtime < max(src.stat().st_mtime, hdr.stat().st_mtime):
        subprocess.check_call(["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-ffp-contract=off", "-fPIC",
                               "-shared", "-o", str(LIB), str(src), "-lm"])
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        l = C.CDLL(str(LIB))
        for n, (r, a) in _SIGS.items():
            f = getattr(l, n)
            f.restype = r
            f.argtypes = a
        _lib = l
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data


def _chk(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"oracle {what} failed ({rc})")


# ------------------------------------------------------------------------- bf16 / RNG
def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().wxo_f32_to_bf16(_ptr(x), _ptr(out), x.size)
    return out


def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    out = np.empty(x.shape, dtype=np.float32)
    lib().wxo_bf16_to_f32(_ptr(x), _ptr(out), x.size)
    return out


def normal_f32(shape, seed: int, stream: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(shape, dtype=np.float32)
    lib().wxo_fill_normal_f32(_ptr(out), out.size, seed, stream, mean, std)
    return out


def normal_bf16(shape, seed: int, stream: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(shape, dtype=np.uint16)
    lib().wxo_fill_normal_bf16(_ptr(out), out.size, seed, stream, mean, std)
    return out


# ------------------------------------------------------------------------ quantization
def quantize(w: np.ndarray, bits: int = 6, group: int = 64):
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    wq = np.empty((n, k * bits // 32), dtype=np.uint32)
    sc = np.empty((n, k // group), dtype=np.uint16)
    bi = np.empty((n, k // group), dtype=np.uint16)
    _chk(lib().wxo_quantize_affine(_ptr(w), n, k, group, bits, _ptr(wq), _ptr(sc), _ptr(bi)), "quantize")
    return wq, sc, bi


def dequantize(wq, sc, bi, k: int, bits: int = 6, group: int = 64) -> np.ndarray:
    n = wq.shape[0]
    out = np.empty((n, k), dtype=np.uint16)
    _chk(lib().wxo_dequantize_affine(_ptr(np.ascontiguousarray(wq)), _ptr(np.ascontiguousarray(sc)),
                                     _ptr(np.ascontiguousarray(bi)), n, k, group, bits, _ptr(out)), "dequantize")
    return out


def qlinear(x, wq, sc, bi, bits=6, group=64, bias=None, epilogue=EPI_NONE, gate=None, resid=None, rowmap=None,
            want_raw=False):
    x = np.ascontiguousarray(x, dtype=np.uint16)
    m, k = x.shape
    n = wq.shape[0]
    ncols = n // 2 if epilogue == EPI_SWIGLU else n
    y = np.empty((m, ncols), dtype=np.uint16)
    raw = np.empty((m, n), dtype=np.uint16) if want_raw else None
    _chk(lib().wxo_qlinear(_ptr(x), m, k, _ptr(np.ascontiguousarray(wq)), _ptr(np.ascontiguousarray(sc)),
                           _ptr(np.ascontiguousarray(bi)), n, group, bits, _ptr(bias), epilogue, _ptr(gate),
                           _ptr(resid), _ptr(rowmap), _ptr(y), _ptr(raw)), "qlinear")
    return (y, raw) if want_raw else y


def lora_delta(x, loras):
    """loraDelta (H3Common.swift:424-433) with the reference's bf16 intermediates:
    sum_i bf16(bf16(bf16(x A_i) B_i) * scale_i), accumulated in bf16. x [m, k] bf16 bits;
    loras = [(a [k, r] bf16 bits, b [r, n] bf16 bits, scale)]. Returns fp32 values."""
    xf = bf16_to_f32(np.ascontiguousarray(x, dtype=np.uint16))
    acc = None
    for a, b, scale in loras:
        xa = bf16_to_f32(f32_to_bf16(xf @ bf16_to_f32(a)))
        d = bf16_to_f32(f32_to_bf16(xa @ bf16_to_f32(b)))
        d = bf16_to_f32(f32_to_bf16(d * np.float32(bf16_to_f32(f32_to_bf16(np.float32(scale))))))
        acc = d if acc is None else bf16_to_f32(f32_to_bf16(acc + d))
    return acc


def qlinear_lora(x, wq, sc, bi, loras, bits=6, group=64, bias=None, epilogue=EPI_NONE, gate=None, resid=None,
                 rowmap=None, want_raw=False):
    """MfLinear.forward with adapters (H3Common.swift:341-375): bf16(qmm + bias) + delta, rounded,
    then the epilogue (GELU, or resid + y * gate[rowmap[r]]) in fp32 with one bf16 rounding.
    want_raw: also return the linear's output before the epilogue."""
    base = bf16_to_f32(qlinear(x, wq, sc, bi, bits, group, bias))
    y = bf16_to_f32(f32_to_bf16(base + lora_delta(x, loras)))
    if epilogue == EPI_NONE:
        out = f32_to_bf16(y)
    elif epilogue == EPI_GELU:
        c = np.float32(0.7978845608028654)
        out = f32_to_bf16(np.float32(0.5) * y * (np.float32(1) + np.tanh(c * (y + np.float32(0.044715) * y ** 3))))
    elif epilogue == EPI_GATE_RESID:
        g = bf16_to_f32(gate)[np.asarray(rowmap, dtype=np.int64)]
        out = f32_to_bf16(bf16_to_f32(resid) + y * g)
    else:
        raise ValueError("qlinear_lora: unsupported epilogue")
    return (out, f32_to_bf16(y)) if want_raw else out


# --------------------------------------------------------------------------- row ops
def qk_norm_rope(x: np.ndarray, w, cos, sin, rot: int, eps: float) -> np.ndarray:
    """x [S, H, hd] uint16 (contiguous)."""
    x = np.ascontiguousarray(x)
    S, H, hd = x.shape
    out = np.empty_like(x)
    _chk(lib().wxo_qk_norm_rope(_ptr(x), H * hd, S, H, hd, _ptr(w), _ptr(cos), _ptr(sin), rot, eps, _ptr(out),
                                H * hd), "qk_norm_rope")
    return out


def norm_modscale(x, w, shift, scale, rowmap, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x)
    S, hidden = x.shape
    out = np.empty_like(x)
    _chk(lib().wxo_norm_modscale(_ptr(x), S, hidden, _ptr(w), _ptr(shift), _ptr(scale), _ptr(rowmap), eps,
                                 _ptr(out)), "norm_modscale")
    return out


def mod_gate(x, other, gate, rowmap) -> np.ndarray:
    x = np.ascontiguousarray(x)
    S, hidden = x.shape
    out = np.empty_like(x)
    _chk(lib().wxo_mod_gate(_ptr(x), _ptr(np.ascontiguousarray(other)), _ptr(gate), _ptr(rowmap), S, hidden,
                            _ptr(out)), "mod_gate")
    return out


# ------------------------------------------------------------------------- attention
def sol_route(q, k, v, g: int, scale: float, tau: float, block: int = 64, sink=(0, 0)):
    """q/k/v [S, H, hd] uint16 contiguous. Returns dict(sel, thr, cm, vsum, lens)."""
    S, H, hd = q.shape
    nb = (S - g + block - 1) // block
    sel = np.empty((H, nb, nb), dtype=np.uint8)
    thr = np.empty((H, nb), dtype=np.float32)
    cm = np.empty((H, nb, nb), dtype=np.uint16)
    vsum = np.empty((H, nb, hd), dtype=np.uint16)
    lens = np.empty((nb,), dtype=np.float32)
    _chk(lib().wxo_sol_route(_ptr(q), _ptr(k), _ptr(v), H * hd, S, H, hd, g, block, scale, tau, sink[0], sink[1],
                             _ptr(sel), _ptr(thr), _ptr(cm), _ptr(vsum), _ptr(lens)), "sol_route")
    return dict(sel=sel, thr=thr, cm=cm, vsum=vsum, lens=lens)


def topk_route(q, k, v, g: int, scale: float, density: float, block: int = 128):
    S, H, hd = q.shape
    nb = (S - g + block - 1) // block
    sel = np.empty((H, nb, nb), dtype=np.uint8)
    scores = np.empty((H, nb, nb), dtype=np.float32)
    cm = np.empty((H, nb, nb), dtype=np.uint16)
    vsum = np.empty((H, nb, hd), dtype=np.uint16)
    lens = np.empty((nb,), dtype=np.float32)
    _chk(lib().wxo_topk_route(_ptr(q), _ptr(k), _ptr(v), H * hd, S, H, hd, g, block, scale, density, _ptr(sel),
                              _ptr(scores), _ptr(cm), _ptr(vsum), _ptr(lens)), "topk_route")
    return dict(sel=sel, scores=scores, cm=cm, vsum=vsum, lens=lens)


def sparse_attention(q, k, v, g: int, scale: float, block: int = 64, route=None, tail: bool = True):
    """route None: dense attention for every row; else SOL semantics with route's tables."""
    S, H, hd = q.shape
    out = np.empty((S, H, hd), dtype=np.uint16)
    if route is None:
        _chk(lib().wxo_sparse_attention(_ptr(q), _ptr(k), _ptr(v), H * hd, S, H, hd, 0, block, scale, None, None,
                                        None, None, 0, _ptr(out), H * hd), "attention")
    else:
        _chk(lib().wxo_sparse_attention(_ptr(q), _ptr(k), _ptr(v), H * hd, S, H, hd, g, block, scale,
                                        _ptr(route["sel"]), _ptr(route["cm"]), _ptr(route["vsum"]),
                                        _ptr(route["lens"]), int(tail), _ptr(out), H * hd), "attention")
    return out


def attention_rows(q, k, v, g: int, scale: float, row0: int, row1: int, block: int = 128, route=None,
                   tail: bool = False):
    """Attention output for query rows [row0, row1) only; q/k/v [S, H, hd] uint16."""
    S, H, hd = q.shape
    out = np.zeros((S, H, hd), dtype=np.uint16)
    r = route or {}
    _chk(lib().wxo_sparse_attention_rows(_ptr(q), _ptr(k), _ptr(v), H * hd, S, H, hd, g if route else 0, block,
                                         scale, _ptr(r.get("sel")), _ptr(r.get("cm")), _ptr(r.get("vsum")),
                                         _ptr(r.get("lens")), int(tail), row0, row1, _ptr(out), H * hd),
         "attention_rows")
    return out[row0:row1]


def dense_f32(x, w, b=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    m, k = x.shape
    n = w.shape[1]
    y = np.empty((m, n), dtype=np.float32)
    _chk(lib().wxo_dense_f32(_ptr(x), m, k, _ptr(w), n, _ptr(b), _ptr(y)), "dense_f32")
    return y


def num_threads() -> int:
    return lib().wxo_num_threads()


def set_num_threads(n: int = 0) -> int:
    """OpenMP threads of later oracle calls, overriding OMP_NUM_THREADS (n <= 0: all processors)."""
    return lib().wxo_set_num_threads(int(n))


# ---------------------------------------------------------------- block composition
def block_forward(h, w, mods, rowmap, cos, sin, cfg, route_fn=None, at_cached=None, refresh=True,
                  qkv_override=None):
    """One H3 DiT block (H3Transformer.swift:1078-1159) composed from the oracle ops.

    w: dict of quantized triples qkv/out/fc1/fc2 (wq, sc, bi, bias) and norms, optionally
    w["lora"][name] = [(a, b, scale), ...] (loraDelta, H3Common.swift:424-433); mods: 6 tables;
    route_fn(q, k, v) -> route dict or None for dense. qkv_override: the qkv projection's
    output [S, 3*inner] to use instead of computing it (a test that checks the projection on
    its own can feed the block the checked tensor). Returns (h_new, at)."""
    S, hidden = h.shape
    H, hd = cfg["heads"], cfg["head_dim"]
    inner = H * hd
    eps = cfg["eps"]
    lora = w.get("lora", {})

    def lin(name, x, **kw):  # quantized linear, with its LoRA adapters when attached
        if lora.get(name):
            return qlinear_lora(x, *w[name][:3], lora[name], bias=w[name][3], **kw)
        return qlinear(x, *w[name][:3], bias=w[name][3], **kw)

    if refresh or at_cached is None:
        if qkv_override is None:
            m1 = norm_modscale(h, w["norm1"], mods[0], mods[1], rowmap, eps)
            qkv = lin("qkv", m1)
        else:
            qkv = np.ascontiguousarray(qkv_override, dtype=np.uint16)
        q = qkv[:, :inner].reshape(S, H, hd)
        k = qkv[:, inner:2 * inner].reshape(S, H, hd)
        v = np.ascontiguousarray(qkv[:, 2 * inner:].reshape(S, H, hd))
        q = qk_norm_rope(q, w["q_norm"], cos, sin, cfg["rot"], eps)
        k = qk_norm_rope(k, w["k_norm"], cos, sin, cfg["rot"], eps)
        scale = 1.0 / np.sqrt(np.float32(hd))
        route = route_fn(q, k, v) if route_fn else None
        if route is None:
            att = sparse_attention(q, k, v, 0, float(scale))
        else:
            att = sparse_attention(q, k, v, route["g"], float(scale), block=route["block"], route=route,
                                   tail=route["tail"])
        ha, at = lin("out", att.reshape(S, inner), epilogue=EPI_GATE_RESID, gate=mods[2], resid=h, rowmap=rowmap,
                     want_raw=True)
    else:
        at = at_cached
        ha = mod_gate(h, at, mods[2], rowmap)
    m2 = norm_modscale(ha, w["norm2"], mods[3], mods[4], rowmap, eps)
    act = EPI_SWIGLU if cfg.get("mlp_kind", 0) == 1 else EPI_GELU
    f1 = lin("fc1", m2, epilogue=act)
    hn = lin("fc2", f1, epilogue=EPI_GATE_RESID, gate=mods[5], resid=ha, rowmap=rowmap)
    return hn, at


# ------------------------------------------------------------ conditioning (per generation)
def timestep_sinusoid(ts, dim: int = 256) -> np.ndarray:
    """H3TimeEmbedder.forward's host loop (H3Transformer.swift:288-299): row i =
    [cos(t_i f_j) | sin(t_i f_j)], f_j = exp(-ln(10000) j / half), in double, stored fp32."""
    half = dim // 2
    j = np.arange(half, dtype=np.float64)
    freq = np.exp(-np.log(10000.0) * j / half)
    arg = np.asarray(ts, dtype=np.float64)[:, None] * freq[None, :]
    return np.concatenate([np.cos(arg), np.sin(arg)], axis=1).astype(np.float32)


def sigmoid_mlx(x: np.ndarray) -> np.ndarray:
    """MLX's sigmoid: y = 1 / (1 + exp(-|x|)), mirrored for x < 0 (fp32)."""
    x = np.asarray(x, dtype=np.float32)
    y = (np.float32(1) / (np.float32(1) + np.exp(-np.abs(x)))).astype(np.float32)
    return np.where(x < 0, np.float32(1) - y, y).astype(np.float32)


def silu_f32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return (x * sigmoid_mlx(x)).astype(np.float32)


def silu_bf16(x: np.ndarray) -> np.ndarray:
    """silu on a bf16 array as MLX composes it: bf16(x * bf16(sigmoid(x)))."""
    xf = bf16_to_f32(x)
    s = bf16_to_f32(f32_to_bf16(sigmoid_mlx(xf)))
    return f32_to_bf16(xf * s)


def time_embed(ts, w_in, b_in, w_out, b_out, freq_dim: int = 256) -> np.ndarray:
    """H3TimeEmbedder.forward (H3Transformer.swift:287-302): [m, out] fp32."""
    h1 = silu_f32(dense_f32(timestep_sinusoid(ts, freq_dim), w_in, b_in))
    return dense_f32(h1, w_out, b_out)


def lut_rows(ts, n_rows: int) -> np.ndarray:
    """H3AdalnLUT.coeffs row index (H3Transformer.swift:340-345): Double.rounded() (ties away
    from zero) of t·(n-1), clamped to [0, n-1]."""
    x = np.asarray(ts, dtype=np.float64) * (n_rows - 1)
    r = np.where(x < 0, -np.floor(-x + 0.5), np.floor(x + 0.5))
    return np.clip(r, 0, n_rows - 1).astype(np.int64)


def lut_coeffs(ts, t_table: np.ndarray) -> np.ndarray:
    return f32_to_bf16(np.asarray(t_table, dtype=np.float32)[lut_rows(ts, t_table.shape[0])])


def linear_bf16(x, w, bias=None) -> np.ndarray:
    """Dense MfLinear (H3Common.swift:361-366): bf16(bf16(x w) + bias), w [in, out] bf16."""
    acc = bf16_to_f32(x).astype(np.float64) @ bf16_to_f32(w).astype(np.float64)
    y = bf16_to_f32(f32_to_bf16(acc.astype(np.float32)))
    if bias is not None:
        y = y + bf16_to_f32(bias)[None, :]
    return f32_to_bf16(y.astype(np.float32))


def adaln_split(y: np.ndarray, expand: int, modalities: int) -> list:
    """H3AdalnW.forward's reshape + split (H3Transformer.swift:397-403): y [m, modalities·expand·hidden]
    -> expand tables [m·modalities, hidden]."""
    m, n = y.shape
    hidden = n // (expand * modalities)
    v = y.reshape(m * modalities, expand * hidden)
    return [np.ascontiguousarray(v[:, e * hidden:(e + 1) * hidden]) for e in range(expand)]


def adaln_tables(t_emb, expand: int, modalities: int, apply_silu: bool, q=None, dense=None, lora=None):
    """H3AdalnW.forward (H3Transformer.swift:392-404): q = (wq, sc, bi, bias) quantized linear
    (with optional LoRA adapters), or dense = (w [in, out], bias)."""
    x = silu_bf16(t_emb) if apply_silu else np.ascontiguousarray(t_emb)
    if q is not None:
        wq, sc, bi, bias = q
        y = qlinear_lora(x, wq, sc, bi, lora, bias=bias) if lora else qlinear(x, wq, sc, bi, bias=bias)
    else:
        y = linear_bf16(x, dense[0], dense[1])
    return adaln_split(y, expand, modalities)


def rms_norm(x, w, eps: float) -> np.ndarray:
    """rmsNormLast (H3Common.swift:502-508): bf16(x * rsqrt(mean(x^2) + eps) * w), the same
    arithmetic as the fused norm with zero modulation (bf16(n)·(0+1)+0 is exact)."""
    x = np.ascontiguousarray(x)
    zero = np.zeros((1, x.shape[1]), dtype=np.uint16)
    return norm_modscale(x, w, zero, zero, None, eps)


def refiner_block_forward(h, w, cfg):
    """One token-refiner block (H3DiT.refineText loop body, H3Transformer.swift:1003-1010):
    h += attn(rmsNorm(h, norm1)) with q/k RMSNorm and no RoPE, dense attention;
    h += mlp(rmsNorm(h, norm2)). Residual adds are bf16(h + bf16(branch))."""
    L, hidden = h.shape
    H, hd = cfg["heads"], cfg["head_dim"]
    inner = H * hd
    eps = cfg["eps"]
    lora = w.get("lora", {})
    ones = f32_to_bf16(np.ones((1, hidden), dtype=np.float32))

    def lin(name, x, **kw):
        if lora.get(name):
            return qlinear_lora(x, *w[name][:3], lora[name], bias=w[name][3], **kw)
        return qlinear(x, *w[name][:3], bias=w[name][3], **kw)

    n1 = rms_norm(h, w["norm1"], eps)
    qkv = lin("qkv", n1)
    q = qk_norm_rope(qkv[:, :inner].reshape(L, H, hd), w["q_norm"], None, None, 0, eps)
    k = qk_norm_rope(qkv[:, inner:2 * inner].reshape(L, H, hd), w["k_norm"], None, None, 0, eps)
    v = np.ascontiguousarray(qkv[:, 2 * inner:].reshape(L, H, hd))
    att = sparse_attention(q, k, v, 0, float(1.0 / np.sqrt(np.float64(hd))))
    ha = lin("out", att.reshape(L, inner), epilogue=EPI_GATE_RESID, gate=ones, resid=h)
    n2 = rms_norm(ha, w["norm2"], eps)
    act = EPI_SWIGLU if cfg.get("mlp_kind", 0) == 1 else EPI_GELU
    f1 = lin("fc1", n2, epilogue=act)
    return lin("fc2", f1, epilogue=EPI_GATE_RESID, gate=ones, resid=ha)


def refine_text(text, cfg, condition_proj=None, blocks=(), final_norm=None, cp_lora=None):
    """H3DiT.refineText (H3Transformer.swift:993-1016); condition_proj = (wq, sc, bi, bias)."""
    if text.shape[1] == cfg["hidden"]:
        return np.array(text, copy=True)
    wq, sc, bi, bias = condition_proj
    h = qlinear_lora(text, wq, sc, bi, cp_lora, bias=bias) if cp_lora else qlinear(text, wq, sc, bi, bias=bias)
    for b in blocks:
        h = refiner_block_forward(h, b, cfg)
    return rms_norm(h, final_norm, cfg["eps"]) if final_norm is not None else h


# ---------------------------------------------------------------- RoPE and positions
def axis_from_sqrt_area(dim: int, patch: int, sqrt_area: float) -> np.ndarray:
    """axisFromSqrtArea (H3Layout.swift:188-194), float64."""
    n = dim // patch
    ratio = float(dim) / sqrt_area
    step = ratio / n
    start = (1.0 - ratio) / 2.0
    return np.array([(i * step + start) * 32.0 for i in range(n)], dtype=np.float64)


def video_t_grid(n: int, origin: float) -> np.ndarray:
    """videoTGrid (H3Layout.swift:202-210) with videoTSpan = 5/3 * [1,4,4,4,4][k % 5]."""
    out, acc = [], float(origin)
    for i in range(n):
        out.append(acc)
        acc += (5.0 / 3.0) * (1, 4, 4, 4, 4)[i % 5]
    return np.array(out, dtype=np.float64)


def build_rope(pos: np.ndarray, inv_freq: np.ndarray):
    """buildRope (H3Layout.swift:725-740): fp32 angles pos*inv, cos/sin evaluated in float64
    and rounded to fp32, then to bf16."""
    p = np.asarray(pos, dtype=np.float32)
    inv = np.asarray(inv_freq, dtype=np.float32)
    ang = (p[:, :, None] * inv[None, None, :]).astype(np.float32).reshape(p.shape[0], -1)
    a64 = ang.astype(np.float64)
    return f32_to_bf16(np.cos(a64).astype(np.float32)), f32_to_bf16(np.sin(a64).astype(np.float32))
