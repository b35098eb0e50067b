"""Host-side mirror of the reference's H3 hot-path interface over libwx.

Names follow the Swift API of HuaChayu/wuxianhuabu so that a caller (and the
parity tests) read like the reference:

* ``MfLinear``              — model/minimax h3/H3Common.swift:283-404
* ``H3FusedKernels``        — model/2网络算子/网络算子-融合-RMSNormRoPE-通用.swift:28-345
* ``H3SolAttnConfig`` / ``H3SolAttn`` — 网络算子-稀疏注意力-SOL通用.swift:79-678
* ``H3AttnBroadcast`` + ``attn_broadcast_*`` — 网络算子-注意力跨步缓存-通用.swift:36-112
* ``sigma_schedule`` / ``sparse_mode_for_layer`` — model/minimax h3/H3Layout.swift:175-182, 896-906
* ``H3DiTBlocks``           — the block loop of H3DiT.forward, H3Transformer.swift:1078-1159

Tensors are torch CUDA tensors used purely as device buffers; all compute is
in libwx (sm_100a). q/k/v use the reference's pre-transpose layout [S, H, hd].
Errors raise ``WxError``; nothing falls back to a CPU path.
"""
from __future__ import annotations

import ctypes as C
import math
import os
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import (EPI_GATE_RESID, EPI_GELU, EPI_NONE, EPI_SWIGLU, MLP_GELU, MLP_SWIGLU, SPARSE_DENSE, SPARSE_SOL,
                   SPARSE_TOPK, BlockMods, BlockWeights, DitConfig, Lora, LoraPack, ModRun, QWeight, SparseSpec, StInfo,
                   WxError, check)

__all__ = [
    "Context", "context", "MfLinear", "H3FusedKernels", "H3SolAttnConfig", "H3SolAttn", "H3AttnBroadcast",
    "attn_broadcast_refresh", "attn_broadcast_must_refresh", "attn_broadcast_plan",
    "attn_broadcast_default_max_stale", "sigma_schedule", "sparse_mode_for_layer", "SparsePolicy",
    "H3DiTConfig", "H3BlockWeights", "H3DiTBlocks", "ModRun", "WxError", "LoraRef", "H3Weights", "load_block",
    "EPI_NONE", "EPI_GELU", "EPI_GATE_RESID", "EPI_SWIGLU",
    "DenseLinear", "H3TimeEmbedder", "H3AdalnLUT", "H3AdalnW", "H3AdalnTables", "precompute_adaln",
    "H3TextRefiner", "rms_norm", "load_refiner_block", "load_text_refiner", "load_time_embedder", "load_adaln",
    "axis_from_sqrt_area", "video_t_span", "video_t_grid", "write_frame_grid", "packed_positions", "build_rope",
    "H3DiT", "H3AudioRows",
]


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


class Context:
    """One libwx context per CUDA device; calls are ordered on torch's current stream."""

    def __init__(self, device: int = 0):
        self.lib = _lib.load()
        if not torch.cuda.is_available():
            raise RuntimeError("libwx needs a CUDA device (sm_100a); no CPU fallback exists")
        self.device = device
        self.sp_size, self.sp_rank = 1, 0
        h = C.c_void_p()
        st = self.lib.wx_ctx_create(device, C.byref(h))
        if st != 0:
            raise WxError(st, f"wx_ctx_create(device={device}) failed")
        self.h = h

    def sync_stream(self) -> None:
        s = torch.cuda.current_stream(self.device).cuda_stream
        check(self.lib.wx_ctx_set_stream(self.h, C.c_void_p(s)), self.h)

    def check_device(self) -> None:
        check(self.lib.wx_ctx_check_device(self.h), self.h)

    def sp_exchange(self) -> int:
        """Sequence-parallel exchange path: 1 NVLink peer memory, 0 NCCL all-to-alls,
        -1 not decided yet (no refreshed block has run on the group)."""
        return int(self.lib.wx_ctx_sp_exchange(self.h))

    def call(self, name: str, *args) -> None:
        self.sync_stream()
        check(getattr(self.lib, name)(self.h, *args), self.h)

    TRACE_PHASES = ("norm1", "qkv", "rope", "attn", "out", "mlp")
    TRACE_MODES = ("dense", "sparse", "reuse")

    def trace(self, enable: bool = True) -> None:
        """Start (or stop) the per-layer phase trace; clears what was recorded."""
        check(self.lib.wx_ctx_trace_enable(self.h, int(enable)), self.h)

    def trace_read(self, max_records: int = 4096) -> list:
        """Records since trace()/the last read, one per block forward: dicts with the layer
        (block forwards counted from 0), mode, the milliseconds of each phase and the total."""
        import ctypes
        nf = 9
        buf = (ctypes.c_double * (nf * max_records))()
        n = ctypes.c_int(0)
        check(self.lib.wx_ctx_trace_read(self.h, buf, max_records, ctypes.byref(n)), self.h)
        out = []
        for i in range(n.value):
            r = buf[i * nf:(i + 1) * nf]
            d = dict(layer=int(r[0]), mode=self.TRACE_MODES[int(r[1])], total_ms=r[8])
            d.update({p + "_ms": r[2 + j] for j, p in enumerate(self.TRACE_PHASES)})
            out.append(d)
        return out

    @staticmethod
    def format_trace(records: list) -> str:
        """The records as the reference's per-layer profile lines
        (H3Transformer.swift:587-588: qkv, ropeN, attn(mode), out, tot), with norm1 and mlp added."""
        lines = []
        for r in records:
            mode = {"dense": "dense", "sparse": "sol", "reuse": "pab"}[r["mode"]]
            lines.append("[PROF] L%02d norm1=%.2fms qkv=%.2fms ropeN=%.2fms attn(%s)=%.2fms out=%.2fms mlp=%.2fms "
                         "tot=%.2fms" % (r["layer"] + 1, r["norm1_ms"], r["qkv_ms"], r["rope_ms"], mode,
                                         r["attn_ms"], r["out_ms"], r["mlp_ms"], r["total_ms"]))
        return "\n".join(lines)

    def close(self) -> None:
        if self.h:
            self.lib.wx_ctx_destroy(self.h)
            self.h = None


_contexts: dict[int, Context] = {}


def context(device: Optional[int] = None) -> Context:
    dev = torch.cuda.current_device() if device is None else device
    if dev not in _contexts:
        _contexts[dev] = Context(dev)
    return _contexts[dev]


def _need_bf16_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda or t.dtype != torch.bfloat16:
            raise WxError(_lib.WX_ERR_INVALID, f"expected a CUDA bf16 tensor, got {t.dtype} on {t.device}")


# --------------------------------------------------------------------------- MfLinear
@dataclass
class LoraRef:
    """LoraRef (H3Common.swift:407-411): the layer adds scale * ((x a) b)."""
    a: torch.Tensor  # [in, r] bf16
    b: torch.Tensor  # [r, out] bf16
    scale: float


class MfLinear:
    """6-bit (2..8-bit) MLX-affine group-quantized linear layer (H3Common.swift:283-404).

    ``w`` packed uint32 [out, in*bits/32] (stored as int32), ``scales``/``biases`` bf16
    [out, in/group], optional ``bias`` bf16 [out]. bits and group are derived as in
    MfLinear.load (:321-323)."""

    def __init__(self, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, in_dim: int,
                 bias: Optional[torch.Tensor] = None):
        if w.dtype not in (torch.int32, torch.uint32):
            raise WxError(_lib.WX_ERR_INVALID, "packed weight must be 32-bit words")
        self.w, self.scales, self.biases, self.bias = w.contiguous(), scales.contiguous(), biases.contiguous(), bias
        self.in_dim = in_dim
        self.out_dim = w.shape[0]
        self.bits = 32 * w.shape[1] // in_dim
        self.group_size = in_dim // scales.shape[1]
        self.lora: list[LoraRef] = []  # LoraSlot.refs (H3Common.swift:413-417)
        self._pack = None

    def set_lora(self, refs: Sequence["LoraRef"]) -> None:
        """LoraSlot.set (H3Common.swift:416): attach adapters (empty = detach)."""
        self.lora = list(refs)
        self._pack = None

    def lora_pack(self) -> Optional[LoraPack]:
        """The adapters packed as the GEMM's K extension (wx_lora_pack_build), built once."""
        if not self.lora:
            return None
        if self._pack is None:
            lib = _lib.load()
            dev = self.w.device
            for r in self.lora:
                _need_bf16_cuda(r.a, r.b)
            arr = (Lora * len(self.lora))(*[Lora(_p(r.a.contiguous()), _p(r.b.contiguous()), r.a.shape[1],
                                                 float(r.scale)) for r in self.lora])
            R, ab, bb = C.c_int64(), C.c_size_t(), C.c_size_t()
            check(lib.wx_lora_pack_bytes(self.out_dim, self.in_dim, arr, len(self.lora), C.byref(R), C.byref(ab),
                                         C.byref(bb)))
            at = torch.empty(ab.value // 2, dtype=torch.bfloat16, device=dev)
            bt = torch.empty(bb.value // 2, dtype=torch.bfloat16, device=dev)
            pack = LoraPack(_p(at), _p(bt), 0, 0, 0)
            context(dev.index).call("wx_lora_pack_build", self.out_dim, self.in_dim, arr, len(self.lora),
                                    C.byref(pack))
            self._pack = (pack, at, bt)
        return self._pack[0]

    @classmethod
    def quantize(cls, w_f32: torch.Tensor, bits: int = 6, group: int = 64,
                 bias: Optional[torch.Tensor] = None) -> "MfLinear":
        """Quantize an fp32 [out, in] weight on the GPU (offline step of tools/quantize_h3_g64.py)."""
        n, k = w_f32.shape
        dev = w_f32.device
        wq = torch.empty((n, k * bits // 32), dtype=torch.int32, device=dev)
        sc = torch.empty((n, k // group), dtype=torch.bfloat16, device=dev)
        bi = torch.empty_like(sc)
        ctx = context(dev.index)
        ctx.call("wx_quantize_affine", _p(w_f32.contiguous()), n, k, group, bits, _p(wq), _p(sc), _p(bi))
        return cls(wq, sc, bi, k, bias)

    def qweight(self) -> QWeight:
        return QWeight(_p(self.w), _p(self.scales), _p(self.biases), _p(self.bias), self.out_dim, self.in_dim,
                       self.group_size, self.bits)

    def dequantized_weight(self) -> torch.Tensor:
        """MfLinear.dequantizedWeight (:379-401): [out, in] bf16."""
        out = torch.empty((self.out_dim, self.in_dim), dtype=torch.bfloat16, device=self.w.device)
        qw = self.qweight()
        context(self.w.device.index).call("wx_dequantize_affine", C.byref(qw), _p(out))
        return out

    def forward(self, x: torch.Tensor, epilogue: int = EPI_NONE, gate: Optional[torch.Tensor] = None,
                resid: Optional[torch.Tensor] = None, rowmap: Optional[torch.Tensor] = None,
                y_raw: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x[..., in] -> [..., out] (quantizedMM + bias, :341-377) with a fused epilogue."""
        _need_bf16_cuda(x, gate, resid, y_raw)
        x2 = x.reshape(-1, self.in_dim)
        if x2.stride(1) != 1:
            x2 = x2.contiguous()
        m = x2.shape[0]
        n_out = self.out_dim // 2 if epilogue == EPI_SWIGLU else self.out_dim
        y = out if out is not None else torch.empty((m, n_out), dtype=torch.bfloat16, device=x.device)
        qw = self.qweight()
        pack = self.lora_pack()
        if pack is not None:  # quantizedMM + bias + loraDelta (:358-375)
            context(x.device.index).call("wx_qlinear_lora", _p(x2), m, x2.stride(0), C.byref(qw), C.byref(pack),
                                         epilogue, _p(gate), _p(resid), _p(rowmap), _p(y), y.stride(0), _p(y_raw))
        else:
            context(x.device.index).call("wx_qlinear", _p(x2), m, x2.stride(0), C.byref(qw), epilogue, _p(gate),
                                         _p(resid), _p(rowmap), _p(y), y.stride(0), _p(y_raw))
        return y.reshape(*x.shape[:-1], n_out)

    __call__ = forward

    def qkv_norm_rope(self, x: torch.Tensor, heads: int, head_dim: int, q_norm: torch.Tensor,
                      k_norm: torch.Tensor, cos: Optional[torch.Tensor], sin: Optional[torch.Tensor], rot: int,
                      eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The q|k|v projection of H3AttnW.forward with its two fusedRmsnormRope calls
        (H3Transformer.swift:451-475) as one call (wx_qkv_norm_rope): x [m, in] -> [m, 3*heads*head_dim]
        with q and k normalised and rotated (in the GEMM's epilogue where the geometry allows)."""
        _need_bf16_cuda(x, q_norm, k_norm, cos, sin)
        x2 = x.reshape(-1, self.in_dim)
        if x2.stride(1) != 1:
            x2 = x2.contiguous()
        m = x2.shape[0]
        y = out if out is not None else torch.empty((m, self.out_dim), dtype=torch.bfloat16, device=x.device)
        qw = self.qweight()
        pack = self.lora_pack()
        context(x.device.index).call("wx_qkv_norm_rope", _p(x2), m, x2.stride(0), C.byref(qw),
                                     C.byref(pack) if pack is not None else None, heads, head_dim, _p(q_norm),
                                     _p(k_norm), _p(cos), _p(sin), rot, float(eps), _p(y), y.stride(0))
        return y


# ------------------------------------------------------------------- fused row kernels
class H3FusedKernels:
    """h3_fused_rmsnorm_rope / h3_fused_norm_modscale / h3_fused_mod_gate (fused:28-345)."""

    @staticmethod
    def build_row_mod_map(count: int, runs: Sequence[ModRun]) -> np.ndarray:
        """buildRowModMap (fused:238-250): [count] uint32 row -> modRow."""
        lib = _lib.load()
        arr = (ModRun * max(1, len(runs)))(*runs)
        out = np.zeros(count, dtype=np.uint32)
        check(lib.wx_build_row_mod_map(arr, len(runs), count, out.ctypes.data))
        return out

    @staticmethod
    def fused_rmsnorm_rope(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                           rot: int, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """fusedRmsnormRope (fused:111-129). x [S, H, hd] (row stride may exceed H*hd)."""
        _need_bf16_cuda(x, weight, cos, sin)
        S, H, hd = x.shape
        if x.stride(2) != 1 or x.stride(1) != hd:
            raise WxError(_lib.WX_ERR_INVALID, "x must have contiguous heads")
        o = out if out is not None else torch.empty((S, H, hd), dtype=torch.bfloat16, device=x.device)
        context(x.device.index).call("wx_qk_norm_rope", _p(x), x.stride(0), S, H, hd, _p(weight), _p(cos), _p(sin),
                                     rot, float(eps), _p(o), o.stride(0))
        return o

    @staticmethod
    def fused_norm_modscale(x: torch.Tensor, weight: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
                            rowmap: Optional[torch.Tensor], eps: float,
                            out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """fusedNormModscale (fused:262-283); rowmap [S] int32/uint32 on the device."""
        _need_bf16_cuda(x, weight, shift, scale)
        S, hidden = x.shape
        o = out if out is not None else torch.empty_like(x)
        context(x.device.index).call("wx_norm_modscale", _p(x), S, hidden, _p(weight), _p(shift), _p(scale),
                                     _p(rowmap), float(eps), _p(o))
        return o

    @staticmethod
    def fused_norm_modscale_row(x: torch.Tensor, weight: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
                                eps: float) -> torch.Tensor:
        """fusedNormModscaleRow (fused:295-315): one shift/scale row for every row."""
        return H3FusedKernels.fused_norm_modscale(x, weight, shift, scale, None, eps)

    @staticmethod
    def fused_mod_gate(x: torch.Tensor, gate: torch.Tensor, other: torch.Tensor,
                       rowmap: Optional[torch.Tensor], out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """fusedModGate (fused:324-343): x + other * gate[map[r]]."""
        _need_bf16_cuda(x, gate, other)
        S, hidden = x.shape
        o = out if out is not None else torch.empty_like(x)
        context(x.device.index).call("wx_mod_gate", _p(x), _p(other), _p(gate), _p(rowmap), S, hidden, _p(o))
        return o


# --------------------------------------------------------------------- SOL attention
@dataclass
class H3SolAttnConfig:
    """H3SolAttnConfig (SOL:79-98). ``topk_ratio`` selects the top-k router (benchmark mode)."""
    tau: float = 1.3
    sink_blocks: Optional[range] = None
    tail: bool = True
    block: int = 64
    topk_ratio: Optional[float] = None

    def spec(self, g: int) -> SparseSpec:
        mode = SPARSE_TOPK if self.topk_ratio is not None else SPARSE_SOL
        sink = self.sink_blocks or range(0, 0)
        return SparseSpec(mode, self.block, g, float(self.tau), float(self.topk_ratio or 0.0), sink.start,
                          sink.stop, int(self.tail), 0)


def dense_spec() -> SparseSpec:
    return SparseSpec(SPARSE_DENSE, 128, 0, 0.0, 0.0, 0, 0, 0, 0)


class H3SolAttn:
    """H3SolAttn (SOL:383-678) over q/k/v in [S, H, 128] (rows may be strided, e.g. a packed qkv)."""

    @staticmethod
    def _geom(q: torch.Tensor):
        S, H, hd = q.shape
        if q.stride(2) != 1 or q.stride(1) != hd:
            raise WxError(_lib.WX_ERR_INVALID, "q/k/v must have contiguous heads")
        return S, H, hd, q.stride(0)

    @staticmethod
    def forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: int, scale: float,
                cfg: Optional[H3SolAttnConfig] = H3SolAttnConfig(),
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """SOL attention (cfg) or dense SDPA (cfg None). Returns [S, H, hd] bf16."""
        _need_bf16_cuda(q, k, v)
        S, H, hd, rs = H3SolAttn._geom(q)
        if k.stride(0) != rs or v.stride(0) != rs:
            raise WxError(_lib.WX_ERR_INVALID, "q, k and v must share one row stride")
        o = out if out is not None else torch.empty((S, H, hd), dtype=torch.bfloat16, device=q.device)
        spec = dense_spec() if cfg is None else cfg.spec(g)
        context(q.device.index).call("wx_sparse_attention", _p(q), _p(k), _p(v), rs, S, H, hd, C.byref(spec),
                                     float(scale), _p(o), o.stride(0))
        return o

    @staticmethod
    def route(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: int, scale: float, cfg: H3SolAttnConfig):
        """Routing tables: dict(sel, thr|scores, cm, vsum, lens) as device tensors."""
        _need_bf16_cuda(q, k, v)
        S, H, hd, rs = H3SolAttn._geom(q)
        nb = (S - g + cfg.block - 1) // cfg.block
        dev = q.device
        sel = torch.empty((H, nb, nb), dtype=torch.uint8, device=dev)
        cm = torch.empty((H, nb, nb), dtype=torch.bfloat16, device=dev)
        vsum = torch.empty((H, nb, hd), dtype=torch.bfloat16, device=dev)
        lens = torch.empty((nb,), dtype=torch.float32, device=dev)
        spec = cfg.spec(g)
        if spec.mode == SPARSE_SOL:
            thr = torch.empty((H, nb), dtype=torch.float32, device=dev)
            context(dev.index).call("wx_sol_route", _p(q), _p(k), _p(v), rs, S, H, hd, C.byref(spec), float(scale),
                                    _p(sel), _p(thr), _p(cm), _p(vsum), _p(lens))
            return dict(sel=sel, thr=thr, cm=cm, vsum=vsum, lens=lens)
        scores = torch.empty((H, nb, nb), dtype=torch.float32, device=dev)
        context(dev.index).call("wx_topk_route", _p(q), _p(k), _p(v), rs, S, H, hd, C.byref(spec), float(scale),
                                _p(sel), _p(scores), _p(cm), _p(vsum), _p(lens))
        return dict(sel=sel, scores=scores, cm=cm, vsum=vsum, lens=lens)

    @staticmethod
    def attend_with_selection(q, k, v, g: int, scale: float, cfg: H3SolAttnConfig, sel: torch.Tensor,
                              cm=None, vsum=None, lens=None) -> torch.Tensor:
        """The flash kernel alone over a given block selection [H, nb, nb]."""
        _need_bf16_cuda(q, k, v)
        S, H, hd, rs = H3SolAttn._geom(q)
        o = torch.empty((S, H, hd), dtype=torch.bfloat16, device=q.device)
        spec = cfg.spec(g)
        context(q.device.index).call("wx_attention_from_sel", _p(q), _p(k), _p(v), rs, S, H, hd, C.byref(spec),
                                     float(scale), _p(sel), _p(cm), _p(vsum), _p(lens), _p(o), o.stride(0))
        return o


# ----------------------------------------------------------------- PAB + schedules
def attn_broadcast_refresh(i: int, steps: int, k: int) -> bool:
    """attnBroadcastRefresh (PAB:73-79)."""
    return bool(_lib.load().wx_pab_refresh(i, steps, k))


def attn_broadcast_must_refresh(cached_sigma: float, sigma: float, max_stale: float) -> bool:
    """attnBroadcastMustRefresh (PAB:85-87)."""
    return bool(_lib.load().wx_pab_must_refresh(cached_sigma, sigma, max_stale))


def attn_broadcast_plan(sigmas: Sequence[float], k: int, max_stale: float) -> list[bool]:
    """attnBroadcastPlan (PAB:92-105): per-step refresh flags."""
    arr = np.asarray(sigmas, dtype=np.float64)
    out = np.zeros(max(0, len(arr) - 1), dtype=np.uint8)
    _lib.load().wx_pab_plan(arr.ctypes.data, len(arr), k, max_stale, out.ctypes.data if len(out) else None)
    return [bool(x) for x in out]


def attn_broadcast_default_max_stale() -> float:
    """attnBroadcastDefaultMaxStale (PAB:112)."""
    return 0.04


def sigma_schedule(steps: int, shift: float) -> list[float]:
    """sigmaSchedule (H3Layout.swift:175-182)."""
    out = np.zeros(steps + 1, dtype=np.float64)
    check(_lib.load().wx_sigma_schedule(steps, shift, out.ctypes.data))
    return out.tolist()


class SparsePolicy:
    OFF, MIX, SPATIAL, TEMPORAL = 0, 1, 2, 3


def sparse_mode_for_layer(layer: int, n_layers: int, policy: int) -> int:
    """sparseModeForLayer (H3Layout.swift:896-906): 0 dense, 1 spatial, 2 temporal."""
    return _lib.load().wx_sparse_mode_for_layer(layer, n_layers, policy)


class H3AttnBroadcast:
    """PAB cache (PAB:36-52): one device slot [S, hidden] per block, allocated on first refresh."""

    def __init__(self, count: int):
        self.blocks: list[Optional[torch.Tensor]] = [None] * count
        self.cached_sigma = math.inf

    def reset(self) -> None:
        self.blocks = [None] * len(self.blocks)
        self.cached_sigma = math.inf

    def slot(self, bi: int, rows: int, hidden: int, device) -> torch.Tensor:
        t = self.blocks[bi]
        if t is None or t.shape != (rows, hidden):
            t = torch.empty((rows, hidden), dtype=torch.bfloat16, device=device)
            self.blocks[bi] = t
        return t


# ------------------------------------------------------------------------ DiT blocks
@dataclass
class H3DiTConfig:
    hidden: int = 3072
    heads: int = 24
    head_dim: int = 128
    ffn: int = 12288
    mlp_kind: int = MLP_GELU
    rot: int = 96
    eps: float = 1e-6
    layers: int = 48

    def c(self, lora_rank: int = 0) -> DitConfig:
        return DitConfig(self.hidden, self.heads, self.head_dim, self.ffn, self.mlp_kind, self.rot, self.eps,
                         lora_rank)


@dataclass
class H3BlockWeights:
    qkv: MfLinear
    out: MfLinear
    fc1: MfLinear
    fc2: MfLinear
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    norm1: torch.Tensor
    norm2: torch.Tensor

    def linears(self) -> list[MfLinear]:
        return [self.qkv, self.out, self.fc1, self.fc2]

    def c(self) -> BlockWeights:
        packs = [lin.lora_pack() for lin in self.linears()]
        ptrs = (C.POINTER(LoraPack) * 4)(*[C.pointer(pk) if pk is not None else C.POINTER(LoraPack)()
                                           for pk in packs])
        return BlockWeights(self.qkv.qweight(), self.out.qweight(), self.fc1.qweight(), self.fc2.qweight(),
                            _p(self.q_norm), _p(self.k_norm), _p(self.norm1), _p(self.norm2), ptrs)


def sp_plan(S: int, H: int, head_dim: int, P: int, rank: int) -> _lib.SpPlan:
    """Ulysses partition (wx_sp_make_plan): this rank's rows and heads."""
    plan = _lib.SpPlan()
    check(_lib.load().wx_sp_make_plan(S, H, head_dim, P, rank, C.byref(plan)))
    return plan


def init_sequence_parallel(world: int, rank: int, broadcast_id) -> None:
    """Create the NCCL communicator of this process's context. ``broadcast_id(bytes_or_None)``
    returns rank 0's 128-byte id on every rank (e.g. torch.distributed.broadcast_object_list)."""
    lib = _lib.load()
    uid = None
    if rank == 0:
        buf = (C.c_uint8 * 128)()
        check(lib.wx_comm_unique_id(buf))
        uid = bytes(buf)
    uid = broadcast_id(uid)
    buf = (C.c_uint8 * 128).from_buffer_copy(uid)
    ctx = context()
    check(lib.wx_ctx_init_comm(ctx.h, world, rank, buf), ctx.h)
    ctx.sp_size, ctx.sp_rank = world, rank


class H3DiTBlocks:
    """The block loop of H3DiT.forward (H3Transformer.swift:1078-1159) on libwx.

    ``mods[bi]`` = six [num_mod_rows, hidden] bf16 tables (shift/scale/gate MSA, shift/scale/gate MLP).
    With a sequence-parallel context (init_sequence_parallel) h, rowmap, cos/sin and the PAB
    slots are this rank's rows and ``S_total`` is the length of the whole sequence."""

    def __init__(self, cfg: H3DiTConfig, blocks: list[H3BlockWeights]):
        self.cfg = cfg
        self.blocks = blocks
        self._wc = [b.c() for b in blocks]
        # scratch for x at^T of the widest attached LoRA pack
        rank = max([lin.lora_pack().R for b in blocks for lin in b.linears() if lin.lora] or [0])
        self._c = cfg.c(int(rank))
        self._scratch: Optional[torch.Tensor] = None

    def scratch(self, S: int, device, P: int = 1) -> torch.Tensor:
        lib = _lib.load()
        need = int(lib.wx_dit_block_scratch_bytes(C.byref(self._c), S) if P == 1 else
                   lib.wx_dit_block_sp_scratch_bytes(C.byref(self._c), S, P))
        if need <= 0:
            raise WxError(_lib.WX_ERR_INVALID, f"no block plan for S={S} over {P} ranks")
        if self._scratch is None or self._scratch.numel() < need or self._scratch.device != torch.device(device):
            self._scratch = None
            self._scratch = torch.empty(need, dtype=torch.uint8, device=device)
        return self._scratch

    def block_forward(self, bi: int, h: torch.Tensor, mods: Sequence[torch.Tensor], rowmap: torch.Tensor,
                      cos: torch.Tensor, sin: torch.Tensor, spec: Optional[SparseSpec],
                      pab_slot: Optional[torch.Tensor] = None, refresh: bool = True,
                      S_total: Optional[int] = None) -> torch.Tensor:
        """One block, h [rows, hidden] updated in place."""
        _need_bf16_cuda(h, cos, sin, *mods)
        ctx = context(h.device.index)
        P = getattr(ctx, "sp_size", 1)
        bm = BlockMods(*[_p(m) for m in mods])
        sp = spec if spec is not None else dense_spec()
        if P == 1:
            S = h.shape[0]
            scr = self.scratch(S, h.device)
            ctx.call("wx_dit_block_forward", C.byref(self._c), C.byref(self._wc[bi]), C.byref(bm), _p(rowmap),
                     _p(h), S, _p(cos), _p(sin), C.byref(sp), _p(pab_slot), int(refresh), _p(scr))
        else:
            S = S_total if S_total is not None else h.shape[0] * P
            scr = self.scratch(S, h.device, P)
            ctx.call("wx_dit_block_forward_sp", C.byref(self._c), C.byref(self._wc[bi]), C.byref(bm), _p(rowmap),
                     _p(h), S, _p(cos), _p(sin), C.byref(sp), _p(pab_slot), int(refresh), _p(scr))
        return h

    def block_graph(self, bi: int, h: torch.Tensor, mods: Sequence[torch.Tensor], rowmap: torch.Tensor,
                    cos: torch.Tensor, sin: torch.Tensor, spec: Optional[SparseSpec],
                    pab_slot: Optional[torch.Tensor] = None, refresh: bool = True) -> "BlockGraph":
        """block_forward of block bi on exactly these buffers, captured as a CUDA graph
        (wx_dit_block_graph_create); BlockGraph.launch() replays it (single GPU)."""
        return BlockGraph(self, bi, h, mods, rowmap, cos, sin, spec, pab_slot, refresh)

    def forward(self, h: torch.Tensor, mods: Sequence[Sequence[torch.Tensor]], rowmap: torch.Tensor,
                cos: torch.Tensor, sin: torch.Tensor, sparse_cfg: Optional[H3SolAttnConfig], g: int,
                policy: int = SparsePolicy.MIX, attn_bcast: Optional[H3AttnBroadcast] = None,
                attn_refresh: bool = True, sigma: Optional[float] = None,
                S_total: Optional[int] = None) -> torch.Tensor:
        """All blocks in order; the PAB slot of block bi is written on refresh, read on reuse."""
        n = len(self.blocks)
        for bi in range(n):
            mode = sparse_mode_for_layer(bi, n, policy) if sparse_cfg is not None else 0
            spec = sparse_cfg.spec(g) if mode != 0 else None
            slot = None
            refresh = True
            if attn_bcast is not None:
                cached = attn_bcast.blocks[bi]
                refresh = attn_refresh or cached is None
                slot = attn_bcast.slot(bi, h.shape[0], self.cfg.hidden, h.device)
            self.block_forward(bi, h, mods[bi], rowmap, cos, sin, spec, slot, refresh, S_total=S_total)
        if attn_bcast is not None and attn_refresh and sigma is not None:
            attn_bcast.cached_sigma = sigma
        return h


class BlockGraph:
    """One block forward captured as a CUDA graph (wx_dit_block_graph_create) and replayed
    by launch() (wx_graph_launch) on the current stream. The graph holds the buffers'
    addresses: this object keeps the tensors alive, owns its own scratch, and the caller
    refreshes the contents (h is updated in place by each replay)."""

    def __init__(self, blocks: "H3DiTBlocks", bi: int, h: torch.Tensor, mods: Sequence[torch.Tensor],
                 rowmap: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, spec: Optional[SparseSpec],
                 pab_slot: Optional[torch.Tensor], refresh: bool):
        _need_bf16_cuda(h, cos, sin, *mods)
        ctx = context(h.device.index)
        if getattr(ctx, "sp_size", 1) != 1:
            raise WxError(_lib.WX_ERR_UNSUPPORTED, "block graphs are single-GPU")
        S = h.shape[0]
        need = int(ctx.lib.wx_dit_block_scratch_bytes(C.byref(blocks._c), S))
        self._scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=h.device)
        self._keep = (blocks, h, list(mods), rowmap, cos, sin, pab_slot)
        bm = BlockMods(*[_p(m) for m in mods])
        sp = spec if spec is not None else dense_spec()
        self._ctx = ctx
        self._g = C.c_void_p()
        ctx.call("wx_dit_block_graph_create", C.byref(blocks._c), C.byref(blocks._wc[bi]), C.byref(bm), _p(rowmap),
                 _p(h), S, _p(cos), _p(sin), C.byref(sp), _p(pab_slot), int(refresh), _p(self._scratch),
                 C.byref(self._g))

    def launch(self) -> None:
        self._ctx.call("wx_graph_launch", self._g)

    def kernels(self) -> int:
        return int(self._ctx.lib.wx_graph_kernels(self._g))

    def close(self) -> None:
        if self._g is not None and self._g.value:
            self._ctx.sync_stream()
            torch.cuda.current_stream(self._scratch.device).synchronize()
            self._ctx.lib.wx_graph_destroy(self._g)
        self._g = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class H3AudioRows:
    """Audio rows of one sampler step: packed-row segments [start, end) (refAudio and the
    target audio segment of the PackedLayout, ascending, before the video), their fp32 latents
    [rows, audio_dim] in segment order, the index of the denoised segment (-1 none), this step's
    audio row of the final AdaLN tables, and the update factors: out.audio = aout * vscale with
    vscale = -slope (H3DiT.forward, H3Transformer.swift:1186-1188), audioX += out.audio * dsigma
    with dsigma = dσa / slope (H3Pipeline.swift:1438-1442)."""
    segs: Sequence[tuple]
    latents: torch.Tensor
    target: int
    final_shift: Optional[torch.Tensor]
    final_scale: Optional[torch.Tensor]
    vscale: float
    dsigma: float


class H3DiT:
    """H3DiT (H3Transformer.swift:1022-1203) around the blocks: patch embed, final head,
    and the sampler step of H3Pipeline.swift:1398-1445 as one native call (wx_dit_step);
    optional audio patch embed / audio head (audioPatchW/B, audioOutW/B)."""

    def __init__(self, blocks: H3DiTBlocks, mods: Sequence[Sequence[torch.Tensor]], embed_w: torch.Tensor,
                 embed_b: torch.Tensor, final_norm: torch.Tensor, out_w: torch.Tensor, out_b: torch.Tensor,
                 audio_embed_w: Optional[torch.Tensor] = None, audio_embed_b: Optional[torch.Tensor] = None,
                 audio_out_w: Optional[torch.Tensor] = None, audio_out_b: Optional[torch.Tensor] = None):
        self.blocks = blocks
        self.mods = [list(m) for m in mods]
        self._bw = (BlockWeights * len(blocks.blocks))(*blocks._wc)
        self._bm = (BlockMods * len(self.mods))(*[BlockMods(*[_p(t) for t in m]) for m in self.mods])
        self.embed_w, self.embed_b, self.final_norm, self.out_w, self.out_b = embed_w, embed_b, final_norm, out_w, out_b
        self.audio = (audio_embed_w, audio_embed_b, audio_out_w, audio_out_b)
        self.patch_dim = embed_w.shape[0]
        audio_dim = audio_embed_w.shape[0] if audio_embed_w is not None else 0
        self._m = _lib.DitModel(C.pointer(blocks._c), len(blocks.blocks), self.patch_dim, self._bw, self._bm,
                                _p(embed_w), _p(embed_b), _p(final_norm), _p(out_w), _p(out_b), audio_dim,
                                _p(audio_embed_w), _p(audio_embed_b), _p(audio_out_w), _p(audio_out_b))
        self._scratch: Optional[torch.Tensor] = None

    def step(self, S: int, text_rows: int, video_start: int, text_states: torch.Tensor, latents: torch.Tensor,
             rowmap: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, final_shift: torch.Tensor,
             final_scale: torch.Tensor, sparse_cfg: Optional[H3SolAttnConfig], policy: int,
             attn_bcast: Optional[H3AttnBroadcast], attn_refresh: bool, dsigma: float,
             sigma: Optional[float] = None, audio: Optional[H3AudioRows] = None,
             text_states_neg: Optional[torch.Tensor] = None, cfg_scale: float = 0.0, update: bool = True,
             velocity_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One denoising step; latents [S - text_rows (- audio rows), patch] fp32 (and the audio
        latents) are updated in place. With text_states_neg (and cfg_scale > 0) the step is the
        SelfLift CFG step (SelfLiftH3-(h3专属).swift:826-845): a second forward on the negative
        condition without the PAB cache and v = v_neg + cfg·(v_pos − v_neg). update=False leaves
        the latents untouched; velocity_out receives the video output (the negated velocity)."""
        ctx = context(latents.device.index)
        lib = ctx.lib
        guided = (text_states_neg is not None and cfg_scale > 0) or not update or velocity_out is not None
        if guided:
            need = int(lib.wx_dit_step_guided_scratch_bytes(ctx.h, C.byref(self._m), S))
        else:
            need = int(lib.wx_dit_step_scratch_bytes(ctx.h, C.byref(self._m), S))
        if need <= 0:
            raise WxError(_lib.WX_ERR_INVALID, f"no step plan for S={S}")
        if self._scratch is None or self._scratch.numel() < need:
            self._scratch = None
            self._scratch = torch.empty(need, dtype=torch.uint8, device=latents.device)
        slots = None
        rows = S // getattr(ctx, "sp_size", 1)
        refresh = attn_refresh
        if attn_bcast is not None:
            refresh = attn_refresh or any(b is None for b in attn_bcast.blocks)
            ptrs = [attn_bcast.slot(bi, rows, self.blocks.cfg.hidden, latents.device).data_ptr()
                    for bi in range(len(self.blocks.blocks))]
            slots = (C.c_void_p * len(ptrs))(*ptrs)
        spec = sparse_cfg.spec(video_start) if sparse_cfg is not None else None
        args = _lib.StepArgs(S, text_rows, video_start, _p(text_states), _p(latents), _p(rowmap), _p(cos), _p(sin),
                             _p(final_shift), _p(final_scale), C.pointer(spec) if spec is not None else None,
                             policy if sparse_cfg is not None else SparsePolicy.OFF, int(refresh), slots,
                             float(dsigma), 0, _p(self._scratch))
        if audio is not None:
            segs = (C.c_int64 * (2 * max(1, len(audio.segs))))(*[int(v) for sg in audio.segs for v in sg])
            args.audio_segs = C.cast(segs, C.c_void_p)
            args.n_audio_segs = len(audio.segs)
            args.audio_target = audio.target
            args.audio_latents = _p(audio.latents)
            args.audio_final_shift = _p(audio.final_shift)
            args.audio_final_scale = _p(audio.final_scale)
            args.audio_vscale = float(audio.vscale)
            args.audio_dsigma = float(audio.dsigma)
        else:
            args.audio_target = -1
        # WX_H3PROF set: per-layer phase lines after the step, as the reference's NA_H3PROF prints them
        prof = bool(os.environ.get("WX_H3PROF"))
        if prof:
            ctx.trace(True)
        if guided:
            g = _lib.Guidance(_p(text_states_neg) if cfg_scale > 0 else None, float(cfg_scale), int(bool(update)),
                              _p(velocity_out))
            ctx.call("wx_dit_step_guided", C.byref(self._m), C.byref(args), C.byref(g))
        else:
            ctx.call("wx_dit_step", C.byref(self._m), C.byref(args))
        if prof:
            print(Context.format_trace(ctx.trace_read()), flush=True)
            ctx.trace(False)
        if attn_bcast is not None and refresh and sigma is not None:
            attn_bcast.cached_sigma = sigma
        return latents


# ------------------------------------------------------------------- RoPE and positions
def axis_from_sqrt_area(dim: int, patch: int, sqrt_area: float) -> list[float]:
    """axisFromSqrtArea (H3Layout.swift:188-194)."""
    lib = _lib.load()
    n = lib.wx_axis_from_sqrt_area(dim, patch, float(sqrt_area), None, 0)
    check(min(n, 0))
    out = (C.c_double * max(n, 1))()
    check(min(lib.wx_axis_from_sqrt_area(dim, patch, float(sqrt_area), out, n), 0))
    return list(out)[:n]


def video_t_span(k: int) -> float:
    """videoTSpan (H3Layout.swift:197-200)."""
    return float(_lib.load().wx_video_t_span(k))


def video_t_grid(n: int, origin: float) -> list[float]:
    """videoTGrid (H3Layout.swift:202-210)."""
    out = (C.c_double * max(n, 1))()
    check(_lib.load().wx_video_t_grid(n, float(origin), out))
    return list(out)[:n]


def write_frame_grid(pos: np.ndarray, row: int, t: float, h_axis: Sequence[float], w_axis: Sequence[float]) -> None:
    """writeFrameGrid (H3Layout.swift:683-694) into pos [S, 3] float64 (in place)."""
    if pos.dtype != np.float64 or not pos.flags.c_contiguous:
        raise WxError(_lib.WX_ERR_INVALID, "positions must be a C-contiguous float64 [S, 3] array")
    ha = (C.c_double * max(len(h_axis), 1))(*h_axis)
    wa = (C.c_double * max(len(w_axis), 1))(*w_axis)
    if row + len(h_axis) * len(w_axis) > pos.shape[0]:
        raise WxError(_lib.WX_ERR_INVALID, "frame grid runs past the end of the positions")
    check(_lib.load().wx_write_frame_grid(pos.ctypes.data, row, float(t), ha, len(h_axis), wa, len(w_axis)))


def packed_positions(text_len: int, ref_images: Sequence[tuple], latent_t: int, latent_h: int,
                     latent_w: int) -> np.ndarray:
    """positionIds of PackedLayout (H3Layout.swift:336-650) for a layout of text, reference
    images (ref2va image blocks) and the target video, without audio, keyframes or
    continuation rows: text rows t = 0..L-1 (:409-411); each image block a frame grid at
    the cursor, cursor += 1 (:524-537); the target video's frames at videoTGrid(latent_t,
    cursor) (:638-643). ref_images: (latent_h, latent_w) per image. Returns [S, 3] float64."""
    def grid(lh, lw):
        area = math.sqrt(float(lh) * float(lw))
        return axis_from_sqrt_area(lh, 2, area), axis_from_sqrt_area(lw, 2, area)
    grids = [grid(h, w) for h, w in ref_images]
    vh, vw = grid(latent_h, latent_w)
    frame_rows = len(vh) * len(vw)
    S = text_len + sum(len(a) * len(b) for a, b in grids) + latent_t * frame_rows
    pos = np.zeros((S, 3), dtype=np.float64)
    pos[:text_len, 0] = np.arange(text_len, dtype=np.float64)
    row, cursor = text_len, float(text_len)
    for ha, wa in grids:
        write_frame_grid(pos, row, cursor, ha, wa)
        row += len(ha) * len(wa)
        cursor += 1.0
    for f, tv in enumerate(video_t_grid(latent_t, cursor)):
        write_frame_grid(pos, row + f * frame_rows, tv, vh, vw)
    return pos


def build_rope(positions: np.ndarray, inv_freq: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """buildRope (H3Layout.swift:725-740): positions [S, 3] (host, cast to fp32 as the reference
    does) and inv_freq [nf] fp32 on the GPU -> cos, sin [S, 3*nf] bf16."""
    if not inv_freq.is_cuda or inv_freq.dtype != torch.float32:
        raise WxError(_lib.WX_ERR_INVALID, "inv_freq must be a CUDA fp32 tensor")
    dev = inv_freq.device
    pos = torch.from_numpy(np.ascontiguousarray(positions, dtype=np.float32)).to(dev)
    S, nf = pos.shape[0], inv_freq.numel()
    cos = torch.empty((S, 3 * nf), dtype=torch.bfloat16, device=dev)
    sin = torch.empty_like(cos)
    context(dev.index).call("wx_build_rope", _p(pos), S, _p(inv_freq.contiguous()), nf, _p(cos), _p(sin))
    return cos, sin


# ------------------------------------------------------------ conditioning (per generation)
class DenseLinear:
    """The dense branch of MfLinear (H3Common.swift:304-308, 361-366): ``w`` [in, out] bf16
    stored pre-transposed, optional ``bias`` [out]; forward = bf16(bf16(x w) + bias)."""

    def __init__(self, w: torch.Tensor, bias: Optional[torch.Tensor] = None):
        _need_bf16_cuda(w, bias)
        self.w, self.bias = w.contiguous(), bias
        self.in_dim, self.out_dim = w.shape

    def c(self) -> _lib.DenseBf16:
        return _lib.DenseBf16(_p(self.w), _p(self.bias), self.in_dim, self.out_dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _need_bf16_cuda(x)
        x2 = x.reshape(-1, self.in_dim).contiguous()
        y = torch.empty((x2.shape[0], self.out_dim), dtype=torch.bfloat16, device=x.device)
        dw = self.c()
        context(x.device.index).call("wx_linear_bf16", _p(x2), x2.shape[0], C.byref(dw), _p(y))
        return y.reshape(*x.shape[:-1], self.out_dim)

    __call__ = forward


class H3TimeEmbedder:
    """H3TimeEmbedder (H3Transformer.swift:255-302), the fp32 island: sinusoid of the
    timesteps → proj_in → SiLU → proj_out. Weights fp32 [in, out] as the reference stores them."""

    def __init__(self, input_dim: int, out_dim: int, proj_in_w: torch.Tensor, proj_in_b: Optional[torch.Tensor],
                 proj_out_w: torch.Tensor, proj_out_b: Optional[torch.Tensor]):
        for t in (proj_in_w, proj_in_b, proj_out_w, proj_out_b):
            if t is not None and (not t.is_cuda or t.dtype != torch.float32):
                raise WxError(_lib.WX_ERR_INVALID, "time embedder weights must be CUDA fp32 tensors")
        self.input_dim, self.out_dim = input_dim, out_dim
        self.proj_in_w, self.proj_in_b = proj_in_w.contiguous(), proj_in_b
        self.proj_out_w, self.proj_out_b = proj_out_w.contiguous(), proj_out_b

    def forward(self, t_vals: Sequence[float]) -> torch.Tensor:
        """t_vals → [m, out_dim] fp32 (the caller casts to bf16, as precomputeAdaln does)."""
        m = len(t_vals)
        ts = (C.c_double * m)(*[float(t) for t in t_vals])
        out = torch.empty((m, self.out_dim), dtype=torch.float32, device=self.proj_in_w.device)
        context(out.device.index).call("wx_time_embed", ts, m, self.input_dim, _p(self.proj_in_w),
                                       _p(self.proj_in_b), self.out_dim, _p(self.proj_out_w), _p(self.proj_out_b),
                                       _p(out))
        return out

    __call__ = forward


class H3AdalnLUT:
    """H3AdalnLUT (H3Transformer.swift:319-350): lookup-table time modulation of pruned /
    fused checkpoints; ``t_table`` [n, rank] fp32 (basis and mean are kept for reference only)."""

    def __init__(self, basis: Optional[torch.Tensor], mean: Optional[torch.Tensor], t_table: torch.Tensor):
        if not t_table.is_cuda or t_table.dtype != torch.float32:
            raise WxError(_lib.WX_ERR_INVALID, "adaln_t_table must be a CUDA fp32 tensor")
        self.basis, self.mean, self.t_table = basis, mean, t_table.contiguous()
        self.rank = t_table.shape[1]

    def coeffs(self, ts: Sequence[float]) -> torch.Tensor:
        """coeffs(ts).asType(bf16): [m, rank] rows round(t·(n-1)) of the table."""
        m = len(ts)
        arr = (C.c_double * m)(*[float(t) for t in ts])
        out = torch.empty((m, self.rank), dtype=torch.bfloat16, device=self.t_table.device)
        context(out.device.index).call("wx_adaln_lut_coeffs", arr, m, _p(self.t_table), self.t_table.shape[0],
                                       self.rank, _p(out))
        return out


class H3AdalnW:
    """H3AdalnW (H3Transformer.swift:353-404): ``linear`` (quantized MfLinear, optionally with
    LoRA, or DenseLinear for folded LUT checkpoints) [time_embed_dim → expand·modalities·hidden];
    forward splits it into ``expand`` tables of [m·modalities, hidden]."""

    def __init__(self, linear, expand: int, modalities: int):
        self.linear, self.expand, self.modalities = linear, expand, modalities

    def forward(self, t_emb: torch.Tensor, apply_silu: bool = True) -> list[torch.Tensor]:
        _need_bf16_cuda(t_emb)
        t_emb = t_emb.contiguous()
        m, k = t_emb.shape
        n = self.linear.out_dim
        hidden = n // (self.expand * self.modalities)
        tabs = [torch.empty((m * self.modalities, hidden), dtype=torch.bfloat16, device=t_emb.device)
                for _ in range(self.expand)]
        ptrs = (C.c_void_p * self.expand)(*[t.data_ptr() for t in tabs])
        qw = pack = dw = None
        if isinstance(self.linear, MfLinear):
            qw = self.linear.qweight()
            pack = self.linear.lora_pack()
        else:
            dw = self.linear.c()
        context(t_emb.device.index).call("wx_adaln_tables", _p(t_emb), m, k, int(apply_silu),
                                         C.byref(qw) if qw is not None else None,
                                         C.byref(pack) if pack is not None else None,
                                         C.byref(dw) if dw is not None else None, self.expand, self.modalities, ptrs)
        return tabs

    __call__ = forward


@dataclass
class H3AdalnTables:
    """H3AdalnTables (H3Transformer.swift:406-411)."""
    ts: list
    blocks: list  # [layer][6] each [t·modalities, hidden]
    final: list   # [2] each [t, hidden]


def precompute_adaln(ts: Sequence[float], block_adalns: Sequence[Optional[H3AdalnW]],
                     final_adaln: Optional[H3AdalnW], hidden: int, embedder: Optional[H3TimeEmbedder] = None,
                     lut: Optional[H3AdalnLUT] = None, device=None) -> H3AdalnTables:
    """H3DiT.precomputeAdaln (H3Transformer.swift:957-988): the t-embedding (LUT coefficients,
    no SiLU; or the time embedder, SiLU in the adaln forward) folded into every block's six
    tables and the final layer's two. Absent (ablated) block modulation gives zero tables
    (the reference allocates them with ts.count rows; here they get ts.count·3 rows so that
    every mod row a plan can address exists — the values are the same zeros)."""
    if lut is not None:
        t_emb, apply_silu = lut.coeffs(ts), False
    elif embedder is not None:
        t_emb, apply_silu = embedder(ts), True
        src = t_emb
        t_emb = torch.empty(src.shape, dtype=torch.bfloat16, device=src.device)
        context(src.device.index).call("wx_f32_to_bf16", _p(src), src.numel(), _p(t_emb))
    else:
        raise WxError(_lib.WX_ERR_INVALID, "precompute_adaln needs the time embedder or the LUT")
    dev = t_emb.device if device is None else device
    blocks = []
    for ad in block_adalns:
        if ad is None:
            zero = torch.zeros((len(ts) * 3, hidden), dtype=torch.bfloat16, device=dev)
            blocks.append([zero] * 6)
        else:
            blocks.append(ad(t_emb, apply_silu))
    final = final_adaln(t_emb, apply_silu) if final_adaln is not None else []
    return H3AdalnTables(list(ts), blocks, final)


class H3TextRefiner:
    """H3DiT.refineText (H3Transformer.swift:993-1016) on libwx: condition_proj [text_dim →
    hidden], the token-refiner blocks (H3RefinerBlockW, :676-700; same weight set as a DiT
    block, used without modulation or RoPE, dense attention), then the final RMSNorm.
    Text states already ``hidden`` wide come back unchanged, as in the reference."""

    def __init__(self, cfg: H3DiTConfig, condition_proj: Optional[MfLinear], blocks: Sequence[H3BlockWeights],
                 final_norm: Optional[torch.Tensor]):
        self.cfg = cfg
        self.condition_proj = condition_proj
        self.blocks = list(blocks)
        self.final_norm = final_norm
        self._wc = [b.c() for b in self.blocks]
        lins = [lin for b in self.blocks for lin in b.linears()] + ([condition_proj] if condition_proj else [])
        rank = max([lin.lora_pack().R for lin in lins if lin.lora] or [0])
        self._c = cfg.c(int(rank))
        self._bw = (BlockWeights * max(1, len(self._wc)))(*self._wc)

    def block_forward(self, bi: int, h: torch.Tensor) -> torch.Tensor:
        """One refiner block, h [L, hidden] updated in place."""
        _need_bf16_cuda(h)
        lib = _lib.load()
        L = h.shape[0]
        need = int(lib.wx_refiner_scratch_bytes(C.byref(self._c), L))
        scr = torch.empty(need, dtype=torch.uint8, device=h.device)
        context(h.device.index).call("wx_refiner_block_forward", C.byref(self._c), C.byref(self._wc[bi]), _p(h), L,
                                     _p(scr))
        return h

    def forward(self, text_states: torch.Tensor) -> torch.Tensor:
        _need_bf16_cuda(text_states, self.final_norm)
        x = text_states.contiguous()
        L, text_dim = x.shape
        lib = _lib.load()
        out = torch.empty((L, self.cfg.hidden), dtype=torch.bfloat16, device=x.device)
        need = int(lib.wx_refine_text_scratch_bytes(C.byref(self._c), L, text_dim))
        scr = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        qw = self.condition_proj.qweight() if self.condition_proj is not None else None
        pack = self.condition_proj.lora_pack() if self.condition_proj is not None else None
        context(x.device.index).call("wx_refine_text", C.byref(self._c), C.byref(qw) if qw is not None else None,
                                     C.byref(pack) if pack is not None else None, self._bw, len(self._wc),
                                     _p(self.final_norm), _p(x), L, text_dim, _p(out), _p(scr))
        return out

    __call__ = forward


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """rmsNormLast (H3Common.swift:502-508) over the last axis."""
    _need_bf16_cuda(x, weight)
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    out = torch.empty_like(x2)
    context(x.device.index).call("wx_rms_norm", _p(x2), x2.shape[0], x2.shape[1], _p(weight), float(eps), _p(out))
    return out.reshape(x.shape)


# ------------------------------------------------------------------------ checkpoints
_ST_DTYPES = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32, "I32": torch.int32,
              "U32": torch.int32, "I64": torch.int64, "U8": torch.uint8, "I8": torch.int8, "BOOL": torch.bool}


class H3Weights:
    """H3Weights (H3Common.swift:180-261): a memory-mapped safetensors file whose tensors are
    copied to the GPU on demand (wx_st_*). U32 tensors come back as int32 (same bits)."""

    def __init__(self, path: str):
        self._lib = _lib.load()
        h = C.c_void_p()
        st = self._lib.wx_st_open(str(path).encode(), C.byref(h))
        if st != 0:
            raise WxError(st, self._lib.wx_st_last_error().decode(errors="replace"))
        self._h = h
        self.path = str(path)

    def close(self) -> None:
        if self._h:
            self._lib.wx_st_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def keys(self) -> list[str]:
        n = self._lib.wx_st_count(self._h)
        return [self._lib.wx_st_name(self._h, i).decode() for i in range(n)]

    def info(self, key: str) -> Optional[StInfo]:
        inf = StInfo()
        return inf if self._lib.wx_st_find(self._h, key.encode(), C.byref(inf)) == 0 else None

    def contains(self, key: str) -> bool:
        return self.info(key) is not None

    def _upload(self, key: str, inf: StInfo, device) -> torch.Tensor:
        dt = _ST_DTYPES.get(inf.dtype.decode())
        if dt is None:
            raise WxError(_lib.WX_ERR_UNSUPPORTED, f"{key}: dtype {inf.dtype.decode()} not supported")
        shape = [inf.shape[i] for i in range(inf.ndim)]
        t = torch.empty(shape, dtype=dt, device=device)
        context(t.device.index).call("wx_st_upload", self._h, key.encode(), _p(t), t.numel() * t.element_size())
        return t

    def get(self, key: str, device=None) -> Optional[torch.Tensor]:
        """H3Weights.get (:229-235): the tensor on the GPU, or None when absent."""
        inf = self.info(key)
        if inf is None:
            return None
        return self._upload(key, inf, device if device is not None else torch.device("cuda", torch.cuda.current_device()))

    def get_linear(self, prefix: str, in_features: int, device=None) -> MfLinear:
        """MfLinear.load (H3Common.swift:311-338) of a quantized linear; either naming variant
        of the triple (getQuantized, :243-258)."""
        infos = [StInfo() for _ in range(4)]
        bits, group = C.c_int32(), C.c_int32()
        st = self._lib.wx_st_find_qlinear(self._h, prefix.encode(), in_features, *[C.byref(i) for i in infos],
                                          C.byref(bits), C.byref(group))
        if st != 0:
            raise WxError(st, self._lib.wx_st_last_error().decode(errors="replace"))
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        names = [prefix + ".weight"]
        for suf in (".scales", ".biases"):
            names.append(prefix + suf if self.contains(prefix + suf) else prefix + ".weight" + suf)
        w, sc, bi = [self._upload(n, i, dev) for n, i in zip(names, infos[:3])]
        bias = self._upload(prefix + ".bias", infos[3], dev) if infos[3].dtype else None
        if sc.dtype != torch.bfloat16:
            sc, bi = sc.to(torch.bfloat16), bi.to(torch.bfloat16)
        if bias is not None and bias.dtype != torch.bfloat16:
            bias = bias.to(torch.bfloat16)
        return MfLinear(w, sc, bi, in_features, bias)


def load_block(w: H3Weights, idx: int, cfg: H3DiTConfig, device=None) -> H3BlockWeights:
    """H3DiTBlock.load (H3Transformer.swift:648-660): blocks.{idx}.{norm1,norm2}.weight,
    attn.{qkv_proj,q_norm,k_norm,out_proj}, mlp.{fc1,fc2}."""
    p = f"blocks.{idx}"
    inner = cfg.heads * cfg.head_dim

    def need(key):
        t = w.get(key, device)
        if t is None:
            raise WxError(_lib.WX_ERR_INVALID, f"missing weight: {key}")
        return t.to(torch.bfloat16) if t.dtype != torch.bfloat16 else t
    return H3BlockWeights(w.get_linear(p + ".attn.qkv_proj", cfg.hidden, device),
                          w.get_linear(p + ".attn.out_proj", inner, device),
                          w.get_linear(p + ".mlp.fc1", cfg.hidden, device),
                          w.get_linear(p + ".mlp.fc2", cfg.ffn, device),
                          need(p + ".attn.q_norm.weight"), need(p + ".attn.k_norm.weight"),
                          need(p + ".norm1.weight"), need(p + ".norm2.weight"))


def _need_bf16(w: H3Weights, key: str, device=None) -> torch.Tensor:
    t = w.get(key, device)
    if t is None:
        raise WxError(_lib.WX_ERR_INVALID, f"missing weight: {key}")
    return t.to(torch.bfloat16) if t.dtype != torch.bfloat16 else t


def load_refiner_block(w: H3Weights, idx: int, cfg: H3DiTConfig, device=None) -> H3BlockWeights:
    """H3RefinerBlockW.load (H3Transformer.swift:690-699): token_refiner.blocks.{idx}.*"""
    p = f"token_refiner.blocks.{idx}"
    inner = cfg.heads * cfg.head_dim
    return H3BlockWeights(w.get_linear(p + ".attn.qkv_proj", cfg.hidden, device),
                          w.get_linear(p + ".attn.out_proj", inner, device),
                          w.get_linear(p + ".mlp.fc1", cfg.hidden, device),
                          w.get_linear(p + ".mlp.fc2", cfg.ffn, device),
                          _need_bf16(w, p + ".attn.q_norm.weight", device),
                          _need_bf16(w, p + ".attn.k_norm.weight", device),
                          _need_bf16(w, p + ".norm1.weight", device), _need_bf16(w, p + ".norm2.weight", device))


def load_text_refiner(w: H3Weights, cfg: H3DiTConfig, text_dim: int, device=None) -> H3TextRefiner:
    """The text-side weights of H3DiT.load (H3Transformer.swift:792-807): condition_proj
    when present, token_refiner.blocks.0.. while their qkv_proj exists, and
    token_refiner.final_norm.weight when present."""
    cp = w.get_linear("condition_proj", text_dim, device) if w.contains("condition_proj.weight") else None
    blocks = []
    while (w.contains(f"token_refiner.blocks.{len(blocks)}.attn.qkv_proj.weight")
           or w.contains(f"token_refiner.blocks.{len(blocks)}.attn.qkv_proj.scales")):
        blocks.append(load_refiner_block(w, len(blocks), cfg, device))
    fn = w.get("token_refiner.final_norm.weight", device)
    if fn is not None and fn.dtype != torch.bfloat16:
        fn = fn.to(torch.bfloat16)
    return H3TextRefiner(cfg, cp, blocks, fn)


def load_time_embedder(w: H3Weights, input_dim: int = 256, out_dim: int = 2688, device=None) -> H3TimeEmbedder:
    """H3TimeEmbedder.load (H3Transformer.swift:274-286); weights kept fp32 [in, out]."""
    def f32(key):
        t = w.get(key, device)
        return None if t is None else (t if t.dtype == torch.float32 else t.to(torch.float32))
    win, wout = f32("time_embedder.proj_in.weight"), f32("time_embedder.proj_out.weight")
    if win is None or wout is None:
        raise WxError(_lib.WX_ERR_INVALID, "missing weight: time_embedder.proj_in.weight / proj_out.weight")
    return H3TimeEmbedder(input_dim, out_dim, win, f32("time_embedder.proj_in.bias"), wout,
                          f32("time_embedder.proj_out.bias"))


def load_adaln(w: H3Weights, prefix: str, time_embed_dim: int, expand: int, modalities: int,
               device=None) -> H3AdalnW:
    """H3AdalnW.load (H3Transformer.swift:366-382): {prefix}.linear quantized (in =
    time_embed_dim), or dense [out, in] stored transposed to [in, out] as MfLinear.load does."""
    if w.contains(prefix + ".linear.scales") or w.contains(prefix + ".linear.weight.scales"):
        return H3AdalnW(w.get_linear(prefix + ".linear", time_embed_dim, device), expand, modalities)
    raw = w.get(prefix + ".linear.weight", device)
    if raw is None:
        raise WxError(_lib.WX_ERR_INVALID, f"missing weight: {prefix}.linear.weight")
    bias = w.get(prefix + ".linear.bias", device)
    wt = raw.to(torch.bfloat16).t().contiguous()  # raw [out, in] -> [in, out]
    return H3AdalnW(DenseLinear(wt, bias.to(torch.bfloat16) if bias is not None else None), expand, modalities)
