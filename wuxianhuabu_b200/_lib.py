"""ctypes binding of libwx.so (the C ABI declared in include/wx_api.h).

The shared library is loaded from the package directory only; there is no
fallback implementation. Every call is checked: a non-zero wx_status raises
``WxError`` carrying ``wx_last_error``.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
# WX_LIB_VARIANT=checked loads the bounds-checked build of the same sources
LIB_PATH = _PKG / ("libwx_checked.so" if os.environ.get("WX_LIB_VARIANT") == "checked" else "libwx.so")

WX_OK = 0
WX_ERR_INVALID = -1
WX_ERR_CUDA = -2
WX_ERR_NOMEM = -3
WX_ERR_DEVICE = -4
WX_ERR_UNSUPPORTED = -5

EPI_NONE, EPI_GELU, EPI_GATE_RESID, EPI_SWIGLU = 0, 1, 2, 3
SPARSE_DENSE, SPARSE_SOL, SPARSE_TOPK = 0, 1, 2
MLP_GELU, MLP_SWIGLU = 0, 1


class WxError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"wx status {status}: {msg}")
        self.status = status


class QWeight(C.Structure):
    _fields_ = [("wq", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p), ("bias", C.c_void_p),
                ("n", C.c_int64), ("k", C.c_int64), ("group", C.c_int32), ("bits", C.c_int32)]


class SparseSpec(C.Structure):
    _fields_ = [("mode", C.c_int32), ("block", C.c_int32), ("g", C.c_int64), ("tau", C.c_float),
                ("density", C.c_float), ("sink_start", C.c_int32), ("sink_end", C.c_int32),
                ("tail", C.c_int32), ("reserved", C.c_int32)]


class StInfo(C.Structure):
    _fields_ = [("dtype", C.c_char * 8), ("ndim", C.c_int32), ("shape", C.c_int64 * 8), ("offset", C.c_uint64),
                ("nbytes", C.c_uint64), ("host", C.c_void_p)]


class Lora(C.Structure):
    _fields_ = [("a", C.c_void_p), ("b", C.c_void_p), ("r", C.c_int32), ("scale", C.c_float)]


class LoraPack(C.Structure):
    _fields_ = [("at", C.c_void_p), ("bt", C.c_void_p), ("R", C.c_int64), ("n", C.c_int64), ("k", C.c_int64)]


class BlockWeights(C.Structure):
    _fields_ = [("qkv", QWeight), ("out", QWeight), ("fc1", QWeight), ("fc2", QWeight),
                ("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("norm1", C.c_void_p), ("norm2", C.c_void_p),
                ("lora", C.POINTER(LoraPack) * 4)]


class DitConfig(C.Structure):
    _fields_ = [("hidden", C.c_int64), ("heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int64),
                ("mlp_kind", C.c_int32), ("rot", C.c_int32), ("eps", C.c_float), ("lora_rank", C.c_int32)]


class BlockMods(C.Structure):
    _fields_ = [("shift_msa", C.c_void_p), ("scale_msa", C.c_void_p), ("gate_msa", C.c_void_p),
                ("shift_mlp", C.c_void_p), ("scale_mlp", C.c_void_p), ("gate_mlp", C.c_void_p)]


class ModRun(C.Structure):
    _fields_ = [("start", C.c_uint32), ("end", C.c_uint32), ("mod_row", C.c_uint32)]


class SpPlan(C.Structure):
    _fields_ = [("S", C.c_int64), ("rows", C.c_int64), ("row0", C.c_int64), ("P", C.c_int32), ("rank", C.c_int32),
                ("H", C.c_int32), ("heads", C.c_int32), ("head0", C.c_int32), ("head_dim", C.c_int32),
                ("qkv_chunk", C.c_int64), ("out_chunk", C.c_int64)]


class DitModel(C.Structure):
    _fields_ = [("cfg", C.POINTER(DitConfig)), ("n_blocks", C.c_int32), ("patch_dim", C.c_int32),
                ("blocks", C.POINTER(BlockWeights)), ("mods", C.POINTER(BlockMods)), ("embed_w", C.c_void_p),
                ("embed_b", C.c_void_p), ("final_norm", C.c_void_p), ("out_w", C.c_void_p), ("out_b", C.c_void_p),
                ("audio_dim", C.c_int32), ("audio_embed_w", C.c_void_p), ("audio_embed_b", C.c_void_p),
                ("audio_out_w", C.c_void_p), ("audio_out_b", C.c_void_p)]


class StepArgs(C.Structure):
    _fields_ = [("S", C.c_int64), ("text_rows", C.c_int64), ("video_start", C.c_int64), ("text_states", C.c_void_p),
                ("latents", C.c_void_p), ("rowmap", C.c_void_p), ("cos_t", C.c_void_p), ("sin_t", C.c_void_p),
                ("final_shift", C.c_void_p), ("final_scale", C.c_void_p), ("spec", C.POINTER(SparseSpec)),
                ("policy", C.c_int32), ("refresh", C.c_int32), ("pab_slots", C.POINTER(C.c_void_p)),
                ("dsigma", C.c_float), ("reserved", C.c_int32), ("scratch", C.c_void_p),
                ("audio_segs", C.c_void_p), ("n_audio_segs", C.c_int32), ("audio_target", C.c_int32),
                ("audio_latents", C.c_void_p), ("audio_final_shift", C.c_void_p), ("audio_final_scale", C.c_void_p),
                ("audio_vscale", C.c_float), ("audio_dsigma", C.c_float)]


class Guidance(C.Structure):
    _fields_ = [("text_states_neg", C.c_void_p), ("cfg_scale", C.c_float), ("update", C.c_int32),
                ("velocity_out", C.c_void_p)]


class DenseBf16(C.Structure):
    _fields_ = [("w", C.c_void_p), ("bias", C.c_void_p), ("k", C.c_int64), ("n", C.c_int64)]


_vp, _i64, _i32, _f32, _f64, _u32 = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_double, C.c_uint32

# name -> (restype, argtypes)
_SIGS = {
    "wx_version": (_i32, []),
    "wx_ctx_create": (_i32, [_i32, C.POINTER(_vp)]),
    "wx_ctx_destroy": (_i32, [_vp]),
    "wx_ctx_set_stream": (_i32, [_vp, _vp]),
    "wx_last_error": (C.c_char_p, [_vp]),
    "wx_ctx_check_device": (_i32, [_vp]),
    "wx_ctx_workspace_bytes": (C.c_size_t, [_vp]),
    "wx_ctx_launch_count": (_i64, [_vp]),
    "wx_alloc": (_i32, [_vp, C.c_size_t, C.POINTER(_vp)]),
    "wx_free": (_i32, [_vp, _vp]),
    "wx_upload": (_i32, [_vp, _vp, _vp, C.c_size_t]),
    "wx_download": (_i32, [_vp, _vp, _vp, C.c_size_t]),
    "wx_ctx_synchronize": (_i32, [_vp]),
    "wx_dit_block_graph_create": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _i32, _vp,
                                          C.POINTER(_vp)]),
    "wx_graph_launch": (_i32, [_vp, _vp]),
    "wx_graph_kernels": (_i64, [_vp]),
    "wx_graph_destroy": (_i32, [_vp]),
    "wx_ctx_profile_enable": (_i32, [_vp, _i32]),
    "wx_ctx_profile_read": (_i32, [_vp, _vp, _vp, _i32]),
    "wx_ctx_trace_enable": (_i32, [_vp, _i32]),
    "wx_ctx_trace_read": (_i32, [_vp, _vp, _i32, C.POINTER(_i32)]),
    "wx_quantize_affine": (_i32, [_vp, _vp, _i64, _i64, _i32, _i32, _vp, _vp, _vp]),
    "wx_dequantize_affine": (_i32, [_vp, C.POINTER(QWeight), _vp]),
    "wx_qlinear": (_i32, [_vp, _vp, _i64, _i64, C.POINTER(QWeight), _i32, _vp, _vp, _vp, _vp, _i64, _vp]),
    "wx_lora_pack_bytes": (_i32, [_i64, _i64, C.POINTER(Lora), _i32, C.POINTER(_i64), C.POINTER(C.c_size_t),
                                  C.POINTER(C.c_size_t)]),
    "wx_lora_pack_build": (_i32, [_vp, _i64, _i64, C.POINTER(Lora), _i32, C.POINTER(LoraPack)]),
    "wx_qlinear_lora": (_i32, [_vp, _vp, _i64, _i64, C.POINTER(QWeight), C.POINTER(LoraPack), _i32, _vp, _vp, _vp,
                               _vp, _i64, _vp]),
    "wx_qkv_norm_rope": (_i32, [_vp, _vp, _i64, _i64, C.POINTER(QWeight), C.POINTER(LoraPack), _i32, _i32, _vp, _vp,
                                _vp, _vp, _i32, _f32, _vp, _i64]),
    "wx_qlinear_noalloc": (_i32, [_vp, _vp, _i64, _i64, C.POINTER(QWeight), _i32, _vp, _vp, _vp, _vp, _i64, _vp]),
    "wx_qlinear_noalloc_check": (_i32, [_vp]),
    "wx_qlinear_noalloc_last_error": (C.c_char_p, []),
    "wx_st_open": (_i32, [C.c_char_p, C.POINTER(_vp)]),
    "wx_st_close": (_i32, [_vp]),
    "wx_st_last_error": (C.c_char_p, []),
    "wx_st_count": (_i64, [_vp]),
    "wx_st_name": (C.c_char_p, [_vp, _i64]),
    "wx_st_find": (_i32, [_vp, C.c_char_p, C.POINTER(StInfo)]),
    "wx_st_upload": (_i32, [_vp, _vp, C.c_char_p, _vp, C.c_uint64]),
    "wx_st_find_qlinear": (_i32, [_vp, C.c_char_p, _i64, C.POINTER(StInfo), C.POINTER(StInfo), C.POINTER(StInfo),
                                  C.POINTER(StInfo), C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "wx_qk_norm_rope": (_i32, [_vp, _vp, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _i32, _f32, _vp, _i64]),
    "wx_qk_norm_rope_qkv": (_i32, [_vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _i32, _f32]),
    "wx_norm_modscale": (_i32, [_vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _f32, _vp]),
    "wx_mod_gate": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "wx_build_row_mod_map": (_i32, [C.POINTER(ModRun), _i32, _i64, _vp]),
    "wx_sol_route": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32, C.POINTER(SparseSpec), _f32,
                            _vp, _vp, _vp, _vp, _vp]),
    "wx_topk_route": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32, C.POINTER(SparseSpec), _f32,
                             _vp, _vp, _vp, _vp, _vp]),
    "wx_sparse_attention": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32, C.POINTER(SparseSpec), _f32,
                                   _vp, _i64]),
    "wx_attention_from_sel": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32, C.POINTER(SparseSpec), _f32,
                                     _vp, _vp, _vp, _vp, _vp, _i64]),
    "wx_pab_refresh": (_i32, [_i32, _u32, _u32]),
    "wx_pab_must_refresh": (_i32, [_f64, _f64, _f64]),
    "wx_pab_plan": (_i32, [_vp, _i32, _u32, _f64, _vp]),
    "wx_sigma_schedule": (_i32, [_u32, _f64, _vp]),
    "wx_sparse_mode_for_layer": (_i32, [_i32, _i32, _i32]),
    "wx_dit_block_scratch_bytes": (_i64, [C.POINTER(DitConfig), _i64]),
    "wx_dit_block_forward": (_i32, [_vp, C.POINTER(DitConfig), C.POINTER(BlockWeights), C.POINTER(BlockMods), _vp,
                                    _vp, _i64, _vp, _vp, C.POINTER(SparseSpec), _vp, _i32, _vp]),
    "wx_sp_make_plan": (_i32, [_i64, _i32, _i32, _i32, _i32, C.POINTER(SpPlan)]),
    "wx_comm_unique_id": (_i32, [_vp]),
    "wx_ctx_init_comm": (_i32, [_vp, _i32, _i32, _vp]),
    "wx_ctx_comm_check": (_i32, [_vp]),
    "wx_ctx_comm_abort": (_i32, [_vp]),
    "wx_ctx_sp_exchange": (_i32, [_vp]),
    "wx_ctx_set_peer_wait_limit": (_i32, [_vp, C.c_double]),
    "wx_ctx_signal_flags": (_i32, [_vp, _vp, _i32, C.c_uint32]),
    "wx_ctx_wait_flags": (_i32, [_vp, _vp, _i32, C.c_uint32]),
    "wx_dit_block_sp_scratch_bytes": (_i64, [C.POINTER(DitConfig), _i64, _i32]),
    "wx_dit_block_forward_sp": (_i32, [_vp, C.POINTER(DitConfig), C.POINTER(BlockWeights), C.POINTER(BlockMods),
                                       _vp, _vp, _i64, _vp, _vp, C.POINTER(SparseSpec), _vp, _i32, _vp]),
    "wx_dit_step_scratch_bytes": (_i64, [_vp, C.POINTER(DitModel), _i64]),
    "wx_dit_step": (_i32, [_vp, C.POINTER(DitModel), C.POINTER(StepArgs)]),
    "wx_dit_step_guided_scratch_bytes": (_i64, [_vp, C.POINTER(DitModel), _i64]),
    "wx_dit_step_guided": (_i32, [_vp, C.POINTER(DitModel), C.POINTER(StepArgs), C.POINTER(Guidance)]),
    "wx_dense_f32": (_i32, [_vp, _vp, _i64, _i64, _vp, _i64, _vp, _vp]),
    "wx_bf16_to_f32": (_i32, [_vp, _vp, _i64, _vp]),
    "wx_f32_to_bf16": (_i32, [_vp, _vp, _i64, _vp]),
    "wx_euler_update": (_i32, [_vp, _vp, _vp, _i64, _f32]),
    "wx_axis_from_sqrt_area": (_i32, [_u32, _u32, _f64, _vp, _i32]),
    "wx_video_t_span": (_f64, [_i32]),
    "wx_video_t_grid": (_i32, [_u32, _f64, _vp]),
    "wx_write_frame_grid": (_i32, [_vp, _i64, _f64, _vp, _i32, _vp, _i32]),
    "wx_build_rope": (_i32, [_vp, _vp, _i64, _vp, _i32, _vp, _vp]),
    "wx_linear_bf16": (_i32, [_vp, _vp, _i64, C.POINTER(DenseBf16), _vp]),
    "wx_time_embed": (_i32, [_vp, _vp, _i32, _i32, _vp, _vp, _i64, _vp, _vp, _vp]),
    "wx_adaln_lut_coeffs": (_i32, [_vp, _vp, _i32, _vp, _i64, _i32, _vp]),
    "wx_silu_bf16": (_i32, [_vp, _vp, _i64, _vp]),
    "wx_adaln_tables": (_i32, [_vp, _vp, _i64, _i64, _i32, C.POINTER(QWeight), C.POINTER(LoraPack),
                               C.POINTER(DenseBf16), _i32, _i32, _vp]),
    "wx_rms_norm": (_i32, [_vp, _vp, _i64, _i64, _vp, _f32, _vp]),
    "wx_refiner_scratch_bytes": (_i64, [C.POINTER(DitConfig), _i64]),
    "wx_refiner_block_forward": (_i32, [_vp, C.POINTER(DitConfig), C.POINTER(BlockWeights), _vp, _i64, _vp]),
    "wx_refine_text_scratch_bytes": (_i64, [C.POINTER(DitConfig), _i64, _i64]),
    "wx_refine_text": (_i32, [_vp, C.POINTER(DitConfig), C.POINTER(QWeight), C.POINTER(LoraPack),
                              C.POINTER(BlockWeights), _i32, _vp, _vp, _i64, _i64, _vp, _vp]),
}

_lib = None


def load() -> C.CDLL:
    """Load libwx.so (raises if it has not been built: there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() (no CPU fallback exists)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(status: int, ctx=None) -> None:
    if status != WX_OK:
        msg = ""
        if ctx is not None:
            raw = load().wx_last_error(ctx)
            msg = raw.decode() if raw else ""
        raise WxError(status, msg)
