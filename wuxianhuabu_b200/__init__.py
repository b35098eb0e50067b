"""wuxianhuabu_b200 — B200 (sm_100a) implementation of the MiniMax-H3 video-DiT
denoising step of HuaChayu/wuxianhuabu: 6-bit MLX-affine quantized linears on
tcgen05 tensor cores, SOL block-sparse flash attention, fused QK-RMSNorm+RoPE
and the PAB attention-broadcast cache, behind the C ABI of include/wx_api.h.
"""
from ._lib import LIB_PATH, WxError, load  # noqa: F401

__version__ = "0.1.0"
