"""wx_qlinear_noalloc: the quantized linear layer for callers that cannot
allocate device memory (a host whose engine or restricted allocator owns every
device allocation, or a plugin handed only a stream and tensors). It keeps the
expanded weight in a static device array inside libwx instead of the context
workspace that wx_qlinear grows with cudaMalloc.

The test calls it through the C ABI twice in a row, with different weights and
epilogues, and checks each result against wx_qlinear on the same inputs. This
file sorts last so that a run stopping at the first failure has already run
every other test; it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16

pytestmark = pytest.mark.gpu


def _linear(seed, n, k):
    import torch
    from wuxianhuabu_b200 import h3
    wq, sc, bi = O.quantize(O.normal_f32((n, k), seed, 1, std=0.02))
    bias = O.normal_bf16((n,), seed, 2, std=0.05)
    return h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                       to_torch_bf16(bias))


def test_qlinear_noalloc_matches_qlinear_on_two_calls():
    import torch
    from wuxianhuabu_b200 import _lib, h3
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    cases = [
        # (m, k, n, epilogue): a qkv-like GEMM, then a gated-residual out-projection
        (300, 1024, 3072, h3.EPI_NONE),
        (257, 3072, 1024, h3.EPI_GATE_RESID),
    ]
    for call, (m, k, n, epi) in enumerate(cases):
        lin = _linear(60 + call, n, k)
        x = to_torch_bf16(O.normal_bf16((m, k), 70 + call, 1))
        gate = resid = rowmap = None
        if epi == h3.EPI_GATE_RESID:
            gate = to_torch_bf16(O.normal_bf16((4, n), 80, 1))
            resid = to_torch_bf16(O.normal_bf16((m, n), 80, 2))
            rowmap = torch.from_numpy((np.arange(m) % 4).astype(np.int32)).cuda()
        raw_ref = torch.empty((m, n), dtype=torch.bfloat16, device="cuda") if gate is not None else None
        ref = lin(x, epilogue=epi, gate=gate, resid=resid, rowmap=rowmap, y_raw=raw_ref)  # wx_qlinear
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        raw = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda") if gate is not None else None
        qw = lin.qweight()
        st = lib.wx_qlinear_noalloc(C.c_void_p(stream), x.data_ptr(), m, x.stride(0), C.byref(qw), epi,
                                    None if gate is None else gate.data_ptr(),
                                    None if resid is None else resid.data_ptr(),
                                    None if rowmap is None else rowmap.data_ptr(), out.data_ptr(), out.stride(0),
                                    None if raw is None else raw.data_ptr())
        assert st == _lib.WX_OK, f"call {call}: status {st}"
        torch.cuda.synchronize()
        assert_close(f32(to_np_bf16(out)), f32(to_np_bf16(ref)), rel=1e-2, cos=0.9999, what=f"noalloc call {call}")
        if raw is not None:
            assert_close(f32(to_np_bf16(raw)), f32(to_np_bf16(raw_ref)), rel=1e-2, cos=0.9999, what="raw")


def test_qlinear_noalloc_rejects_weights_beyond_the_static_scratch():
    import torch
    from wuxianhuabu_b200 import _lib, h3
    lib = _lib.load()
    n, k = 12288, 3072  # 37.7M elements > 33,554,432
    lin = h3.MfLinear(torch.zeros((n, k * 6 // 32), dtype=torch.int32, device="cuda"),
                      torch.zeros((n, k // 64), dtype=torch.bfloat16, device="cuda"),
                      torch.zeros((n, k // 64), dtype=torch.bfloat16, device="cuda"), k)
    x = torch.zeros((8, k), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((8, n), dtype=torch.bfloat16, device="cuda")
    qw = lin.qweight()
    stream = torch.cuda.current_stream().cuda_stream
    st = lib.wx_qlinear_noalloc(C.c_void_p(stream), x.data_ptr(), 8, k, C.byref(qw), h3.EPI_NONE, None, None,
                                None, y.data_ptr(), n, None)
    assert st == _lib.WX_ERR_INVALID
    st = lib.wx_qlinear_noalloc(C.c_void_p(stream), x.data_ptr(), 8, k, C.byref(qw), h3.EPI_SWIGLU, None, None,
                                None, y.data_ptr(), n, None)
    assert st == _lib.WX_ERR_UNSUPPORTED
