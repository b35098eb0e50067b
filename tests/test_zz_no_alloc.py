"""wx_qlinear_noalloc: the quantized linear layer for callers that cannot
allocate device memory (a host whose engine or restricted allocator owns every
device allocation, or a plugin handed only a stream and tensors). It keeps the
expanded weight in a static device array inside libwx instead of the context
workspace that wx_qlinear grows with cudaMalloc.

The test calls it through the C ABI twice in a row, with different weights and
epilogues, checks that no device memory is allocated across the two calls and
that the device error word stays clear (wx_qlinear_noalloc_check), and compares
each result with the oracle and with wx_qlinear on the same inputs. This file
sorts last so that a run stopping at the first failure has already run every
other test; it also passes on its own in a fresh process.
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
    lin = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                      to_torch_bf16(bias))
    return lin, (wq, sc, bi, bias)


def _call(lib, stream, case):
    x, qw, epi, gate, resid, rowmap, out, raw = case
    return lib.wx_qlinear_noalloc(C.c_void_p(stream), x.data_ptr(), x.shape[0], x.stride(0), C.byref(qw), epi,
                                  None if gate is None else gate.data_ptr(),
                                  None if resid is None else resid.data_ptr(),
                                  None if rowmap is None else rowmap.data_ptr(), out.data_ptr(), out.stride(0),
                                  None if raw is None else raw.data_ptr())


def test_qlinear_noalloc_matches_oracle_and_qlinear_on_two_calls():
    """Two calls in a row (a qkv-like GEMM, then a gated-residual out-projection) with no
    device allocation between them: free device memory is the same before and after,
    the device error word stays clear, and each output matches the oracle and wx_qlinear."""
    import torch
    from wuxianhuabu_b200 import _lib, h3
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    shapes = [(300, 1024, 3072, h3.EPI_NONE), (257, 3072, 1024, h3.EPI_GATE_RESID)]
    cases, refs, keep = [], [], []  # keep: the linears whose device memory the QWeight structs point at
    for call, (m, k, n, epi) in enumerate(shapes):
        lin, (wq, sc, bi, bias) = _linear(60 + call, n, k)
        xn = O.normal_bf16((m, k), 70 + call, 1)
        x = to_torch_bf16(xn)
        gate = resid = rowmap = None
        gn = rn = rmn = None
        if epi == h3.EPI_GATE_RESID:
            gn, rn = O.normal_bf16((4, n), 80, 1), O.normal_bf16((m, n), 80, 2)
            rmn = (np.arange(m) % 4).astype(np.uint32)
            gate, resid = to_torch_bf16(gn), to_torch_bf16(rn)
            rowmap = torch.from_numpy(rmn.view(np.int32)).cuda()
        raw_q = torch.empty((m, n), dtype=torch.bfloat16, device="cuda") if gate is not None else None
        via_ctx = lin(x, epilogue=epi, gate=gate, resid=resid, rowmap=rowmap, y_raw=raw_q)  # wx_qlinear
        oracle = O.qlinear(xn, wq, sc, bi, bias=bias, epilogue=epi, gate=gn, resid=rn, rowmap=rmn,
                           want_raw=gate is not None)
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        raw = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda") if gate is not None else None
        keep.append(lin)
        cases.append((x, lin.qweight(), epi, gate, resid, rowmap, out, raw))
        refs.append((via_ctx, raw_q, oracle))
    # set-up call: with lazy module loading this reserves the static array on the device
    assert _call(lib, stream, cases[0]) == _lib.WX_OK, lib.wx_qlinear_noalloc_last_error()
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for call, case in enumerate(cases):
        case[6].fill_(float("nan"))
        if case[7] is not None:
            case[7].fill_(float("nan"))
    torch.cuda.synchronize()
    for call, case in enumerate(cases):
        st = _call(lib, stream, case)
        assert st == _lib.WX_OK, f"call {call}: status {st}: {lib.wx_qlinear_noalloc_last_error()}"
    assert lib.wx_qlinear_noalloc_check(C.c_void_p(stream)) == _lib.WX_OK, lib.wx_qlinear_noalloc_last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before, "device memory was allocated during the calls"
    for call, (case, (via_ctx, raw_q, oracle)) in enumerate(zip(cases, refs)):
        out, raw = case[6], case[7]
        ref_o = oracle[0] if raw is not None else oracle
        assert_close(f32(to_np_bf16(out)), f32(ref_o), rel=1e-2, cos=0.9999, what=f"noalloc call {call} vs oracle")
        assert_close(f32(to_np_bf16(out)), f32(to_np_bf16(via_ctx)), rel=1e-2, cos=0.9999,
                     what=f"noalloc call {call} vs wx_qlinear")
        if raw is not None:
            assert_close(f32(to_np_bf16(raw)), f32(oracle[1]), rel=1e-2, cos=0.9999, what="raw vs oracle")
            assert_close(f32(to_np_bf16(raw)), f32(to_np_bf16(raw_q)), rel=1e-2, cos=0.9999, what="raw")


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
    assert b"static scratch" in lib.wx_qlinear_noalloc_last_error()
    st = lib.wx_qlinear_noalloc(C.c_void_p(stream), x.data_ptr(), 8, k, C.byref(qw), h3.EPI_SWIGLU, None, None,
                                None, y.data_ptr(), n, None)
    assert st == _lib.WX_ERR_UNSUPPORTED
