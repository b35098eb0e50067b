"""The C ABI driven with host buffers only, as a host without its own CUDA runtime would
(the Swift wrapper): wx_alloc / wx_upload / wx_qlinear / wx_download / wx_free through ctypes,
numpy arrays on the host side, no torch tensor holding the data. The result equals the same
call made on torch-owned device memory bit for bit, and the oracle within the GEMM bound."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16

pytestmark = pytest.mark.gpu


def test_qlinear_through_abi_memory_calls():
    import torch
    from wuxianhuabu_b200 import _lib, h3
    ctx = h3.context()
    lib = ctx.lib
    m, k, n = 700, 1024, 768
    wq, sc, bi = O.quantize(O.normal_f32((n, k), 81, 1, std=0.02))
    bias = O.normal_bf16((n,), 81, 2, std=0.1)
    x = O.normal_bf16((m, k), 81, 3)
    host = {"x": x, "wq": wq.view(np.uint32), "sc": sc, "bi": bi, "bias": bias}
    dev = {}
    try:
        for name, arr in host.items():
            p = C.c_void_p()
            assert lib.wx_alloc(ctx.h, arr.nbytes, C.byref(p)) == _lib.WX_OK
            assert p.value and p.value % 256 == 0
            dev[name] = p
            assert lib.wx_upload(ctx.h, p, arr.ctypes.data, arr.nbytes) == _lib.WX_OK
        y = C.c_void_p()
        assert lib.wx_alloc(ctx.h, m * n * 2, C.byref(y)) == _lib.WX_OK
        dev["y"] = y
        qw = _lib.QWeight(dev["wq"].value, dev["sc"].value, dev["bi"].value, dev["bias"].value, n, k, 64, 6)
        st = lib.wx_qlinear(ctx.h, dev["x"], m, k, C.byref(qw), _lib.EPI_NONE, None, None, None, y, n, None)
        assert st == _lib.WX_OK, lib.wx_last_error(ctx.h)
        got = np.empty((m, n), dtype=np.uint16)
        assert lib.wx_download(ctx.h, got.ctypes.data, y, got.nbytes) == _lib.WX_OK
        assert lib.wx_ctx_synchronize(ctx.h) == _lib.WX_OK
        ctx.check_device()
    finally:
        for p in dev.values():
            assert lib.wx_free(ctx.h, p) == _lib.WX_OK
    # the same call on torch-owned memory
    lin = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                      to_torch_bf16(bias))
    want = to_np_bf16(lin(to_torch_bf16(x)))
    assert np.array_equal(got, want.view(np.uint16))
    assert_close(f32(got), f32(O.qlinear(x, wq, sc, bi, bias=bias)), rel=1e-2, cos=0.9999, what="abi qlinear")
    # empty requests and null frees are no-ops
    p = C.c_void_p(1)
    assert lib.wx_alloc(ctx.h, 0, C.byref(p)) == _lib.WX_OK and not p.value
    assert lib.wx_free(ctx.h, None) == _lib.WX_OK
    assert lib.wx_upload(ctx.h, None, None, 0) == _lib.WX_OK
