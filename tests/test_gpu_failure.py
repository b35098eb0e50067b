"""Failure handling on the GPU without faulting it, and checks of output bounds.

* A cross-GPU wait that nobody signals (wx_ctx_wait_flags on a flag array that stays zero)
  gives up after the context's peer wait limit: the kernel records a device error and returns,
  wx_ctx_check_device reports WX_ERR_DEVICE, and the context keeps working (signal + wait and
  a quantized linear afterwards are correct). This is the path a rank that never signals takes
  in the peer-memory exchange (wx_dit_block_forward_sp).
* Kernel shared-memory limits are set per device: with two GPUs in one process, the same calls
  on device 0 then on device 1 give identical results (skipped with fewer than two GPUs).
* Canary-padded outputs: the GEMM, attention and row kernels write no element outside their
  outputs (a sentinel before and after each output buffer stays untouched).
"""
import time

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16

pytestmark = pytest.mark.gpu


def test_unsignalled_peer_wait_expires_into_a_device_error():
    import torch
    from wuxianhuabu_b200 import _lib, h3
    ctx = h3.context()
    lib = ctx.lib
    flags = torch.zeros(6, dtype=torch.int32, device="cuda")
    assert lib.wx_ctx_set_peer_wait_limit(ctx.h, 0.5) == _lib.WX_OK
    try:
        t0 = time.perf_counter()
        ctx.call("wx_ctx_wait_flags", flags.data_ptr(), 6, 1)  # nothing ever stores epoch 1
        st = lib.wx_ctx_check_device(ctx.h)                     # synchronises the stream
        dt = time.perf_counter() - t0
        assert st == _lib.WX_ERR_DEVICE, st
        assert b"device error word 7" in lib.wx_last_error(ctx.h)  # the peer-signal timeout code
        assert 0.4 < dt < 10.0, dt
        # the word was cleared and the context still works: signal, then wait, succeeds
        ctx.call("wx_ctx_signal_flags", flags.data_ptr(), 6, 1)
        ctx.call("wx_ctx_wait_flags", flags.data_ptr(), 6, 1)
        assert lib.wx_ctx_check_device(ctx.h) == _lib.WX_OK
        assert (flags == 1).all()
        # wrap-around order: epoch 0 is older than 1, so waiting for it passes at once
        ctx.call("wx_ctx_wait_flags", flags.data_ptr(), 6, 0)
        assert lib.wx_ctx_check_device(ctx.h) == _lib.WX_OK
        # and ordinary kernels are unaffected
        n, k, m = 256, 512, 64
        wq, sc, bi = O.quantize(O.normal_f32((n, k), 5, 1, std=0.02))
        x = O.normal_bf16((m, k), 5, 2)
        lin = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k)
        got = lin(to_torch_bf16(x))
        ctx.check_device()
        assert_close(f32(to_np_bf16(got)), f32(O.qlinear(x, wq, sc, bi)), rel=1e-2, cos=0.9999, what="after wait")
    finally:
        assert lib.wx_ctx_set_peer_wait_limit(ctx.h, 10.0) == _lib.WX_OK
    assert lib.wx_ctx_set_peer_wait_limit(ctx.h, 0.0) == _lib.WX_ERR_INVALID


def _calls_on(device):
    """A quantized linear (two-pass GEMM and small-M fused paths) and a dense + a top-k
    attention on `device`; returns the outputs as host arrays."""
    import torch
    from wuxianhuabu_b200 import h3
    with torch.cuda.device(device):
        dev = torch.device("cuda", device)
        wq, sc, bi = O.quantize(O.normal_f32((768, 1024), 6, 1, std=0.02))
        lin = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).to(dev), to_torch_bf16(sc, dev),
                          to_torch_bf16(bi, dev), 1024)
        outs = [lin(to_torch_bf16(O.normal_bf16((m, 1024), 6, 2 + m), dev)) for m in (100, 1000)]
        q, k, v = (to_torch_bf16(O.normal_bf16((1200, 2, 128), 6, 10 + i), dev) for i in range(3))
        sc_ = float(1 / np.sqrt(128))
        outs.append(h3.H3SolAttn.forward(q, k, v, 0, sc_, None))
        outs.append(h3.H3SolAttn.forward(q, k, v, 200, sc_, h3.H3SolAttnConfig(block=128, topk_ratio=0.25,
                                                                                tail=False)))
        h3.context(device).check_device()
        return [to_np_bf16(o) for o in outs]


def test_two_devices_in_one_process_give_identical_results():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    a = _calls_on(0)
    b = _calls_on(1)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


class Canary:
    """An output buffer with `pad` sentinel elements before and after it."""

    def __init__(self, shape, dtype, pad=4096, fill=-12345.0):
        import torch
        n = int(np.prod(shape))
        self.pad, self.n = pad, n
        self.buf = torch.full((n + 2 * pad,), fill, dtype=dtype, device="cuda")
        self.ref = self.buf[:pad].clone()
        self.view = self.buf[pad:pad + n].view(*shape)

    def check(self, what):
        import torch
        torch.cuda.synchronize()
        assert torch.equal(self.buf[:self.pad], self.ref), f"{what}: write before the output"
        assert torch.equal(self.buf[self.pad + self.n:], self.ref), f"{what}: write after the output"


def test_kernels_write_only_their_outputs():
    import torch
    from wuxianhuabu_b200 import h3
    bf = torch.bfloat16
    # quantized linear: small-M fused path, two-pass path, gated residual with the raw output
    for m in (37, 300, 700):
        n, k = 640, 768
        wq, sc, bi = O.quantize(O.normal_f32((n, k), 8, m, std=0.02))
        lin = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                          to_torch_bf16(O.normal_bf16((n,), 8, 1)))
        x = to_torch_bf16(O.normal_bf16((m, k), 8, 2))
        y = Canary((m, n), bf)
        lin(x, out=y.view)
        y.check(f"qlinear m={m}")
        gate = to_torch_bf16(O.normal_bf16((3, n), 8, 3))
        resid = to_torch_bf16(O.normal_bf16((m, n), 8, 4))
        rm = torch.from_numpy((np.arange(m) % 3).astype(np.int32)).cuda()
        y2, raw = Canary((m, n), bf), Canary((m, n), bf)
        lin(x, epilogue=h3.EPI_GATE_RESID, gate=gate, resid=resid, rowmap=rm, y_raw=raw.view, out=y2.view)
        y2.check(f"qlinear gate m={m}")
        raw.check(f"qlinear raw m={m}")
    # attention: dense, top-k and SOL with ragged tails, head_dim 128 and 64
    for (S, H, hd, g, cfg) in [(1000, 2, 128, 0, None),
                               (1037, 2, 128, 200, h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False)),
                               (900, 3, 128, 77, h3.H3SolAttnConfig(tau=0.4, tail=True)),
                               (700, 2, 64, 0, None),
                               (777, 2, 64, 100, h3.H3SolAttnConfig(tau=0.4, tail=True))]:
        q, k, v = (to_torch_bf16(O.normal_bf16((S, H, hd), 9, i)) for i in range(3))
        o = Canary((S, H, hd), bf)
        h3.H3SolAttn.forward(q, k, v, g, float(1 / np.sqrt(hd)), cfg, out=o.view)
        h3.context().check_device()
        o.check(f"attention S={S} hd={hd} g={g}")
    # row kernels: norm + modulation, gated residual, QK-norm + RoPE
    S, hidden = 333, 1024
    x = to_torch_bf16(O.normal_bf16((S, hidden), 10, 1))
    w = to_torch_bf16(O.normal_bf16((hidden,), 10, 2, mean=1.0, std=0.02))
    tabs = [to_torch_bf16(O.normal_bf16((4, hidden), 10, 3 + i)) for i in range(3)]
    rm = torch.from_numpy((np.arange(S) % 4).astype(np.int32)).cuda()
    o = Canary((S, hidden), bf)
    h3.H3FusedKernels.fused_norm_modscale(x, w, tabs[0], tabs[1], rm, 1e-6, out=o.view)
    o.check("norm_modscale")
    o2 = Canary((S, hidden), bf)
    h3.H3FusedKernels.fused_mod_gate(x, tabs[2], x, rm, out=o2.view)
    o2.check("mod_gate")
    for hd in (128, 64):
        H = 4
        xq = to_torch_bf16(O.normal_bf16((S, H, hd), 11, hd))
        wq_ = to_torch_bf16(O.normal_bf16((hd,), 11, 1, mean=1.0, std=0.02))
        cs = to_torch_bf16(O.normal_bf16((S, 32), 11, 2))
        sn = to_torch_bf16(O.normal_bf16((S, 32), 11, 3))
        o3 = Canary((S, H, hd), bf)
        h3.H3FusedKernels.fused_rmsnorm_rope(xq, wq_, cs, sn, 64, 1e-6, out=o3.view)
        o3.check(f"qk_norm_rope hd={hd}")
    h3.context().check_device()
