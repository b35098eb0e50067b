"""The q|k|v projection with QK-RMSNorm + RoPE fused into the GEMM's epilogue
(gemm_bf16_tc_kernel<BN, true>) against the separate path (GEMM, then qk_norm_rope_vec_kernel),
which WX_QKV_ROPE_FUSED=0 selects in a child process (both children with WX_QGEMM_TWO_PASS=1,
so that every projection runs the same GEMM).

The two paths round at the same points and form the sum of squares in the same order, so whole
DiT blocks (dense, top-k and SOL attention, ragged last row tile, 2 and 3 heads so that both the
256- and the 128-column tiles run, head_dim 128 and 64 (the config-1 geometry: 16 x 64, rot 64),
with and without a bias on the projection, a PAB slot) must come out bit-identical. The oracle comparison of the fused path is in test_gpu_block /
test_gpu_parity_full (they run the default path)."""
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

CHILD = r'''
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import torch
from oracle import oracle as O
from tests._util import to_np_bf16, to_torch_bf16
from tests.test_gpu_block import gpu_block, make_block
from wuxianhuabu_b200 import h3
outs = {}
for (S, heads, hd, bias, mode, g) in [(300, 2, 128, False, "dense", 0), (1000, 3, 128, True, "topk", 200),
                                      (1000, 2, 128, False, "sol", 130), (2048, 2, 128, True, "dense", 0),
                                      (4096, 16, 64, True, "dense", 0), (777, 4, 64, False, "dense", 0)]:
    hidden, ffn, eps = 256, 512, 1e-6
    rot = 96 if hd == 128 else 64
    w, mods, h, cos, sin, rowmap = make_block(50 + S + heads, hidden, heads, ffn, 0, S, rot, hd=hd)
    wq, sc, bi, b = w["qkv"]
    w["qkv"] = (wq, sc, bi, O.normal_bf16((3 * heads * hd,), 9, S, std=0.5) if bias else None)
    blk = gpu_block(w, hidden, heads, ffn, 0, rot, eps, hd=hd)
    spec = None
    if mode == "topk":
        spec = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False).spec(g)
    elif mode == "sol":
        spec = h3.H3SolAttnConfig(tau=0.4, tail=True).spec(g)
    x = to_torch_bf16(h)
    slot = torch.empty((S, hidden), dtype=torch.bfloat16, device="cuda")
    blk.block_forward(0, x, [to_torch_bf16(m) for m in mods], torch.from_numpy(rowmap.view(np.int32)).cuda(),
                      to_torch_bf16(cos), to_torch_bf16(sin), spec, pab_slot=slot, refresh=True)
    h3.context().check_device()
    key = f"{S}_{heads}_{hd}_{int(bias)}_{mode}"
    outs[key + "_h"] = to_np_bf16(x).view(np.uint16)
    outs[key + "_at"] = to_np_bf16(slot).view(np.uint16)
np.savez(sys.argv[2], **outs)
print("ok")
'''


def _run(fused: str, path: str):
    # both runs on the two-pass GEMM (the separate path would otherwise take the small-M
    # kernel at S = 300, whose split-K sums round differently)
    env = dict(os.environ, WX_QKV_ROPE_FUSED=fused, WX_QGEMM_TWO_PASS="1")
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), path], env=env, capture_output=True, text=True,
                       timeout=600, cwd=str(ROOT))
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-2000:]
    return np.load(path)


def test_fused_qkv_rope_epilogue_is_bit_identical_to_the_separate_kernel():
    with tempfile.TemporaryDirectory() as d:
        a = _run("1", os.path.join(d, "fused.npz"))
        b = _run("0", os.path.join(d, "separate.npz"))
        assert sorted(a.files) == sorted(b.files)
        for k in a.files:
            diff = int(np.count_nonzero(a[k] != b[k]))
            assert diff == 0, f"{k}: {diff} of {a[k].size} elements differ"


@pytest.mark.parametrize("m,heads,hd,bias,lora", [(700, 3, 128, True, False), (2048, 2, 128, False, False),
                                                  (1500, 2, 128, True, True), (1024, 4, 64, True, False),
                                                  (4096, 16, 64, False, False)])
def test_wx_qkv_norm_rope_equals_projection_then_norm_rope(m, heads, hd, bias, lora):
    """The ABI call (one GEMM with the norm/RoPE epilogue) against the two calls it replaces:
    the two-pass projection (M > 512; with the LoRA delta as a K extension) and the row kernel
    on q and k, bit for bit."""
    import torch
    from tests._util import to_torch_bf16
    from wuxianhuabu_b200 import h3
    hidden, eps = 512, 1e-6
    rot = 96 if hd == 128 else 64
    inner = heads * hd
    wq, sc, bi = O.quantize(O.normal_f32((3 * inner, hidden), 71, m, std=0.02))
    b = to_torch_bf16(O.normal_bf16((3 * inner,), 71, 1, std=0.5)) if bias else None
    lin = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), hidden, b)
    if lora:
        a_ = to_torch_bf16(O.normal_bf16((hidden, 16), 71, 2, std=0.05))
        b_ = to_torch_bf16(O.normal_bf16((16, 3 * inner), 71, 3, std=0.05))
        lin.set_lora([h3.LoraRef(a_, b_, 0.5)])
    x = to_torch_bf16(O.normal_bf16((m, hidden), 71, 4))
    qn = to_torch_bf16(O.normal_bf16((hd,), 71, 5, mean=1.0, std=0.02))
    kn = to_torch_bf16(O.normal_bf16((hd,), 71, 6, mean=1.0, std=0.02))
    cos = to_torch_bf16(O.normal_bf16((m, rot // 2), 71, 7))
    sin = to_torch_bf16(O.normal_bf16((m, rot // 2), 71, 8))
    got = lin.qkv_norm_rope(x, heads, hd, qn, kn, cos, sin, rot, eps)
    ref = lin(x)
    for part, w in ((0, qn), (1, kn)):
        view = ref[:, part * inner:(part + 1) * inner].view(m, heads, hd)
        h3.H3FusedKernels.fused_rmsnorm_rope(view, w, cos, sin, rot, eps, out=view)
    h3.context().check_device()
    assert torch.equal(got, ref)


def test_wx_qkv_norm_rope_small_m_and_head_dim_64_against_the_oracle():
    """M <= 512 (the fused epilogue on the two-pass GEMM) and head_dim 64 (the two-call path)
    against the oracle's projection + qk_norm_rope, at the GEMM's bound."""
    import torch
    from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16
    from wuxianhuabu_b200 import h3
    for (m, heads, hd, rot) in [(300, 2, 128, 96), (257, 4, 64, 32)]:
        hidden, eps = 256, 1e-6
        inner = heads * hd
        wq, sc, bi = O.quantize(O.normal_f32((3 * inner, hidden), 72, m, std=0.02))
        bias = O.normal_bf16((3 * inner,), 72, 1, std=0.1)
        lin = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), hidden,
                          to_torch_bf16(bias))
        x = O.normal_bf16((m, hidden), 72, 2)
        qn = O.normal_bf16((hd,), 72, 3, mean=1.0, std=0.02)
        kn = O.normal_bf16((hd,), 72, 4, mean=1.0, std=0.02)
        cos = O.normal_bf16((m, rot // 2), 72, 5)
        sin = O.normal_bf16((m, rot // 2), 72, 6)
        got = to_np_bf16(lin.qkv_norm_rope(to_torch_bf16(x), heads, hd, to_torch_bf16(qn), to_torch_bf16(kn),
                                           to_torch_bf16(cos), to_torch_bf16(sin), rot, eps))
        h3.context().check_device()
        y = O.qlinear(x, wq, sc, bi, bias=bias)
        want = y.copy()
        for part, w in ((0, qn), (1, kn)):
            blk = np.ascontiguousarray(y[:, part * inner:(part + 1) * inner]).reshape(m, heads, hd)
            want[:, part * inner:(part + 1) * inner] = O.qk_norm_rope(blk, w, cos, sin, rot, eps).reshape(m, inner)
        assert_close(f32(got), f32(want), rel=1e-2, cos=0.9999, what=f"qkv_norm_rope m={m} hd={hd}")
