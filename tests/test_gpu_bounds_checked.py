"""The bounds-checked build (libwx_checked.so: -DWX_BOUNDS_CHECK=1, the debug build with
explicit bounds checks that stands in for compute-sanitizer) on the parity workloads: DiT
blocks (dense / top-k / SOL with strip rows and ragged tails, head_dim 128 and 64), the
quantized linear on both paths (small M and two-pass, gated residual), the q|k|v projection
with its norm/RoPE epilogue, and attention with head_dim 128 and 64. Each runs in a child
process on each build: the checked build records no bounds error (every guarded access was
inside its buffer) and its outputs equal the normal build's bit for bit (the checks change
no arithmetic)."""
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest

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
# blocks
for (S, heads, hd, mode, g) in [(1000, 2, 128, "topk", 203), (937, 2, 128, "sol", 130), (700, 3, 128, "dense", 0),
                                (777, 4, 64, "dense", 0)]:
    rot = 96 if hd == 128 else 64
    w, mods, h, cos, sin, rowmap = make_block(90 + S, 256, heads, 512, 0, S, rot, hd=hd)
    blk = gpu_block(w, 256, heads, 512, 0, rot, 1e-6, hd=hd)
    spec = None
    if mode == "topk":
        spec = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False).spec(g)
    elif mode == "sol":
        spec = h3.H3SolAttnConfig(tau=0.4, tail=True).spec(g)
    x = to_torch_bf16(h)
    slot = torch.empty((S, 256), dtype=torch.bfloat16, device="cuda")
    blk.block_forward(0, x, [to_torch_bf16(m) for m in mods], torch.from_numpy(rowmap.view(np.int32)).cuda(),
                      to_torch_bf16(cos), to_torch_bf16(sin), spec, pab_slot=slot, refresh=True)
    outs[f"block_{S}_{mode}_{hd}"] = to_np_bf16(x).view(np.uint16)
    outs[f"slot_{S}_{mode}_{hd}"] = to_np_bf16(slot).view(np.uint16)
# quantized linear, both paths, gated residual
for m in (37, 300, 1100):
    n, k = 640, 768
    wq, sc, bi = O.quantize(O.normal_f32((n, k), 91, m, std=0.02))
    lin = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                      to_torch_bf16(O.normal_bf16((n,), 91, 1)))
    x = to_torch_bf16(O.normal_bf16((m, k), 91, 2))
    gate = to_torch_bf16(O.normal_bf16((3, n), 91, 3))
    resid = to_torch_bf16(O.normal_bf16((m, n), 91, 4))
    rm = torch.from_numpy((np.arange(m) % 3).astype(np.int32)).cuda()
    outs[f"lin_{m}"] = to_np_bf16(lin(x)).view(np.uint16)
    outs[f"lin_gate_{m}"] = to_np_bf16(lin(x, epilogue=h3.EPI_GATE_RESID, gate=gate, resid=resid,
                                           rowmap=rm)).view(np.uint16)
# attention alone, head_dim 128 and 64
for (S, H, hd, g, cfg) in [(1037, 2, 128, 200, h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False)),
                           (901, 3, 128, 77, h3.H3SolAttnConfig(tau=0.4, tail=True)),
                           (777, 2, 64, 100, h3.H3SolAttnConfig(tau=0.4, tail=True))]:
    q, k_, v = (to_torch_bf16(O.normal_bf16((S, H, hd), 92, i)) for i in range(3))
    outs[f"attn_{S}_{hd}"] = to_np_bf16(h3.H3SolAttn.forward(q, k_, v, g, float(1 / np.sqrt(hd)), cfg)).view(np.uint16)
h3.context().check_device()  # raises on a recorded device error (bounds: code 8)
np.savez(sys.argv[2], **outs)
print("ok")
'''


def _run(variant: str, path: str):
    env = dict(os.environ)
    env.pop("WX_LIB_VARIANT", None)
    if variant:
        env["WX_LIB_VARIANT"] = variant
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), path], env=env, capture_output=True, text=True,
                       timeout=600, cwd=str(ROOT))
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-2000:]
    return np.load(path)


def test_checked_build_reports_no_bounds_error_and_matches_the_normal_build():
    if not (ROOT / "wuxianhuabu_b200" / "libwx_checked.so").exists():
        pytest.fail("libwx_checked.so is missing: __graft_entry__.build() builds it")
    with tempfile.TemporaryDirectory() as d:
        a = _run("checked", os.path.join(d, "checked.npz"))
        b = _run("", os.path.join(d, "normal.npz"))
        assert sorted(a.files) == sorted(b.files)
        for k in a.files:
            assert np.array_equal(a[k], b[k]), k
