"""The documented fallbacks of the flash-attention path (switches read once per
process) against the CPU oracle: routed tiles in flash_attn2_kernel
(WX_ATTN_DUO=0) and unpaired strip / dense tiles (WX_ATTN_PAIRS=0). Each runs in
its own child process on dense, SOL and top-k cases with strip rows and ragged
tails."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

CHILD = r'''
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from oracle import oracle as O
from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16
from wuxianhuabu_b200 import h3
H, HD = 2, 128
for (g, L, mode) in [(0, 700, "dense"), (130, 900, "sol"), (300, 1000, "topk"), (17, 260, "topk")]:
    S = g + L
    q, k, v = [O.normal_bf16((S, H, HD), 11 + S, i) for i in (1, 2, 3)]
    sc = float(1 / np.sqrt(HD))
    if mode == "dense":
        cfg, ref = None, O.sparse_attention(q, k, v, 0, sc)
    elif mode == "sol":
        cfg = h3.H3SolAttnConfig(tau=0.4, tail=True)
        route = O.sol_route(q, k, v, g, sc, 0.4)
        route.update(g=g, block=64)
        ref = O.sparse_attention(q, k, v, g, sc, route=route, tail=True)
    else:
        cfg = h3.H3SolAttnConfig(block=128, topk_ratio=0.25, tail=False)
        route = O.topk_route(q, k, v, g, sc, 0.25)
        route.update(g=g, block=128)
        ref = O.sparse_attention(q, k, v, g, sc, block=128, route=route, tail=False)
    tq, tk, tv = [to_torch_bf16(a) for a in (q, k, v)]
    got = h3.H3SolAttn.forward(tq, tk, tv, g, sc, cfg)
    h3.context(0).check_device()
    assert_close(f32(to_np_bf16(got)), f32(ref), rel=2e-2, cos=0.9995, what=f"{mode} g={g} L={L}")
print("ok")
'''


@pytest.mark.parametrize("duo,pairs", [("0", "1"), ("1", "0"), ("0", "0")])
def test_flash_fallback_matches_oracle(duo, pairs):
    env = dict(os.environ, WX_ATTN_DUO=duo, WX_ATTN_PAIRS=pairs)
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], env=env, capture_output=True, text=True,
                       timeout=600, cwd=str(ROOT))
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-2000:]
