"""A plain C host (tests/abi_c/host_qlinear.c) against libwx.so through include/wx_api.h alone,
the way the reference's Swift host would bind it: compiled and linked with gcc here (CPU), and on
a GPU run end to end (context, device buffers, upload, quantized linear, download) with its
output equal bit for bit to the same linear called from Python on torch-owned memory, and within
the GEMM bound of the oracle."""
import os
import subprocess
import tempfile
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "abi_c" / "host_qlinear.c"
LIBDIR = ROOT / "wuxianhuabu_b200"


def _compile(out: Path) -> None:
    r = subprocess.run(["gcc", "-O2", "-Wall", "-Wextra", "-Werror", "-std=c11", f"-I{ROOT / 'include'}", str(SRC),
                        f"-L{LIBDIR}", "-lwx", f"-Wl,-rpath,{LIBDIR}", "-o", str(out)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_c_host_compiles_and_links_against_the_header_and_library():
    with tempfile.TemporaryDirectory() as d:
        exe = Path(d) / "host_qlinear"
        _compile(exe)
        r = subprocess.run([str(exe)], capture_output=True, text=True)
        assert r.returncode == 2 and "usage" in r.stderr  # runs (no GPU needed to print its usage)


@pytest.mark.gpu
def test_c_host_runs_the_quantized_linear():
    import torch
    from tests._util import assert_close, f32, to_np_bf16, to_torch_bf16
    from wuxianhuabu_b200 import h3
    m, k, n = 600, 1024, 768
    wq, sc, bi = O.quantize(O.normal_f32((n, k), 83, 1, std=0.02))
    bias = O.normal_bf16((n,), 83, 2, std=0.1)
    x = O.normal_bf16((m, k), 83, 3)
    with tempfile.TemporaryDirectory() as d:
        exe, fin, fout = Path(d) / "host_qlinear", Path(d) / "in.bin", Path(d) / "out.bin"
        _compile(exe)
        with open(fin, "wb") as f:
            for a in (x, wq.view(np.uint32), sc, bi, bias):
                f.write(np.ascontiguousarray(a).tobytes())
        env = dict(os.environ)
        r = subprocess.run([str(exe), str(m), str(k), str(n), str(fin), str(fout)], capture_output=True, text=True,
                           timeout=300, env=env)
        assert r.returncode == 0, r.stderr
        got = np.fromfile(fout, dtype=np.uint16).reshape(m, n)
    lin = h3.MfLinear(torch.from_numpy(wq.view(np.int32)).cuda(), to_torch_bf16(sc), to_torch_bf16(bi), k,
                      to_torch_bf16(bias))
    want = to_np_bf16(lin(to_torch_bf16(x))).view(np.uint16)
    assert np.array_equal(got, want)
    assert_close(f32(got), f32(O.qlinear(x, wq, sc, bi, bias=bias)), rel=1e-2, cos=0.9999, what="C host qlinear")
