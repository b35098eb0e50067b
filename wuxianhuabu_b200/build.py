"""Build the in-tree native libraries.

* ``wuxianhuabu_b200/libwx.so`` — the CUDA product (sm_100a kernels + C ABI of
  ``include/wx_api.h``), compiled with nvcc for ``compute_100a``/``sm_100a``.
* ``wuxianhuabu_b200/libwx_checked.so`` — the same sources with ``-DWX_BOUNDS_CHECK=1``:
  the guarded global accesses test their indices and record an error instead of
  touching memory outside their buffers (loaded when ``WX_LIB_VARIANT=checked``).
* ``oracle/_build/libwxoracle.so`` — the CPU restatement used only as the
  parity checker by the tests and the CPU baseline of ``bench.py``.

Both land inside the repository so that they travel with it; nothing is
installed into site-packages.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libwx.so"
BUILD_CHECKED = PKG / "_build_checked"
LIB_CHECKED = PKG / "libwx_checked.so"
ORACLE_DIR = ROOT / "oracle"
ORACLE_LIB = ORACLE_DIR / "_build" / "libwxoracle.so"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
    "-I" + str(ROOT / "include"), "--expt-relaxed-constexpr",
]


def _run(cmd: list[str], cwd: Path | None = None) -> str:
    p = subprocess.run(cmd, cwd=cwd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if p.returncode != 0:
        raise RuntimeError(f"command failed ({p.returncode}): {' '.join(cmd)}\n{p.stdout}")
    return p.stdout


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_cuda(force: bool = False, verbose_ptxas: bool = False, checked: bool = False) -> Path:
    build_dir, lib = (BUILD_CHECKED, LIB_CHECKED) if checked else (BUILD, LIB)
    build_dir.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [ROOT / "include" / "wx_api.h"]
    objs = []
    jobs = []
    for src in _sources():
        obj = build_dir / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            flags = NVCC_FLAGS + (["-Xptxas", "-v"] if verbose_ptxas else []) + (["-DWX_BOUNDS_CHECK=1"] if checked else [])
            jobs.append([NVCC] + flags + ["-c", str(src), "-o", str(obj)])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            outs = list(ex.map(_run, jobs))
        if verbose_ptxas:
            for o in outs:
                sys.stdout.write(o)
    if force or jobs or _stale(lib, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", str(lib)] + [str(o) for o in objs])
    return lib


def build_oracle(force: bool = False) -> Path:
    src = ORACLE_DIR / "wx_oracle.c"
    hdr = ORACLE_DIR / "wx_oracle.h"
    ORACLE_LIB.parent.mkdir(exist_ok=True)
    if force or _stale(ORACLE_LIB, [src, hdr]):
        _run(["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared",
              "-o", str(ORACLE_LIB), str(src), "-lm"])
    return ORACLE_LIB


def build_all(force: bool = False, verbose_ptxas: bool = False) -> None:
    build_oracle(force)
    build_cuda(force, verbose_ptxas)
    build_cuda(force, False, checked=True)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
    print("built", LIB, LIB_CHECKED, ORACLE_LIB)
