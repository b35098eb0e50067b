"""CPU tests of the C ABI boundary: libwx.so loads without a GPU and exports
every entry point declared in include/wx_api.h; argument validation returns
error codes instead of aborting."""
import ctypes as C
import re
from pathlib import Path

from wuxianhuabu_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    txt = (ROOT / "include" / "wx_api.h").read_text()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(wx_[a-z0-9_]+)\s*\(", txt)))


def test_every_declared_symbol_is_exported():
    lib = C.CDLL(str(_lib.LIB_PATH))
    names = declared_symbols()
    assert len(names) > 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_checked_build_exports_the_same_symbols():
    """The bounds-checked build (libwx_checked.so, -DWX_BOUNDS_CHECK=1) is the same ABI."""
    import pytest
    path = _lib.LIB_PATH.parent / "libwx_checked.so"
    if not path.exists():
        pytest.skip("libwx_checked.so not built")
    lib = C.CDLL(str(path))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert set(declared_symbols()) == set(_lib.exported_symbols())


def test_null_context_is_an_error_not_a_crash():
    lib = _lib.load()
    assert lib.wx_ctx_check_device(None) == _lib.WX_ERR_INVALID
    assert lib.wx_ctx_create(0, None) == _lib.WX_ERR_INVALID
    assert lib.wx_sigma_schedule(0, 12.0, None) == _lib.WX_ERR_INVALID
    assert lib.wx_build_row_mod_map(None, 1, 4, None) == _lib.WX_ERR_INVALID


def test_ctx_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        return
    h = C.c_void_p()
    assert _lib.load().wx_ctx_create(0, C.byref(h)) != _lib.WX_OK
