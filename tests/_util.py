"""Shared helpers of the test suite: bf16 conversions between torch and numpy
and the tolerance checks used throughout (max relative error against the
largest reference magnitude, and cosine similarity)."""
from __future__ import annotations

import numpy as np

from oracle import oracle


def to_np_bf16(t) -> np.ndarray:
    import torch
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def to_torch_bf16(a: np.ndarray, device="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)


def f32(a_bf16: np.ndarray) -> np.ndarray:
    return oracle.bf16_to_f32(a_bf16)


def max_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    denom = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / denom)


def cosine(got: np.ndarray, ref: np.ndarray) -> float:
    a = got.astype(np.float64).ravel()
    b = ref.astype(np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))


def assert_close(got: np.ndarray, ref: np.ndarray, rel: float = 2e-2, cos: float = 0.999, what: str = ""):
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    e = max_rel_err(got, ref)
    c = cosine(got, ref)
    assert e <= rel and c >= cos, f"{what}: max rel err {e:.3e} (<= {rel}), cosine {c:.6f} (>= {cos})"
