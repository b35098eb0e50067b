"""CPU checks of the oracle's conditioning restatement (no GPU): the timestep sinusoid
(H3TimeEmbedder.forward, H3Transformer.swift:287-302) against a pure-Python loop written
like the reference's, the LUT row rule (H3AdalnLUT.coeffs :338-349), the table split of
H3AdalnW.forward (:392-404), the MLX SiLU and sigmoid, and rmsNormLast (H3Common.swift:502-508)."""
import math

import numpy as np
import pytest

from oracle import oracle as O


def test_sinusoid_matches_reference_loop():
    ts = [0.0, 0.25, 1.0, 27.03, 972.97, 1000.0]
    dim = 256
    got = O.timestep_sinusoid(ts, dim)
    half = dim // 2
    log10k = math.log(10000.0)
    for i, t in enumerate(ts):
        for j in range(half):
            freq = math.exp(-log10k * j / half)
            assert got[i, j] == np.float32(math.cos(t * freq))
            assert got[i, half + j] == np.float32(math.sin(t * freq))


@pytest.mark.parametrize("t,n,want", [(0.0, 1025, 0), (1.0, 1025, 1024), (0.5, 1025, 512),
                                      (0.5 / 1024, 1025, 1), (1.5 / 1024, 1025, 2), (-0.3, 1025, 0),
                                      (1.7, 1025, 1024), (0.49, 3, 1), (0.24, 3, 0), (0.25, 3, 1)])
def test_lut_row_rounds_half_away_from_zero_and_clamps(t, n, want):
    assert int(O.lut_rows([t], n)[0]) == want


def test_lut_coeffs_gather_rows():
    table = np.arange(5 * 3, dtype=np.float32).reshape(5, 3) + 0.5
    got = O.lut_coeffs([0.0, 1.0, 0.5], table)
    assert np.array_equal(got, O.f32_to_bf16(table[[0, 4, 2]]))


@pytest.mark.parametrize("m,expand,modalities", [(1, 6, 3), (3, 6, 3), (2, 2, 1)])
def test_adaln_split_layout(m, expand, modalities):
    """table e, row t*modalities + tag, column c = y[t, (tag*expand + e)*hidden + c]"""
    hidden = 16
    y = np.arange(m * modalities * expand * hidden, dtype=np.uint16).reshape(m, -1)
    tabs = O.adaln_split(y, expand, modalities)
    assert len(tabs) == expand
    for e in range(expand):
        assert tabs[e].shape == (m * modalities, hidden)
        for t in range(m):
            for tag in range(modalities):
                col = (tag * expand + e) * hidden
                assert np.array_equal(tabs[e][t * modalities + tag], y[t, col:col + hidden])


def test_sigmoid_and_silu_values():
    x = np.array([0.0, 1.0, -1.0, 20.0, -20.0, 100.0, -100.0], dtype=np.float32)
    s = O.sigmoid_mlx(x)
    ref = 1.0 / (1.0 + np.exp(-x.astype(np.float64)))
    assert np.allclose(s, ref, rtol=1e-6, atol=1e-7)
    assert s[0] == 0.5 and s[-1] >= 0.0 and s[-2] == 1.0
    assert np.allclose(O.silu_f32(x), x * ref, rtol=1e-6, atol=1e-6)
    xb = O.f32_to_bf16(x)
    got = O.bf16_to_f32(O.silu_bf16(xb))
    want = O.bf16_to_f32(O.f32_to_bf16(O.bf16_to_f32(xb) * O.bf16_to_f32(O.f32_to_bf16(s))))
    assert np.array_equal(got, want)


def test_rms_norm_is_one_rounding_of_the_fp32_formula():
    x = O.normal_bf16((8, 256), 3, 1, std=3.0)
    w = O.normal_bf16((256,), 3, 2, mean=1.0, std=0.1)
    xf = O.bf16_to_f32(x).astype(np.float64)
    rstd = 1.0 / np.sqrt((xf * xf).mean(axis=1, keepdims=True) + 1e-5)
    want = xf * rstd * O.bf16_to_f32(w)[None, :]
    got = O.bf16_to_f32(O.rms_norm(x, w, 1e-5))
    # one bf16 rounding of the exact value: within half a bf16 step (2^-8 relative)
    assert np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -8 + 1e-30)


def test_linear_bf16_rounds_product_then_bias():
    x = O.f32_to_bf16(np.array([[1.0, 2.0]], dtype=np.float32))
    w = O.f32_to_bf16(np.array([[1.0, 0.0], [1.0 / 256, 1.0]], dtype=np.float32))  # [in, out]
    b = O.f32_to_bf16(np.array([1.0 / 512, 0.0], dtype=np.float32))
    got = O.bf16_to_f32(O.linear_bf16(x, w, b))
    # x w = [1 + 2/256, 2]; +1/512 after the first rounding
    step1 = O.bf16_to_f32(O.f32_to_bf16(np.array([1.0 + 2.0 / 256], dtype=np.float32)))[0]
    assert got[0, 0] == O.bf16_to_f32(O.f32_to_bf16(np.array([step1 + 1.0 / 512], dtype=np.float32)))[0]
    assert got[0, 1] == 2.0
