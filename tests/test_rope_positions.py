"""Position primitives of the packed layout (H3Layout.swift:188-210, 683-694) through the
C ABI against the oracle (host code: runs without a GPU), the packed positions of a
text + reference images + video layout, and buildRope (:725-740) on the GPU."""
import math

import numpy as np
import pytest

from oracle import oracle as O
from wuxianhuabu_b200 import h3


@pytest.mark.parametrize("dim,patch", [(90, 2), (160, 2), (120, 2), (46, 2), (7, 2)])
def test_axis_from_sqrt_area_bit_exact(dim, patch):
    for other in (90, 160, 120):
        area = math.sqrt(float(dim) * float(other))
        got = np.array(h3.axis_from_sqrt_area(dim, patch, area))
        assert np.array_equal(got, O.axis_from_sqrt_area(dim, patch, area))
        assert len(got) == dim // patch


def test_video_t_grid_and_span():
    assert [h3.video_t_span(k) for k in range(6)] == [5 / 3, 20 / 3, 20 / 3, 20 / 3, 20 / 3, 5 / 3]
    for n, origin in [(0, 0.0), (1, 3.0), (31, 516.0), (12, -2.5)]:
        assert np.array_equal(np.array(h3.video_t_grid(n, origin)), O.video_t_grid(n, origin))


def test_packed_positions_layout():
    text, refs, (lt, lh, lw) = 7, [(8, 12), (10, 10)], (3, 6, 8)
    pos = h3.packed_positions(text, refs, lt, lh, lw)
    rows = [(h // 2) * (w // 2) for h, w in refs]
    frame = (lh // 2) * (lw // 2)
    assert pos.shape == (text + sum(rows) + lt * frame, 3)
    assert np.array_equal(pos[:text, 0], np.arange(text)) and not pos[:text, 1:].any()
    r, cursor = text, float(text)
    for (h, w), n in zip(refs, rows):
        area = math.sqrt(h * w)
        ha, wa = O.axis_from_sqrt_area(h, 2, area), O.axis_from_sqrt_area(w, 2, area)
        blk = pos[r:r + n]
        assert (blk[:, 0] == cursor).all()
        assert np.array_equal(blk[:, 1], np.repeat(ha, len(wa))) and np.array_equal(blk[:, 2], np.tile(wa, len(ha)))
        r += n
        cursor += 1.0
    tg = O.video_t_grid(lt, cursor)
    for f in range(lt):
        assert (pos[r + f * frame:r + (f + 1) * frame, 0] == tg[f]).all()


def test_write_frame_grid_rejects_overflow():
    pos = np.zeros((4, 3))
    with pytest.raises(h3.WxError):
        h3.write_frame_grid(pos, 2, 0.0, [0.0, 1.0], [0.0, 1.0])


@pytest.mark.gpu
def test_build_rope_vs_oracle():
    import torch
    from tests._util import to_np_bf16
    pos = h3.packed_positions(512, [(120, 120)], 4, 90, 160)
    inv = (1.0 / (10000.0 ** (np.arange(16, dtype=np.float64) * 2 / 32))).astype(np.float32)
    cos, sin = h3.build_rope(pos, torch.from_numpy(inv).cuda())
    h3.context().check_device()
    rc, rs = O.build_rope(pos, inv)
    for got, ref in ((to_np_bf16(cos), rc), (to_np_bf16(sin), rs)):
        assert got.shape == (pos.shape[0], 48)
        ia = np.where(got & 0x8000, -(got.astype(np.int32) & 0x7FFF), got.astype(np.int32) & 0x7FFF)
        ib = np.where(ref & 0x8000, -(ref.astype(np.int32) & 0x7FFF), ref.astype(np.int32) & 0x7FFF)
        # fp32 sin/cos within an ulp of the correctly rounded value: at most one bf16 step apart
        assert np.abs(ia - ib).max() <= 1
        assert (got == ref).mean() > 0.999
