"""The oracle's joint-bilateral upsample (oracle/ops.c or_bilateral) against the
closed forms of refBilateralUpsample (src/model/reference.ts:314-353): a
constant low-resolution map is reproduced exactly, and a guide whose
luminance is constant, or a vertical step, turns the upsample into a
separable normalised 3-tap filter (tests/bilateral_closed_form.py).
Tolerance: the oracle accumulates in double and rounds once to float32, so
it is within one float32 rounding (6e-8 relative) of the closed form."""
import numpy as np
import pytest

from oracle import reference as R
from tests.bilateral_closed_form import separable_upsample


def _guide(luma_cols, rows):
    """Grey guide (R = G = B) with the given per-column value, 4 channels."""
    g = np.ones((rows, luma_cols.size, 4), np.float32)
    g[..., :3] = luma_cols[None, :, None]
    return g


def _luma_of(v):
    # luminanceOf (reference.ts:270-272) of a grey value, in double
    return 0.2126 * np.float64(v) + 0.7152 * np.float64(v) + 0.0722 * np.float64(v)


@pytest.mark.parametrize("lh", [7, 16, 32])
def test_constant_map_is_reproduced(lh):
    rng = np.random.default_rng(lh)
    low = np.full((lh, lh, 4), 0.37, np.float32)
    guide = rng.random((2 * lh, 2 * lh, 4)).astype(np.float32)
    got = R.bilateral_upsample(low, lh, lh, 4, guide, 2 * lh, 4, 0.12)
    assert np.abs(got - np.float32(0.37)).max() <= 6e-8


@pytest.mark.parametrize("lh", [7, 16])
def test_constant_guide_is_the_spatial_filter(lh):
    rng = np.random.default_rng(100 + lh)
    low = rng.random((lh, lh)).astype(np.float32)
    guide = _guide(np.full(2 * lh, 0.5, np.float32), 2 * lh)
    low4 = np.repeat(low[..., None], 4, axis=2)
    got = R.bilateral_upsample(low4, lh, lh, 4, guide, 2 * lh, 4, 0.12).reshape(2 * lh, 2 * lh)
    want = separable_upsample(low.astype(np.float64))
    assert np.abs(got - want).max() <= 6e-8 * np.abs(want).max()


def test_step_guide_is_the_separable_range_filter():
    lh = 12
    rng = np.random.default_rng(7)
    low = rng.random((lh, lh)).astype(np.float32)
    cols = np.where(np.arange(2 * lh) < 10, 0.2, 0.45).astype(np.float32)
    guide = _guide(cols, 2 * lh)
    low4 = np.repeat(low[..., None], 4, axis=2)
    got = R.bilateral_upsample(low4, lh, lh, 4, guide, 2 * lh, 4, 0.12).reshape(2 * lh, 2 * lh)
    want = separable_upsample(low.astype(np.float64), _luma_of(cols), 0.12)
    assert np.abs(got - want).max() <= 6e-8 * np.abs(want).max()
    # the edge holds: across the step the range weight is exp(-(0.25/0.12)^2/2) ~ 0.11
    flat = separable_upsample(low.astype(np.float64))
    assert np.abs(want - flat).max() > 1e-2
