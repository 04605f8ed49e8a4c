"""Closed forms of the joint-bilateral upsample (refBilateralUpsample,
src/model/reference.ts:314-353) for guides whose luminance is constant or a
vertical step.

Output pixel (x, y) of the 2x map has the low-resolution centre
c = ((x + 0.5) / 2 - 0.5, (y + 0.5) / 2 - 0.5) and reads the 3 x 3 taps
q = floor(c + 0.5) + (-1, 0, 1), each coordinate clamped to the map (a clamped
tap counts once per offset that lands on it). The weight of a tap is
exp(-|q - c|^2 / 2) * exp(-(luma(x, y) - luma(2q))^2 / (2 sigma^2)). When the
guide's luminance depends on x only, both factors split into an x part and a
y part, so the upsample is a separable, normalised 3-tap filter:

    out = sum_ab wy[y,a] wx[x,b] low[qy(y,a), qx(x,b)] / (sum_a wy[y,a] sum_b wx[x,b]).
"""
import numpy as np


def taps(n_out: int, n_low: int):
    """Per output coordinate: the 3 clamped tap indices and their spatial weights."""
    x = np.arange(n_out, dtype=np.float64)
    c = (x + 0.5) * 0.5 - 0.5
    b = np.floor(c + 0.5).astype(np.int64)
    q = np.clip(b[:, None] + np.array([-1, 0, 1])[None, :], 0, n_low - 1)
    w = np.exp(-((q - c[:, None]) ** 2) * 0.5)
    return q, w


def separable_upsample(low: np.ndarray, col_luma=None, sigma: float = 0.12) -> np.ndarray:
    """low [lh, lw] float64; col_luma [2 lw] (guide luminance per column) or
    None for a constant guide. Returns the [2 lh, 2 lw] upsample."""
    lh, lw = low.shape
    qy, wy = taps(2 * lh, lh)
    qx, wx = taps(2 * lw, lw)
    if col_luma is not None:
        here = col_luma[:, None]
        there = col_luma[2 * qx]
        wx = wx * np.exp(-(((here - there) / max(sigma, 1e-4)) ** 2) * 0.5)
    g = low[qy[:, :, None, None], qx[None, None, :, :]]  # [Y, 3, X, 3]
    num = np.einsum("ya,yaxb,xb->yx", wy, g, wx)
    return num / (wy.sum(1)[:, None] * wx.sum(1)[None, :])
