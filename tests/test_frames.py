"""Seeded synthetic frames: the host generator (the checker of the device one)
against the workload definition, on the CPU.

The blob frame of a seed is, per channel, 8 anisotropic Gaussian blobs with
centres uniform in the image, sigma 20-120 px, rotation uniform in [0, pi) and
amplitude uniform in [0, 1], plus N(0, 0.02) Box-Muller noise, clamped to
[0, 1], all drawn from the seed's mulberry32 stream (src/model/weights.ts:200-216
for the generator and the transform). The generator evaluates it with
series-defined exp/log/sin/cos in IEEE double so that the device generator can
reproduce it bit for bit; here it is compared with numpy's libm evaluation.
"""
import math

import numpy as np
import pytest

from oracle import frames, lib


def mb32_at(seed, j):
    t = (seed + (j + 1) * 0x6D2B79F5) & 0xFFFFFFFF
    t = ((t ^ (t >> 15)) * (t | 1)) & 0xFFFFFFFF
    t ^= (t + ((t ^ (t >> 7)) * (t | 61) & 0xFFFFFFFF)) & 0xFFFFFFFF
    return (t ^ (t >> 14)) / 4294967296.0


def blob_frame_numpy(seed, S):
    """The workload definition with numpy's exp/log/cos/sin (float64)."""
    out = np.zeros((3, S, S))
    y, x = np.mgrid[0:S, 0:S].astype(np.float64)
    px, py = x + 0.5, y + 0.5
    for c in range(3):
        v = np.zeros((S, S))
        for b in range(8):
            d = (c * 8 + b) * 6
            cx, cy = mb32_at(seed, d) * S, mb32_at(seed, d + 1) * S
            sx, sy = 20 + 100 * mb32_at(seed, d + 2), 20 + 100 * mb32_at(seed, d + 3)
            th, amp = math.pi * mb32_at(seed, d + 4), mb32_at(seed, d + 5)
            dx, dy = px - cx, py - cy
            u = math.cos(th) * dx + math.sin(th) * dy
            w = -math.sin(th) * dx + math.cos(th) * dy
            v += amp * np.exp(-(u * u / (2 * sx * sx) + w * w / (2 * sy * sy)))
        j = (c * S + y.astype(np.int64)) * S + x.astype(np.int64)
        uu = np.array([mb32_at(seed, 144 + 2 * int(k)) for k in j.ravel()]).reshape(S, S)
        vv = np.array([mb32_at(seed, 145 + 2 * int(k)) for k in j.ravel()]).reshape(S, S)
        g = np.sqrt(-2 * np.log(np.maximum(uu, 1e-9))) * np.cos(2 * math.pi * vv)
        out[c] = np.clip(v + 0.02 * g, 0, 1)
    return out


def test_mb32_at_matches_the_sequential_stream():
    import ctypes as C
    seq = np.empty(50, np.float64)
    lib().or_mulberry32(12345, 50, seq.ctypes.data_as(C.POINTER(C.c_double)))
    assert [mb32_at(12345, j) for j in range(50)] == list(seq)


def test_series_functions_match_libm():
    L = lib()
    rng = np.random.default_rng(1)
    for x in np.concatenate([-rng.random(4000) * 700, -rng.random(1000) * 1e-3, [0.0, -1e-300, -707.9]]):
        want = math.exp(x)
        assert abs(L.or_det_exp(x) - want) <= 4e-16 * want, x
    assert L.or_det_exp(-709.0) == 0.0
    for u in np.concatenate([rng.random(4000), [1e-9, 0.5, 1 - 2 ** -32, 2 ** -32]]):
        u = max(u, 1e-9)
        assert abs(L.or_det_log(u) - math.log(u)) <= 2e-15 * max(1.0, abs(math.log(u))), u
    import ctypes as C
    s, c = C.c_double(), C.c_double()
    for v in np.concatenate([np.floor(rng.random(4000) * 2 ** 32) / 2 ** 32, [0.0, 0.25, 0.5, 0.75]]):
        assert abs(L.or_det_cos2pi(v) - math.cos(2 * math.pi * v)) <= 2e-15, v
        th = v * math.pi
        L.or_det_sincos(th, C.byref(s), C.byref(c))
        assert abs(s.value - math.sin(th)) <= 2e-15 and abs(c.value - math.cos(th)) <= 2e-15, th


@pytest.mark.parametrize("seed,size", [(0, 64), (7, 48), (255, 37)])
def test_blob_frame_is_the_workload_definition(seed, size):
    got = frames.blob_frame(seed, size).astype(np.float64)
    want = blob_frame_numpy(seed, size)
    # the two differ only by the last bits of the float64 functions, which the
    # float32 rounding absorbs except at rounding ties: within one float32 ulp
    assert np.abs(got - want).max() <= 6e-8
    assert (got == np.float32(want)).mean() > 0.999


def test_blob_frames_statistics():
    """Smooth images in [0, 1]: neighbouring pixels are close (blobs of sigma >=
    20 px), the noise is N(0, 0.02), frames of different seeds differ."""
    f0, f1 = frames.blob_frame(0, 448), frames.blob_frame(1, 448)
    assert f0.min() >= 0 and f0.max() <= 1 and not np.array_equal(f0, f1)
    inner = (f0 > 0.1) & (f0 < 0.9)
    d = np.diff(f0.astype(np.float64), axis=2)[inner[:, :, 1:] & inner[:, :, :-1]]
    # difference of two independent N(0, 0.02) samples plus a small smooth slope
    assert 0.025 < d.std() < 0.035 and abs(d.mean()) < 2e-3
