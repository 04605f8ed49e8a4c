"""Seeded synthetic frames on the host (oracle/frames.c, ops.c).

TEST INFRASTRUCTURE ONLY: the checker of the device frame generators and the
input of the timed CPU baseline.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import lib


def _f(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def uniform_frame(seed: int, size: int) -> np.ndarray:
    """[3][S][S] float32(mulberry32) values of one seed, (c, y, x) order."""
    out = np.empty((3, size, size), np.float32)
    lib().or_uniform_frame(seed, out.size, _f(out))
    return out


def blob_frame(seed: int, size: int) -> np.ndarray:
    """[3][S][S] smooth procedural frame of one seed: 8 anisotropic Gaussian
    blobs per channel plus N(0, 0.02) noise, clamped to [0, 1]."""
    out = np.empty((3, size, size), np.float32)
    lib().or_blob_frame(seed, size, _f(out))
    return out


def frame(kind: int, seed: int, size: int) -> np.ndarray:
    """kind 0 = uniform, 1 = blobs (illumina_generate_frames' kinds)."""
    return blob_frame(seed, size) if kind == 1 else uniform_frame(seed, size)
