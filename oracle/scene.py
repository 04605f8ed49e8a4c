"""Oracle wrappers for the procedural scene and depth metrics (oracle/scene.c):
src/scene/procedural.ts (scene uniforms and the fragment shader, restated in
float32) and src/scene/metrics.ts (evaluateDepth, restated in double).

TEST INFRASTRUCTURE ONLY.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import lib

_F = C.POINTER(C.c_float)


def scene_params(time=None, orbit=False):
    """12 floats: camera, focus, options. time None = createProceduralScene's initial uniforms."""
    out = np.zeros(12, np.float32)
    lib().or_scene_params(0.0 if time is None else float(time), int(bool(orbit)), int(time is None),
                          out.ctypes.data_as(_F))
    return out


def render(params, w, h):
    """(rgb [3, h, w] float32 = 8-bit/255, rgba8 [h, w, 4] uint8, truth [h, w, 2] float32)."""
    params = np.ascontiguousarray(params, np.float32)
    rgb = np.empty((3, h, w), np.float32)
    rgba8 = np.empty((h, w, 4), np.uint8)
    truth = np.empty((h, w, 2), np.float32)
    lib().or_scene_render(params.ctypes.data_as(_F), w, h, rgb.ctypes.data_as(_F),
                          rgba8.ctypes.data_as(C.POINTER(C.c_uint8)), truth.ctypes.data_as(_F))
    return rgb, rgba8, truth


METRIC_FIELDS = ("samples", "absRel", "rmse", "delta1", "delta2", "delta3", "scale", "shift")


def evaluate_depth(pred, truth, w, h, pred_channels=1):
    """evaluateDepth (metrics.ts:66-161) -> dict of METRIC_FIELDS."""
    pred = np.ascontiguousarray(pred, np.float32)
    truth = np.ascontiguousarray(truth, np.float32)
    out = np.zeros(8, np.float64)
    lib().or_evaluate_depth(pred.ctypes.data_as(_F), pred_channels, truth.ctypes.data_as(_F), w, h,
                            out.ctypes.data_as(C.POINTER(C.c_double)))
    d = dict(zip(METRIC_FIELDS, out.tolist()))
    d["samples"] = int(d["samples"])
    return d
