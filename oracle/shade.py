"""Oracle wrappers for the shading restatement (oracle/shade.c), plus the
host-side packing of lights and settings it needs: packLights
(src/lighting/lights.ts:178-206) and Renderer.update
(src/lighting/renderer.ts:206-231).

TEST INFRASTRUCTURE ONLY.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import lib
from ._sigs import Light, ShadeParams, Steps

MAX_LIGHTS = 8
KIND = {"point": 0, "spot": 1, "directional": 2}
DEBUG_IDS = {"lit": 0, "depth": 1, "normals": 2, "occlusion": 3, "albedo": 4}

DEFAULT_SETTINGS = dict(
    fovY=58 * math.pi / 180, near=0.35, far=14.0, aoStrength=0.85, shadowStrength=0.8,
    volumetric=0.35, exposure=1.15, ambient=(0.16, 0.2, 0.3), ambientIntensity=0.5,
    roughness=0.55, fogDensity=0.028, fogColor=(0.05, 0.07, 0.12), specular=0.6,
    normalStrength=1.0, albedoMix=1.0, contactShadowLength=0.8, aoRadiusPixels=14,
    toneMap="aces", contrast=1.04, saturation=1.06, vignette=0.35, debug="lit")

REFERENCE_STEPS = (12, 6, 4, 10)


def pack_lights(lights):
    """packLights (lights.ts:178-206) -> ctypes array of 8 Light."""
    if len(lights) > MAX_LIGHTS:
        raise ValueError(f"packLights: {len(lights)} lights exceeds the maximum of {MAX_LIGHTS}")
    arr = (Light * MAX_LIGHTS)()
    for i in range(MAX_LIGHTS):
        if i >= len(lights):
            arr[i].direction[:] = [0, 0, -1, -1]
            continue
        l = lights[i]
        d = l.get("direction", (0, 0, -1))
        n = math.hypot(*d) or 1
        d = [d[0] / n, d[1] / n, d[2] / n]
        outer_a = l.get("outerAngle", math.pi / 5)
        inner_a = min(l.get("innerAngle", math.pi / 8), l.get("outerAngle", math.pi / 5))
        p = l["position"]
        c = l["color"]
        arr[i].position[:] = [p[0], p[1], p[2], 1]
        arr[i].color[:] = [c[0], c[1], c[2], l["intensity"]]
        arr[i].direction[:] = [d[0], d[1], d[2], math.cos(outer_a)]
        arr[i].params[:] = [KIND[l["kind"]], math.cos(inner_a), l.get("radius", 8), l.get("shadow", 1)]
    return arr


def pack_params(s: dict, frame: int, width: int, height: int, depth_w: int, depth_h: int):
    """Renderer.update (renderer.ts:206-231) -> ShadeParams (+ composite grade)."""
    P = ShadeParams()
    P.camera[:] = [math.tan(s["fovY"] / 2), width / height, s["near"], s["far"]]
    P.toggles[:] = [s["aoStrength"], s["shadowStrength"], s["volumetric"], s["exposure"]]
    P.ambient[:] = [*s["ambient"], s["ambientIntensity"]]
    P.misc[:] = [frame % 4096, s["roughness"], s["fogDensity"], s["normalStrength"]]
    P.fog[:] = [*s["fogColor"], s["specular"]]
    P.size[:] = [width, height, depth_w, depth_h]
    P.debug[:] = [DEBUG_IDS[s["debug"]], s["albedoMix"], s["contactShadowLength"], s["aoRadiusPixels"]]
    P.grade[:] = [0 if s["toneMap"] == "aces" else 1, s["contrast"], s["saturation"], s["vignette"]]
    return P


def shade(depth, dw, dh, albedo_planar, aw, ah, lights, params, out_w, out_h,
          steps=REFERENCE_STEPS, rows=None):
    """Scalar shading + composite. Returns (hdr[out_h,out_w,4] f32, rgba8[out_h,out_w,4] u8).

    `rows` restricts the work to a row range (r0, r1) for sampled timing.
    """
    depth = np.ascontiguousarray(depth, np.float32)
    alb = np.ascontiguousarray(albedo_planar, np.float32)
    hdr = np.zeros((out_h, out_w, 4), np.float32)
    rgba = np.zeros((out_h, out_w, 4), np.uint8)
    st = Steps(*steps)
    r0, r1 = rows if rows else (0, out_h)
    f = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))  # noqa: E731
    lib().or_shade(f(depth), dw, dh, f(alb), aw, ah, lights, MAX_LIGHTS, C.byref(params),
                   C.byref(st), out_w, out_h, r0, r1, f(hdr),
                   rgba.ctypes.data_as(C.POINTER(C.c_uint8)))
    return hdr, rgba


def resize_bilinear(src, sw, sh, dw, dh):
    src = np.ascontiguousarray(src, np.float32)
    dst = np.empty(dw * dh, np.float32)
    f = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))  # noqa: E731
    lib().or_resize_bilinear(f(src), sw, sh, f(dst), dw, dh)
    return dst
