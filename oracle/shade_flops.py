"""Algorithmic FLOPs per pixel of the depth-aware shading + tone-map pass for
the 1920x1080 relighting frame, from the op-counting build of the shading
restatement (oracle/shade_count.cpp: + - * / compare min max floor fabs = 1,
fused multiply-add = 2, sqrt exp pow sin cos = 1 each).

MEASUREMENT INFRASTRUCTURE ONLY (run here, its output committed):

    python -m oracle.shade_flops > profiles/shade_flops_1080p.json

The frame: the network's disparity for the uniform 448 frame of seed 0
(oracle forward, seed-0 weights), bilinearly upsampled to 1920x1080; albedo =
the frame's RGB; 4 point lights seeded inside the view frustum (seed 0: depth
U[0.5, 3], x/y inside the frustum at that depth, colour U[0,1]^3, intensity
U[1, 5], radius 8, shadow 1); DEFAULT_SETTINGS, frame index 0. Two step
settings: the reference's constants (12 contact, 6x4 AO, 10 volumetric per
light) and the benchmark's (16 contact, 6x4 AO, 12 volumetric per light).
"""
from __future__ import annotations

import ctypes as C
import json
import math
import os

import numpy as np

from . import arch as OA
from . import frames as OF
from . import reference as R
from . import weights as OW
from .shade import DEFAULT_SETTINGS, MAX_LIGHTS, pack_lights, pack_params
from ._sigs import Light, ShadeParams, Steps

W, H, S = 1920, 1080, 448
MODES = {"reference_constants": (12, 6, 4, 10), "benchmark": (16, 6, 4, 12)}


def _lights(seed, aspect, fov_y, count=4):
    """4 point lights inside the view frustum from one mulberry32 stream, 7 draws
    each (depth, x, y, r, g, b, intensity)."""
    state = seed & 0xFFFFFFFF

    def rnd():
        nonlocal state
        state = (state + 0x6D2B79F5) & 0xFFFFFFFF
        t = state
        t = ((t ^ (t >> 15)) * (t | 1)) & 0xFFFFFFFF
        t ^= (t + ((t ^ (t >> 7)) * (t | 61))) & 0xFFFFFFFF
        return ((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296.0

    tn = math.tan(fov_y / 2)
    out = []
    for _ in range(count):
        d = 0.5 + 2.5 * rnd()
        x = (rnd() * 2 - 1) * aspect * tn * d
        y = (rnd() * 2 - 1) * tn * d
        col = (rnd(), rnd(), rnd())
        out.append(dict(kind="point", position=(x, y, -d), color=col, intensity=1 + 4 * rnd(), radius=8, shadow=1))
    return out


def _count_lib():
    here = os.path.dirname(os.path.abspath(__file__))
    path = os.path.join(here, "liboracle_count.so")
    if not os.path.exists(path):
        import subprocess
        subprocess.run(["make", "-s", "-C", here], check=True)
    lib = C.CDLL(path)
    F = C.POINTER(C.c_float)
    lib.or_shade_flops.restype = C.c_double
    lib.or_shade_flops.argtypes = [F, C.c_int, C.c_int, F, C.c_int, C.c_int, C.POINTER(Light), C.c_int,
                                   C.POINTER(ShadeParams), C.POINTER(Steps), C.c_int, C.c_int, C.c_int, C.c_int]
    return lib


def frame_inputs():
    a = OA.build_architecture(S)
    rgb = OF.uniform_frame(0, S)
    _, disp = R.forward_frame(a, OW.synthesize_weights(a, 0), rgb)
    from .shade import resize_bilinear
    depth = resize_bilinear(disp, S, S, W, H)
    return depth, np.ascontiguousarray(rgb, np.float32)


def flops_per_pixel(depth, albedo, steps):
    lib = _count_lib()
    lights = pack_lights(_lights(0, W / H, DEFAULT_SETTINGS["fovY"]))
    P = pack_params(DEFAULT_SETTINGS, 0, W, H, W, H)
    st = Steps(*steps)
    f = lambda x: x.ctypes.data_as(C.POINTER(C.c_float))  # noqa: E731
    return lib.or_shade_flops(f(depth), W, H, f(albedo), S, S, lights, MAX_LIGHTS, C.byref(P), C.byref(st), W, H, 0, H)


def main():
    depth, albedo = frame_inputs()
    out = {"what": "algorithmic FLOPs per shaded pixel (shading + tone-map), 1920x1080 relighting frame",
           "rules": "+ - * / compare min max floor fabs = 1, fma = 2, sqrt exp pow sin cos = 1",
           "frame": "uniform 448 frame seed 0 -> oracle forward (seed-0 weights) -> bilinear 1920x1080; "
                    "albedo = frame RGB; 4 seeded point lights; DEFAULT_SETTINGS; frame index 0",
           "command": "python -m oracle.shade_flops"}
    for name, steps in MODES.items():
        out[name] = {"steps": {"contact": steps[0], "ao_dirs": steps[1], "ao_steps": steps[2],
                               "volumetric_per_light": steps[3]},
                     "flops_per_pixel": round(flops_per_pixel(depth, albedo, steps), 1)}
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
