"""The config-4 light set: 4 point lights seeded uniformly inside the view
frustum (depth 0.5-3 m), colours U[0,1]^3, intensity U[1,5], radius 8 and
shadow 1 (the packLights defaults, lights.ts:89). One mulberry32 stream per
seed, 7 draws per light in the order depth, x, y, r, g, b, intensity.
"""
import math


def _mb32(seed):
    state = seed & 0xFFFFFFFF

    def nxt():
        nonlocal state
        state = (state + 0x6D2B79F5) & 0xFFFFFFFF
        t = state
        t = ((t ^ (t >> 15)) * (t | 1)) & 0xFFFFFFFF
        t ^= (t + ((t ^ (t >> 7)) * (t | 61))) & 0xFFFFFFFF
        return ((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296.0
    return nxt


def config4_lights(seed, aspect, fov_y, count=4):
    rand = _mb32(seed)
    t = math.tan(fov_y / 2)
    out = []
    for _ in range(count):
        d = 0.5 + 2.5 * rand()
        x = (rand() * 2 - 1) * aspect * t * d
        y = (rand() * 2 - 1) * t * d
        col = (rand(), rand(), rand())
        out.append(dict(kind="point", position=(x, y, -d), color=col, intensity=1 + 4 * rand(), radius=8, shadow=1))
    return out
