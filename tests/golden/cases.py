"""Per-kernel parity cases and their seeded inputs.

The case lists follow the reference's own kernel tests
(test/kernels.test.ts:34-49, :137-156, :208-212, :250-254 and
test/shapes.test.ts:24-39, :94-101, :128-134, :162-168), and the inputs are
drawn exactly as those tests draw them: one mulberry32 stream per case, seeded
as in the test, consumed by `randomFloats` in the test's order
(test/helpers/tensors.ts:6-22).

Test infrastructure: drawing uses the oracle's integer-exact PRNG.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

import oracle

NET64_SEED = 20240819          # test/network.test.ts:48
PREPROCESS_EXPOSURE = 1.3       # test/kernels.test.ts preprocess case
KERNEL_TOL = (2e-4, 2e-3)       # test/helpers/tensors.ts:81-105 default (abs, rel)
SHAPES_TOL = (3e-4, 3e-3)       # test/shapes.test.ts:21


def _pad_out(n, k, s):
    pad = (k - 1) >> 1
    return (n + 2 * pad - k) // s + 1


def all_cases():
    out = []
    # kernels.test.ts pointwise
    for i, (h, w, ic, oc, act, res) in enumerate([
            (16, 16, 32, 32, "relu6", False), (13, 17, 12, 8, "hardswish", False),
            (7, 9, 20, 12, "linear", True), (8, 8, 24, 96, "hardswish", False),
            (14, 14, 704, 176, "linear", True), (5, 5, 8, 4, "relu", False)]):
        out.append(dict(id=f"k_pw{i}", kind="pw", h=h, w=w, inC=ic, outC=oc, act=act, residual=res,
                        seed=0xC0FFEE ^ (ic * 131 + oc), scales=(1, 0.25, 0.5, 1), tol=KERNEL_TOL))
    # kernels.test.ts dwpw
    for i, (ih, iw, ic, oc, k, s, ma, a, res) in enumerate([
            (12, 12, 16, 24, 3, 1, "relu6", "linear", False),
            (16, 16, 24, 96, 3, 2, "linear", "hardswish", False),
            (14, 14, 32, 128, 5, 2, "linear", "hardswish", False),
            (8, 8, 224, 56, 5, 1, "hardswish", "linear", True),
            (6, 6, 704, 176, 5, 1, "hardswish", "linear", True),
            (13, 11, 48, 48, 3, 1, "hardswish", "hardswish", True),
            (15, 13, 104, 416, 5, 2, "linear", "hardswish", False)]):
        out.append(dict(id=f"k_dwpw{i}", kind="dwpw", inH=ih, inW=iw, inC=ic, outC=oc, k=k, stride=s,
                        midAct=ma, act=a, residual=res, seed=0xBEEF ^ (ic * 31 + oc * 7 + k),
                        scales=(1, 0.5, 0.3, 0.2, 0.3, 1), tol=KERNEL_TOL))
    # kernels.test.ts conv
    for i, (ih, iw, ic, oc, k, s, a) in enumerate([
            (32, 32, 4, 16, 3, 2, "hardswish"), (9, 11, 8, 12, 3, 1, "relu6"),
            (15, 13, 4, 32, 5, 2, "linear")]):
        out.append(dict(id=f"k_conv{i}", kind="conv", inH=ih, inW=iw, inC=ic, outC=oc, k=k, stride=s,
                        act=a, seed=0x5EED ^ (oc * 17 + k), scales=(1, 0.3, 0.4), tol=KERNEL_TOL))
    # kernels.test.ts lateral
    for i, (ch, cw, oc, sc, a) in enumerate([
            (7, 7, 96, 104, "linear"), (4, 4, 32, 24, "hardswish"), (5, 3, 48, 32, "linear")]):
        out.append(dict(id=f"k_lat{i}", kind="lateral", ch=ch, cw=cw, outC=oc, skipC=sc, act=a,
                        seed=0xFEED ^ (oc * 13 + sc), scales=(1, 1, 0.25, 0.4), tol=KERNEL_TOL))
    # shapes.test.ts dwpw (midAct hardswish, act relu6)
    for i, (ih, iw, ic, oc, k, s, res) in enumerate([
            (1, 1, 20, 12, 3, 1, False), (1, 1, 36, 4, 5, 2, False), (1, 17, 36, 20, 5, 1, False),
            (17, 1, 12, 44, 3, 2, False), (5, 5, 4, 60, 3, 1, False), (6, 6, 68, 36, 5, 1, False),
            (5, 7, 116, 12, 3, 1, False), (9, 7, 28, 52, 3, 2, False), (7, 9, 52, 28, 5, 2, False),
            (11, 11, 44, 4, 5, 2, False), (14, 14, 704, 176, 5, 1, True),
            (28, 28, 104, 416, 5, 2, False), (224, 224, 24, 96, 3, 2, False),
            (4, 4, 704, 4, 3, 1, False)]):
        out.append(dict(id=f"s_dwpw{i}", kind="dwpw", inH=ih, inW=iw, inC=ic, outC=oc, k=k, stride=s,
                        midAct="hardswish", act="relu6", residual=res,
                        seed=0x1234 ^ (ic * 977 + oc * 13 + k * 5 + s + ih),
                        scales=(1, 0.4, 0.3, 0.1, 0.3, 1), tol=SHAPES_TOL))
    # shapes.test.ts pointwise (hardswish, residual)
    for i, (h, w, ic, oc) in enumerate([
            (1, 1, 704, 4), (1, 1, 4, 704), (1, 37, 68, 36), (1, 101, 116, 12), (14, 14, 176, 704),
            (112, 112, 32, 128)]):
        out.append(dict(id=f"s_pw{i}", kind="pw", h=h, w=w, inC=ic, outC=oc, act="hardswish",
                        residual=True, seed=0x777 ^ (ic * 31 + oc + w), scales=(1, 0.12, 0.4, 1),
                        tol=SHAPES_TOL))
    # shapes.test.ts conv (hardswish)
    for i, (ih, iw, ic, oc, k, s) in enumerate([
            (1, 1, 4, 16, 3, 1), (9, 7, 4, 16, 3, 2), (7, 9, 8, 12, 5, 2), (1, 33, 4, 20, 3, 2),
            (448, 448, 4, 16, 3, 2)]):
        out.append(dict(id=f"s_conv{i}", kind="conv", inH=ih, inW=iw, inC=ic, outC=oc, k=k, stride=s,
                        act="hardswish", seed=0x99 ^ (ih * 7 + iw * 13 + k), scales=(1, 0.2, 0.4),
                        tol=SHAPES_TOL))
    # shapes.test.ts lateral (hardswish)
    for i, (cw, ch, oc, sc) in enumerate([
            (1, 1, 8, 12), (7, 7, 12, 104), (3, 5, 4, 4), (14, 14, 96, 104), (112, 112, 32, 24)]):
        out.append(dict(id=f"s_lat{i}", kind="lateral", ch=ch, cw=cw, outC=oc, skipC=sc,
                        act="hardswish", seed=0xABC ^ (cw * 17 + ch * 3 + oc), scales=(1, 1, 0.2, 0.4),
                        tol=SHAPES_TOL))
    return out


def random_floats(state, n, scale):
    """randomFloats over a shared mulberry32 stream; returns (array, new_state)."""
    out = np.empty(n, np.float32)
    st = oracle.lib().or_random_floats(state & 0xFFFFFFFF, n, float(scale),
                                       out.ctypes.data_as(C.POINTER(C.c_float)))
    return out, st


def draw(case):
    """Draws a case's tensors in the reference test's order."""
    st = case["seed"] & 0xFFFFFFFF
    sc = case["scales"]
    d = {}
    kind = case["kind"]
    if kind == "pw":
        p = case["h"] * case["w"]
        d["src"], st = random_floats(st, p * case["inC"], sc[0])
        d["w"], st = random_floats(st, case["outC"] * case["inC"], sc[1])
        d["b"], st = random_floats(st, case["outC"], sc[2])
        d["res"], st = random_floats(st, p * case["outC"], sc[3])
    elif kind == "dwpw":
        oh, ow = _pad_out(case["inH"], case["k"], case["stride"]), _pad_out(case["inW"], case["k"], case["stride"])
        d["outH"], d["outW"] = oh, ow
        d["src"], st = random_floats(st, case["inH"] * case["inW"] * case["inC"], sc[0])
        d["dw_w"], st = random_floats(st, case["inC"] * case["k"] ** 2, sc[1])
        d["dw_b"], st = random_floats(st, case["inC"], sc[2])
        d["pw_w"], st = random_floats(st, case["outC"] * case["inC"], sc[3])
        d["pw_b"], st = random_floats(st, case["outC"], sc[4])
        d["res"], st = random_floats(st, oh * ow * case["outC"], sc[5])
    elif kind == "conv":
        d["outH"] = _pad_out(case["inH"], case["k"], case["stride"])
        d["outW"] = _pad_out(case["inW"], case["k"], case["stride"])
        d["src"], st = random_floats(st, case["inH"] * case["inW"] * case["inC"], sc[0])
        d["w"], st = random_floats(st, case["outC"] * case["inC"] * case["k"] ** 2, sc[1])
        d["b"], st = random_floats(st, case["outC"], sc[2])
    elif kind == "lateral":
        d["coarse"], st = random_floats(st, case["ch"] * case["cw"] * case["outC"], sc[0])
        d["skip"], st = random_floats(st, 4 * case["ch"] * case["cw"] * case["skipC"], sc[1])
        d["w"], st = random_floats(st, case["outC"] * case["skipC"], sc[2])
        d["b"], st = random_floats(st, case["outC"], sc[3])
    return d


def oracle_output(case, data):
    """The oracle's answer for a case (channels-last flat f32)."""
    from oracle import reference as R
    kind = case["kind"]
    if kind == "pw":
        return R.pointwise(data["src"], case["h"], case["w"], case["inC"], data["w"], data["b"],
                           case["outC"], case["act"], data["res"] if case["residual"] else None)
    if kind == "dwpw":
        out, _, _ = R.dwpw(data["src"], case["inH"], case["inW"], case["inC"], data["dw_w"],
                           data["dw_b"], case["midAct"], data["pw_w"], data["pw_b"], case["outC"],
                           case["k"], case["stride"], case["act"],
                           data["res"] if case["residual"] else None)
        return out
    if kind == "conv":
        out, _, _ = R.conv(data["src"], case["inH"], case["inW"], case["inC"], data["w"], data["b"],
                           case["outC"], case["k"], case["stride"], case["act"])
        return out
    if kind == "lateral":
        return R.lateral(data["coarse"], case["ch"], case["cw"], case["outC"], data["skip"],
                         case["skipC"], data["w"], data["b"], case["outC"], case["act"])
    raise ValueError(kind)


def _mb32_stream(seed):
    state = seed & 0xFFFFFFFF

    def nxt():
        nonlocal state
        state = (state + 0x6D2B79F5) & 0xFFFFFFFF
        t = state
        t = ((t ^ (t >> 15)) * (t | 1)) & 0xFFFFFFFF
        t ^= (t + ((t ^ (t >> 7)) * (t | 61))) & 0xFFFFFFFF
        return ((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296.0
    return nxt


def test_image(size):
    """testImage, test/network.test.ts:27-42 (RGBA bytes, size*size*4)."""
    rand = _mb32_stream(0x1234)
    px = np.zeros(size * size * 4, np.uint8)
    for y in range(size):
        for x in range(size):
            i = (y * size + x) * 4
            disc = (x - size * 0.35) ** 2 + (y - size * 0.4) ** 2 < (size * 0.22) ** 2
            stripe = ((x + y) >> 3) & 1
            px[i] = 230 if disc else math.floor((x / size) * 200 + stripe * 25)
            px[i + 1] = 60 if disc else math.floor((y / size) * 180 + rand() * 20)
            px[i + 2] = 90 if disc else math.floor(120 + math.sin(x * 0.4) * 60)
            px[i + 3] = 255
    return px


def preprocess_image(size):
    """The kernels.test.ts preprocess source: mulberry32(0xa11ce) bytes."""
    rand = _mb32_stream(0xA11CE)
    px = np.zeros(size * size * 4, np.uint8)
    for i in range(0, px.size, 4):
        px[i] = math.floor(rand() * 256)
        px[i + 1] = math.floor(rand() * 256)
        px[i + 2] = math.floor(rand() * 256)
        px[i + 3] = 255
    return px


def rgba_bytes_to_planar(px, size):
    """RGBA bytes -> [3][S][S] float32 in [0,1] (the network's frame format)."""
    a = (px.astype(np.float32) / np.float32(255.0)).reshape(size, size, 4)
    return np.ascontiguousarray(np.transpose(a[..., :3], (2, 0, 1)))
