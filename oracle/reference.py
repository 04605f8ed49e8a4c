"""Oracle forward pass: forwardReference (src/model/reference.ts:360-451) over
the C restatements of each op (oracle/ops.c).

TEST INFRASTRUCTURE ONLY.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import lib
from .arch import Architecture

ACT = {"linear": 0, "relu": 1, "relu6": 2, "hardswish": 3}


def _f(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _c(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def out_extent(n: int, k: int, stride: int) -> int:
    return lib().or_out_extent(n, k, stride)


def pointwise(src, h, w, in_c, weights, bias, out_c, act, residual=None):
    """refPointwise (reference.ts:35-57); src (h*w*inC) channels-last."""
    src, weights, bias = _c(src), _c(weights), _c(bias)
    out = np.empty(h * w * out_c, np.float32)
    res = _c(residual) if residual is not None else None
    lib().or_pointwise(_f(src), h * w, in_c, _f(weights), _f(bias), out_c, ACT[act],
                       _f(res) if res is not None else None, _f(out))
    return out


def conv(src, h, w, in_c, weights, bias, out_c, k, stride, act):
    """refConv (reference.ts:60-96)."""
    src, weights, bias = _c(src), _c(weights), _c(bias)
    oh, ow = out_extent(h, k, stride), out_extent(w, k, stride)
    out = np.empty(oh * ow * out_c, np.float32)
    lib().or_conv(_f(src), h, w, in_c, _f(weights), _f(bias), out_c, k, stride, ACT[act], _f(out))
    return out, oh, ow


def depthwise(src, h, w, c, weights, bias, k, stride, act):
    """refDepthwise (reference.ts:99-131)."""
    src, weights, bias = _c(src), _c(weights), _c(bias)
    oh, ow = out_extent(h, k, stride), out_extent(w, k, stride)
    out = np.empty(oh * ow * c, np.float32)
    lib().or_depthwise(_f(src), h, w, c, _f(weights), _f(bias), k, stride, ACT[act], _f(out))
    return out, oh, ow


def dwpw(src, h, w, in_c, dw_w, dw_b, mid_act, pw_w, pw_b, out_c, k, stride, act, residual=None):
    """refDepthwisePointwise (reference.ts:138-153)."""
    src, dw_w, dw_b, pw_w, pw_b = map(_c, (src, dw_w, dw_b, pw_w, pw_b))
    oh, ow = out_extent(h, k, stride), out_extent(w, k, stride)
    out = np.empty(oh * ow * out_c, np.float32)
    res = _c(residual) if residual is not None else None
    rc = lib().or_dwpw(_f(src), h, w, in_c, _f(dw_w), _f(dw_b), ACT[mid_act], _f(pw_w), _f(pw_b),
                       out_c, k, stride, ACT[act], _f(res) if res is not None else None, _f(out))
    if rc != 0:
        raise MemoryError("or_dwpw")
    return out, oh, ow


def upsample2(src, h, w, c):
    """refUpsample2 (reference.ts:161-193)."""
    src = _c(src)
    out = np.empty(4 * h * w * c, np.float32)
    lib().or_upsample2(_f(src), h, w, c, _f(out))
    return out


def lateral(coarse, ch, cw, coarse_c, skip, skip_c, weights, bias, out_c, act):
    """refLateral (reference.ts:202-231)."""
    coarse, skip, weights, bias = map(_c, (coarse, skip, weights, bias))
    out = np.empty(4 * ch * cw * out_c, np.float32)
    rc = lib().or_lateral(_f(coarse), ch, cw, coarse_c, _f(skip), 2 * ch, 2 * cw, skip_c,
                          _f(weights), _f(bias), out_c, ACT[act], _f(out))
    if rc == -1:
        raise ValueError(f"refLateral: coarse has {coarse_c} channels, output has {out_c}")
    if rc != 0:
        raise ValueError("refLateral: shape mismatch")
    return out


def head(src, pixels, c, weights, bias):
    """refHead (reference.ts:241-257): 4-channel broadcast disparity."""
    src, weights = _c(src), _c(weights)
    out = np.empty(pixels * 4, np.float32)
    lib().or_head(_f(src), pixels, c, _f(weights), float(bias), _f(out))
    return out


def head_logit(src, pixels, c, weights, bias):
    src, weights = _c(src), _c(weights)
    out = np.empty(pixels, np.float64)
    lib().or_head_logit(_f(src), pixels, c, _f(weights), float(bias),
                        out.ctypes.data_as(C.POINTER(C.c_double)))
    return out


def preprocess(rgba, size, mean, std, decode_srgb=True, exposure=1.0):
    """refPreprocess (reference.ts:283-308): rgba (size*size*4) -> (input, sceneColor)."""
    rgba = _c(rgba)
    inp = np.empty(size * size * 4, np.float32)
    scene = np.empty(size * size * 4, np.float32)
    m = np.array(mean, np.float64)
    s = np.array(std, np.float64)
    lib().or_preprocess(_f(rgba), size, m.ctypes.data_as(C.POINTER(C.c_double)),
                        s.ctypes.data_as(C.POINTER(C.c_double)), 1 if decode_srgb else 0,
                        float(exposure), _f(inp), _f(scene))
    return inp, scene


def bilateral_upsample(low, lh, lw, lc, guide, gw, gc, range_sigma):
    """refBilateralUpsample (reference.ts:314-353): returns (2lh)*(2lh) f32."""
    low, guide = _c(low), _c(guide)
    out = np.empty(4 * lh * lh, np.float32)
    lib().or_bilateral(_f(low), lh, lw, lc, _f(guide), gw, gc, float(range_sigma), _f(out))
    return out


def rgb_planar_to_rgba(rgb, size):
    """[3][S][S] planar frame -> S*S*4 interleaved (alpha 1), the refPreprocess input."""
    rgb = np.asarray(rgb, np.float32).reshape(3, size, size)
    out = np.ones((size, size, 4), np.float32)
    out[..., :3] = np.transpose(rgb, (1, 2, 0))
    return out.ravel()


def forward_reference(arch: Architecture, weights: dict, inp) -> dict:
    """forwardReference (reference.ts:360-451): every intermediate by tensor name.

    Like the reference it does not run bilateralUp (reference.ts:445-447).
    """
    values = {"input": _c(inp)}
    sh = arch.tensors

    def w(k):
        v = weights.get(k)
        if v is None:
            raise KeyError(f"forwardReference: missing weight {k}")
        return v

    for op in arch.ops:
        if op.kind in ("preprocess", "bilateralUp"):
            continue
        o = sh[op.out]
        if op.kind == "conv":
            i = sh[op.inp]
            values[op.out], _, _ = conv(values[op.inp], i.h, i.w, i.c, w(f"{op.name}.weight"),
                                        w(f"{op.name}.bias"), o.c, op.k, op.stride, op.act)
        elif op.kind == "pw":
            i = sh[op.inp]
            values[op.out] = pointwise(values[op.inp], i.h, i.w, i.c, w(f"{op.name}.weight"),
                                       w(f"{op.name}.bias"), o.c, op.act,
                                       values[op.residual] if op.residual else None)
        elif op.kind == "dwpw":
            i = sh[op.inp]
            values[op.out], _, _ = dwpw(values[op.inp], i.h, i.w, i.c, w(f"{op.name}.dw_weight"),
                                        w(f"{op.name}.dw_bias"), op.mid_act,
                                        w(f"{op.name}.pw_weight"), w(f"{op.name}.pw_bias"), o.c,
                                        op.k, op.stride, op.act,
                                        values[op.residual] if op.residual else None)
        elif op.kind == "lateral":
            c, s = sh[op.coarse], sh[op.skip]
            values[op.out] = lateral(values[op.coarse], c.h, c.w, c.c, values[op.skip], s.c,
                                     w(f"{op.name}.weight"), w(f"{op.name}.bias"), o.c, op.act)
        elif op.kind == "head":
            i = sh[op.inp]
            values[op.out] = head(values[op.inp], i.h * i.w, i.c, w(f"{op.name}.weight"),
                                  w(f"{op.name}.bias")[0])
    return values


def forward_frame(arch: Architecture, weights: dict, rgb_planar, decode_srgb=True, exposure=1.0,
                  range_sigma=0.12):
    """Whole hot path for one [3][S][S] frame: preprocess -> 38 convs -> head -> bilateralUp.

    Returns (values, disparity[S*S]) where values holds every intermediate plus
    'scene_color'.
    """
    S = arch.input_size
    rgba = rgb_planar_to_rgba(rgb_planar, S)
    inp, scene = preprocess(rgba, S, arch.mean, arch.std, decode_srgb, exposure)
    values = forward_reference(arch, weights, inp)
    values["scene_color"] = scene
    low = arch.tensors["depth_low"]
    disp = bilateral_upsample(values["depth_low"], low.h, low.w, 4, scene, S, 4, range_sigma)
    return values, disp
