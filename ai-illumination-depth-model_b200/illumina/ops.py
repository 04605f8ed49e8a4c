"""Per-kernel entry points: the analogues of the reference's kernel factories
(makePointwise, makeDepthwisePointwise, makeConv, makeLateral, makeHead,
makePreprocess, makeDepthUpsample under src/model/kernels/). Arguments are
torch CUDA tensors in the reference's logical layouts; each call launches the
same CUDA kernel the model uses.
"""
from __future__ import annotations

from ._lib import ACT, ENGINE, check, lib, ptr, stream_handle


def set_engine(engine: str) -> None:
    """Engine of this thread's pointwise / dw->pw / lateral entry points: "simt" (default) or "tensor"."""
    check(lib().illumina_set_op_engine(ENGINE[engine]))


def _out(torch, shape, like):
    return torch.empty(shape, dtype=torch.float32, device=like.device)


def pointwise(src, h, w, in_c, weights, bias, out_c, act, residual=None, dst=None, stream=None):
    import torch
    dst = dst if dst is not None else _out(torch, (h * w * out_c,), src)
    check(lib().illumina_op_pointwise(ptr(src), h * w, in_c, ptr(weights), ptr(bias), out_c, ACT[act],
                                      ptr(residual), ptr(dst), stream_handle(stream)))
    return dst


def dwpw(src, in_h, in_w, in_c, dw_w, dw_b, mid_act, pw_w, pw_b, out_c, k, stride, act, residual=None, dst=None,
         stream=None):
    import torch
    pad = (k - 1) >> 1
    oh, ow = (in_h + 2 * pad - k) // stride + 1, (in_w + 2 * pad - k) // stride + 1
    dst = dst if dst is not None else _out(torch, (oh * ow * out_c,), src)
    check(lib().illumina_op_dwpw(ptr(src), in_h, in_w, in_c, ptr(dw_w), ptr(dw_b), ACT[mid_act], ptr(pw_w),
                                 ptr(pw_b), out_c, k, stride, ACT[act], ptr(residual), ptr(dst),
                                 stream_handle(stream)))
    return dst


def conv(src, in_h, in_w, in_c, weights, bias, out_c, k, stride, act, dst=None, stream=None):
    import torch
    pad = (k - 1) >> 1
    oh, ow = (in_h + 2 * pad - k) // stride + 1, (in_w + 2 * pad - k) // stride + 1
    dst = dst if dst is not None else _out(torch, (oh * ow * out_c,), src)
    check(lib().illumina_op_conv(ptr(src), in_h, in_w, in_c, ptr(weights), ptr(bias), out_c, k, stride, ACT[act],
                                 ptr(dst), stream_handle(stream)))
    return dst


def lateral(coarse, ch, cw, skip, skip_c, weights, bias, out_c, act, dst=None, stream=None):
    import torch
    dst = dst if dst is not None else _out(torch, (4 * ch * cw * out_c,), coarse)
    check(lib().illumina_op_lateral(ptr(coarse), ch, cw, ptr(skip), skip_c, ptr(weights), ptr(bias), out_c,
                                    ACT[act], ptr(dst), stream_handle(stream)))
    return dst


def head(src, pixels, in_c, weights, bias, dst=None, stream=None):
    import torch
    dst = dst if dst is not None else _out(torch, (pixels * 4,), src)
    check(lib().illumina_op_head(ptr(src), pixels, in_c, ptr(weights), float(bias), ptr(dst),
                                 stream_handle(stream)))
    return dst


def preprocess(frames, n, layout, size, decode_srgb=True, exposure=1.0, scene=True, stream=None):
    import torch
    inp = _out(torch, (n * size * size * 4,), frames)
    sc = _out(torch, (n * size * size * 4,), frames) if scene else None
    check(lib().illumina_op_preprocess(ptr(frames), n, layout, size, 1 if decode_srgb else 0, float(exposure),
                                       ptr(inp), ptr(sc), stream_handle(stream)))
    return inp, sc


def bilateral(low, lh, lw, low_c, guide, guide_c, range_sigma=0.12, dst=None, stream=None):
    import torch
    dst = dst if dst is not None else _out(torch, (4 * lh * lw,), low)
    check(lib().illumina_op_bilateral(ptr(low), lh, lw, low_c, ptr(guide), guide_c, float(range_sigma), ptr(dst),
                                      stream_handle(stream)))
    return dst
