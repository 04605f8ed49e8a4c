"""Named tensor bundles ("ntb/1"), the activation-dump format of the
reference's scripts/ref-forward.ts:63-165.

Layout: a little-endian u32 header length, the UTF-8 JSON header
{"format": "ntb/1", "tensors": {name: {"dtype": "f32"|"f16", "shape": [...],
"offset": bytes from the blob start, "length": bytes}}}, then the blob.
Reading accepts f32 and f16 tensors and validates like readBundle
(ref-forward.ts:96-136): truncated file, header outside the file, wrong
format, a length that disagrees with the shape, a tensor past the end.
Writing emits f32 tensors packed in insertion order (writeBundle,
ref-forward.ts:138-165).
"""
from __future__ import annotations

import json
import struct

import numpy as np

BUNDLE_FORMAT = "ntb/1"


def _count(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def readBundle(data: bytes, what: str = "bundle") -> dict:
    """ntb/1 bytes -> {name: float32 numpy array of the tensor's shape} (insertion order kept)."""
    buf = memoryview(data)
    if len(buf) < 4:
        raise ValueError(f"{what}: file is truncated")
    (hlen,) = struct.unpack_from("<I", buf, 0)
    if hlen == 0 or 4 + hlen > len(buf):
        raise ValueError(f"{what}: header length {hlen} does not fit the file")
    header = json.loads(bytes(buf[4:4 + hlen]).decode("utf-8"))
    if header.get("format") != BUNDLE_FORMAT:
        raise ValueError(f"{what}: format {header.get('format')}, expected {BUNDLE_FORMAT}")
    base = 4 + hlen
    out = {}
    for name, info in header.get("tensors", {}).items():
        shape = tuple(int(d) for d in info["shape"])
        count = _count(shape)
        f16 = info.get("dtype") == "f16"
        nbytes = count * (2 if f16 else 4)
        if info["length"] != nbytes:
            raise ValueError(f"{what}: {name} claims {info['length']} bytes, shape needs {nbytes}")
        start = base + int(info["offset"])
        if start + nbytes > len(buf):
            raise ValueError(f"{what}: {name} extends past the end of the file")
        raw = bytes(buf[start:start + nbytes])
        # f16 -> f32 is exact (the reference's halfToFloat)
        arr = np.frombuffer(raw, "<f2" if f16 else "<f4").astype(np.float32)
        out[name] = arr.reshape(shape)
    return out


def writeBundle(tensors: dict) -> bytes:
    """{name: array-like (its shape is the tensor's)} or {name: (shape, values)} -> ntb/1 bytes (f32)."""
    header = {"format": BUNDLE_FORMAT, "tensors": {}}
    parts, offset = [], 0
    for name, t in tensors.items():
        if isinstance(t, tuple):
            shape, values = t
        else:
            values = np.asarray(t)
            shape = values.shape
        raw = np.ascontiguousarray(values, "<f4").ravel()
        if raw.size != _count(shape):
            raise ValueError(f"{name}: shape [{', '.join(str(d) for d in shape)}] needs {_count(shape)} values, "
                             f"got {raw.size}")
        b = raw.tobytes()
        header["tensors"][name] = {"dtype": "f32", "shape": [int(d) for d in shape], "offset": offset,
                                   "length": len(b)}
        offset += len(b)
        parts.append(b)
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    return struct.pack("<I", len(hb)) + hb + b"".join(parts)


def dumpForward(model, frame: int = 0, include_scene: bool = True) -> dict:
    """Every tensor forwardReference names (reference.ts:360-451) for batch frame `frame` of
    `model`'s last forward, in layer-table order: "input", each op's output, "depth_low"
    (4 channels, as the reference's head broadcasts it), then "scene_color" when the model
    kept it. The model must keep its intermediates (createDepthModel(keepIntermediates=True))."""
    out = {}
    names = ["input"] + [op.out for op in model.arch.ops if op.kind not in ("preprocess", "bilateralUp")]
    for name in names:
        t = model.debugTensor(name, frame=frame)
        if t is None:
            continue
        data, live = t
        if not live:
            raise ValueError(f"dumpForward: {name} was overwritten by a later op; create the model with "
                             "keepIntermediates=True")
        out[name] = data
    if include_scene:
        try:
            out["scene_color"] = model.debugTensor("scene_color", frame=frame)[0]
        except Exception:  # noqa: BLE001 -- not kept by this model
            pass
    return out
