"""Weight container and seeded initialiser: the Python face of
src/model/weights.ts (weightSpecs, parseWeights, serializeWeights,
synthesizeWeights, halfToFloat, opWeights). All work happens in the native
library; a WeightMap is a dict name -> float32 numpy array (flat).
"""
from __future__ import annotations

import ctypes as C
import json
import struct

import numpy as np

from ._lib import ARCH_MISMATCH, IlluminaError, check, lib
from .arch import Architecture, weightSpecs

CANONICAL_NAME = "IlluminaDepth-448"


def _count(arch: Architecture) -> int:
    n = C.c_size_t(0)
    check(lib().illumina_weights_count(arch.inputSize, C.byref(n)))
    return n.value


def _split(arch: Architecture, blob: np.ndarray) -> dict:
    out, off = {}, 0
    for name, shape in weightSpecs(arch):
        n = int(np.prod(shape))
        out[name] = blob[off:off + n].copy()
        off += n
    return out


def flatten(arch: Architecture, weights: dict) -> np.ndarray:
    """A WeightMap as one float32 blob in weightSpecs order (the .idm blob order)."""
    parts = []
    for name, shape in weightSpecs(arch):
        v = weights.get(name)
        if v is None:
            raise ValueError(f"weights: {name} is missing")
        v = np.asarray(v, np.float32).ravel()
        if v.size != int(np.prod(shape)):
            raise ValueError(f"weights: {name} has {v.size} values, expected {int(np.prod(shape))}")
        parts.append(v)
    return np.ascontiguousarray(np.concatenate(parts))


def totalParameters(arch: Architecture) -> int:
    return _count(arch)


def synthesizeWeights(arch: Architecture, seed: int = 1) -> dict:
    """synthesizeWeights (weights.ts:227-251): deterministic Kaiming-normal weights."""
    blob = np.empty(_count(arch), np.float32)
    check(lib().illumina_weights_synthesize(arch.inputSize, seed & 0xFFFFFFFF, blob.ctypes.data, blob.size))
    return _split(arch, blob)


def parseWeights(buffer: bytes, arch: Architecture) -> dict:
    """parseWeights (weights.ts:97-165); raises ValueError with the reference's messages."""
    buffer = bytes(buffer)
    if arch.name != CANONICAL_NAME and len(buffer) >= 4:
        # The library validates against its own table name; a renamed
        # Architecture (network.test.ts:180-192) is checked here first.
        (hl,) = struct.unpack_from("<I", buffer, 0)
        try:
            got = json.loads(buffer[4:4 + hl].decode("utf-8")).get("arch")
        except Exception:  # noqa: BLE001 - the library reports malformed headers
            got = None
        if got is not None and got != arch.name:
            raise ValueError(f"weights: file is for {got}, this build is {arch.name}")
    blob = np.empty(_count(arch), np.float32)
    src = C.create_string_buffer(buffer, len(buffer))
    try:
        check(lib().illumina_weights_parse(arch.inputSize, C.cast(src, C.c_void_p), len(buffer),
                                           blob.ctypes.data, blob.size))
    except IlluminaError as e:
        err = ValueError(str(e))
        err.status = e.status
        err.arch_mismatch = e.status == ARCH_MISMATCH
        raise err from None
    return _split(arch, blob)


def serializeWeights(arch: Architecture, weights: dict) -> bytes:
    """serializeWeights (weights.ts:168-194)."""
    blob = flatten(arch, weights)
    need = C.c_size_t(0)
    check(lib().illumina_weights_serialize(arch.inputSize, blob.ctypes.data, blob.size, None, 0, C.byref(need)))
    out = C.create_string_buffer(need.value)
    check(lib().illumina_weights_serialize(arch.inputSize, blob.ctypes.data, blob.size, C.cast(out, C.c_void_p),
                                           need.value, C.byref(need)))
    return out.raw[:need.value]


def halfToFloat(h: int) -> float:
    """halfToFloat (weights.ts:82-95)."""
    return lib().illumina_half_to_float(h & 0xFFFF)


def opWeights(op, weights: dict) -> dict:
    """opWeights (weights.ts:254-277): the per-op tensors."""
    def need(suffix):
        key = f"{op.name}.{suffix}"
        if key not in weights:
            raise ValueError(f"weights: {key} is missing")
        return weights[key]
    if op.kind in ("conv", "pw", "lateral", "head"):
        return {"weight": need("weight"), "bias": need("bias")}
    if op.kind == "dwpw":
        return {"dwWeight": need("dw_weight"), "dwBias": need("dw_bias"), "pwWeight": need("pw_weight"),
                "pwBias": need("pw_bias")}
    return {}
