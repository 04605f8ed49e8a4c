"""Oracle restatement of the weight container and seeded init,
src/model/weights.ts:82-251, plus the ntb/1 bundle I/O of
scripts/ref-forward.ts:67-165.

TEST INFRASTRUCTURE ONLY: checks the product's C++ container code and
synthesises the weights the parity tests feed to both sides.
"""
from __future__ import annotations

import json
import struct

import numpy as np

from . import lib
from .arch import Architecture, weight_specs

IDM_FORMAT = "idm/1"
BUNDLE_FORMAT = "ntb/1"


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


def half_to_float(h: int) -> float:
    """halfToFloat, weights.ts:82-95 (delegates to the C restatement)."""
    return lib().or_half_to_float(h)


def synthesize_weights(arch: Architecture, seed: int = 1) -> dict:
    """synthesizeWeights, weights.ts:227-251 -> {name: float32 array (flat)}."""
    specs = weight_specs(arch)
    counts = np.array([_numel(s) for _, s in specs], dtype=np.int64)
    fan_in = []
    for name, shape in specs:
        if "dw_weight" in name:
            fan_in.append(shape[1] * shape[2])
        else:
            fan_in.append(_numel(shape[1:]))
    fan_in = np.array(fan_in, dtype=np.int64)
    is_bias = np.array([1 if n.endswith("bias") else 0 for n, _ in specs], dtype=np.int32)
    is_head = np.array([1 if n.startswith("head") else 0 for n, _ in specs], dtype=np.int32)
    blob = np.zeros(int(counts.sum()), dtype=np.float32)
    import ctypes as C
    lib().or_synthesize(seed & 0xFFFFFFFF, len(specs),
                        counts.ctypes.data_as(C.POINTER(C.c_long)),
                        fan_in.ctypes.data_as(C.POINTER(C.c_long)),
                        is_bias.ctypes.data_as(C.POINTER(C.c_int)),
                        is_head.ctypes.data_as(C.POINTER(C.c_int)),
                        blob.ctypes.data_as(C.POINTER(C.c_float)))
    out, off = {}, 0
    for (name, shape), n in zip(specs, counts):
        out[name] = blob[off:off + n].copy()
        off += n
    return out


def flatten(arch: Architecture, weights: dict) -> np.ndarray:
    """Concatenates a weight map in weightSpecs order (the .idm blob order)."""
    return np.concatenate([np.asarray(weights[n], dtype=np.float32).ravel()
                           for n, _ in weight_specs(arch)])


def serialize_weights(arch: Architecture, weights: dict) -> bytes:
    """serializeWeights, weights.ts:168-194 (compact JSON, f32 blob)."""
    tensors, offset, parts = {}, 0, []
    for name, shape in weight_specs(arch):
        data = weights.get(name)
        if data is None:
            raise ValueError(f"serializeWeights: missing {name}")
        raw = np.asarray(data, dtype="<f4").tobytes()
        tensors[name] = {"dtype": "f32", "shape": list(shape), "offset": offset, "length": len(raw)}
        offset += len(raw)
        parts.append(raw)
    header = json.dumps({"format": IDM_FORMAT, "arch": arch.name, "tensors": tensors},
                        separators=(",", ":")).encode("utf-8")
    return struct.pack("<I", len(header)) + header + b"".join(parts)


def _read_container(buf: bytes, what: str):
    if len(buf) < 4:
        raise ValueError(f"{what}: file is truncated")
    (hl,) = struct.unpack_from("<I", buf, 0)
    if hl == 0 or 4 + hl > len(buf):
        raise ValueError(f"{what}: header length {hl} does not fit the file")
    try:
        header = json.loads(buf[4:4 + hl].decode("utf-8"))
    except Exception as e:  # noqa: BLE001
        raise ValueError(f"{what}: header is not valid JSON ({e})")
    return header, 4 + hl


def _decode(buf: bytes, base: int, name: str, info: dict, what: str):
    count = _numel(info["shape"])
    nbytes = count * (2 if info["dtype"] == "f16" else 4)
    if info["length"] != nbytes:
        raise ValueError(f"{what}: {name} claims {info['length']} bytes but its shape needs {nbytes}")
    if base + info["offset"] + nbytes > len(buf):
        raise ValueError(f"{what}: {name} extends past the end of the file")
    raw = buf[base + info["offset"]: base + info["offset"] + nbytes]
    if info["dtype"] == "f32":
        return np.frombuffer(raw, dtype="<f4").astype(np.float32)
    h = np.frombuffer(raw, dtype="<u2")
    return np.array([half_to_float(int(v)) for v in h], dtype=np.float32)


def parse_weights(buf: bytes, arch: Architecture) -> dict:
    """parseWeights, weights.ts:97-165, with the same error messages."""
    header, base = _read_container(buf, "weights")
    if header.get("format") != IDM_FORMAT:
        raise ValueError(f"weights: unsupported format {header.get('format')}, expected {IDM_FORMAT}")
    if header.get("arch") != arch.name:
        raise ValueError(f"weights: file is for {header.get('arch')}, this build is {arch.name}")
    out = {}
    for name, info in header["tensors"].items():
        out[name] = _decode(buf, base, name, info, "weights")
    missing = []
    for name, shape in weight_specs(arch):
        got = out.get(name)
        if got is None:
            missing.append(name)
        elif got.size != _numel(shape):
            raise ValueError(f"weights: {name} has {got.size} values, expected {_numel(shape)} "
                             f"for shape [{', '.join(map(str, shape))}]")
    if missing:
        raise ValueError(f"weights: {len(missing)} tensor(s) missing, first few: {', '.join(missing[:5])}")
    return out


def write_bundle(tensors: dict) -> bytes:
    """writeBundle, ref-forward.ts:138-165: {name: (shape, f32 array)} -> ntb/1 bytes."""
    header, offset, parts = {"format": BUNDLE_FORMAT, "tensors": {}}, 0, []
    for name, (shape, data) in tensors.items():
        raw = np.asarray(data, dtype="<f4").ravel().tobytes()
        if len(raw) != 4 * _numel(shape):
            raise ValueError(f"{name}: shape {list(shape)} needs {_numel(shape)} values")
        header["tensors"][name] = {"dtype": "f32", "shape": list(shape), "offset": offset,
                                   "length": len(raw)}
        offset += len(raw)
        parts.append(raw)
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    return struct.pack("<I", len(hb)) + hb + b"".join(parts)


def read_bundle(buf: bytes) -> dict:
    """readBundle, ref-forward.ts:96-136 -> {name: (shape, f32 array)}."""
    header, base = _read_container(buf, "bundle")
    if header.get("format") != BUNDLE_FORMAT:
        raise ValueError(f"bundle: format {header.get('format')}, expected {BUNDLE_FORMAT}")
    return {n: (tuple(i["shape"]), _decode(buf, base, n, i, "bundle"))
            for n, i in header["tensors"].items()}
