"""Host-side logic of the product library, checked on CPU against the oracle.

No GPU is needed: these exercise the C ABI's layer table, weight container,
seeded initialiser and arena planner (the reference's pure helpers).
"""
import ctypes as C
import json
import os
import re

import numpy as np
import pytest

import illumina
from illumina import _lib
from oracle import arch as OA
from oracle import arena as OAR
from oracle import weights as OW

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(REPO, "include", "illumina.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(illumina_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = header_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the ctypes table covers exactly the declared functions
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_library_reports_no_device_here_or_counts_devices():
    n = _lib.lib().illumina_device_count()
    assert n >= 0
    assert b"sm_100a" in _lib.lib().illumina_version()


@pytest.mark.parametrize("size", [64, 448, 96])
def test_arch_matches_oracle_and_golden(golden_dir, size):
    a = illumina.buildArchitecture(size)
    o = OA.build_architecture(size)
    assert a.name == o.name and a.inputSize == size
    assert {n: (s.h, s.w, s.c) for n, s in a.tensors.items()} == {n: (s.h, s.w, s.c) for n, s in o.tensors.items()}
    assert list(a.tensors) == list(o.tensors)  # insertion order, as the JS object
    for x, y in zip(a.ops, o.ops):
        assert (x.kind, x.name, x.out, x.inp, x.k, x.stride, x.act, x.midAct, x.residual, x.coarse, x.skip) == \
            (y.kind, y.name, y.out, y.inp, y.k, y.stride, y.act, y.mid_act, y.residual, y.coarse, y.skip)
    cost = illumina.costOf(a)
    per, macs, params = OA.cost_of(o)
    assert (cost.totalMacs, cost.totalParams, cost.dispatches) == (macs, params, 40)
    assert [(c.name, c.macs, c.params) for c in cost.ops] == [(c["name"], c["macs"], c["params"]) for c in per]
    assert illumina.weightSpecs(a) == [(n, tuple(s)) for n, s in OA.weight_specs(o)]
    if size in (64, 448):
        doc = json.load(open(os.path.join(golden_dir, "arch.json")))[str(size)]
        assert cost.totalMacs == doc["total_macs"] and cost.totalParams == doc["total_params"]


def test_arch_rejects_bad_size():
    with pytest.raises(ValueError, match="multiple of 32"):
        illumina.buildArchitecture(100)


def test_format_cost_mentions_totals():
    text = illumina.formatCost(illumina.buildArchitecture(448))
    assert "dispatches            : 40" in text and "GFLOP / frame         : 2.198" in text


@pytest.mark.parametrize("seed", [0, 1, 20240819])
def test_synthesize_bit_exact_with_oracle(seed):
    a = illumina.buildArchitecture(64)
    got = illumina.synthesizeWeights(a, seed)
    want = OW.synthesize_weights(OA.build_architecture(64), seed)
    assert list(got) == list(want)
    for n in want:
        np.testing.assert_array_equal(got[n], want[n])


def test_serialize_byte_identical_to_oracle_and_reference_writer(golden_dir):
    a = illumina.buildArchitecture(448)
    wts = {}
    for i, (n, shape) in enumerate(illumina.weightSpecs(a)):
        j = np.arange(int(np.prod(shape)), dtype=np.int64)
        wts[n] = (((i * 7919 + j * 31) % 1000) / 1000.0 - 0.5).astype(np.float32)
    raw = illumina.serializeWeights(a, wts)
    import hashlib
    doc = json.load(open(os.path.join(golden_dir, "idm.json")))
    assert hashlib.sha256(raw).hexdigest() == doc["f32"]["sha256"]
    assert raw == OW.serialize_weights(OA.build_architecture(448), wts)


def test_parse_f16_container(golden_dir):
    """A reference-exporter f16 container (rebuilt from its header) decodes like struct 'e'."""
    import struct
    doc = json.load(open(os.path.join(golden_dir, "idm.json")))["f16"]
    a = illumina.buildArchitecture(448)
    header = json.dumps(doc["header"], separators=(",", ":")).encode()
    blob = []
    for i, (n, shape) in enumerate(illumina.weightSpecs(a)):
        j = np.arange(int(np.prod(shape)), dtype=np.int64)
        blob.append((((i * 7919 + j * 31) % 1000) / 1000.0 - 0.5).astype("<f2").tobytes())
    raw = struct.pack("<I", len(header)) + header + b"".join(blob)
    got = illumina.parseWeights(raw, a)
    for n, vals in doc["samples"].items():
        np.testing.assert_array_equal(got[n][:8], np.array(vals, np.float32))


def test_roundtrip_and_errors():
    """network.test.ts:168-192 and the parseWeights error classes (weights.ts:97-165)."""
    a = illumina.buildArchitecture(64)
    w = illumina.synthesizeWeights(a, 99)
    raw = illumina.serializeWeights(a, w)
    back = illumina.parseWeights(raw, a)
    assert list(back) == list(w)
    for n in w:
        np.testing.assert_array_equal(back[n], w[n])
    import dataclasses
    with pytest.raises(ValueError, match="SomethingElse"):
        illumina.parseWeights(raw, dataclasses.replace(a, name="SomethingElse"))
    cases = [
        (raw[:3], "file is truncated"),
        (raw[:40], "does not fit the file"),
        (raw[:-4], "extends past the end of the file"),
        (b"\x05\x00\x00\x00{nope" + raw[9:], "header is not valid JSON"),
    ]
    for buf, msg in cases:
        with pytest.raises(ValueError, match=msg):
            illumina.parseWeights(buf, a)
    # wrong format / arch / length / missing, by editing the header
    import struct
    hl = struct.unpack_from("<I", raw, 0)[0]
    hdr = json.loads(raw[4:4 + hl])
    body = raw[4 + hl:]

    def rebuild(h):
        hb = json.dumps(h, separators=(",", ":")).encode()
        return struct.pack("<I", len(hb)) + hb + body
    h = dict(hdr, format="idm/0")
    with pytest.raises(ValueError, match="unsupported format idm/0, expected idm/1"):
        illumina.parseWeights(rebuild(h), a)
    h = dict(hdr, arch="Other")
    with pytest.raises(ValueError, match="file is for Other, this build is IlluminaDepth-448") as ei:
        illumina.parseWeights(rebuild(h), a)
    assert ei.value.status == _lib.ARCH_MISMATCH
    t = dict(hdr["tensors"])
    t["stem.bias"] = dict(t["stem.bias"], length=8)
    with pytest.raises(ValueError, match="stem.bias claims 8 bytes but its shape needs 64"):
        illumina.parseWeights(rebuild(dict(hdr, tensors=t)), a)
    t = {k: v for k, v in hdr["tensors"].items() if k not in ("head.weight", "head.bias")}
    with pytest.raises(ValueError, match=r"2 tensor\(s\) missing, first few: head.weight, head.bias"):
        illumina.parseWeights(rebuild(dict(hdr, tensors=t)), a)
    t = dict(hdr["tensors"])
    t["stem.bias"] = dict(t["stem.bias"], shape=[8], length=32)
    with pytest.raises(ValueError, match=r"stem.bias has 8 values, expected 16 for shape \[16\]"):
        illumina.parseWeights(rebuild(dict(hdr, tensors=t)), a)


def test_half_to_float_matches_oracle():
    for h in [0, 1, 0x3C00, 0xBC00, 0x7BFF, 0x0400, 0x03FF, 0x7C00, 0xFC00, 0x3555, 0x8001]:
        assert illumina.halfToFloat(h) == OW.half_to_float(h)
    assert np.isnan(illumina.halfToFloat(0x7E00))


@pytest.mark.parametrize("size", [64, 448])
def test_arena_matches_oracle(size):
    a = illumina.buildArchitecture(size)
    plan = illumina.planArena(a)
    sizes, assign, total, naive = OAR.plan_arena(OA.build_architecture(size), {"depth"})
    assert list(plan.bufferSizes) == sizes and plan.assignment == assign
    assert (plan.totalBytes, plan.naiveBytes) == (total, naive)
    illumina.validateArena(a, plan)
    if size == 448:
        assert len(plan.bufferSizes) == 7 and abs(plan.totalBytes / 1e6 - 19.03) < 0.01


def test_validate_arena_catches_overlap():
    a = illumina.buildArchitecture(64)
    plan = illumina.planArena(a)
    import dataclasses
    bad = dataclasses.replace(plan, assignment=dict(plan.assignment, s0=plan.assignment["stem"]))
    with pytest.raises(ValueError, match="overlap"):
        illumina.validateArena(a, bad)


def test_model_create_without_gpu_fails_loudly():
    if _lib.lib().illumina_device_count() > 0:
        pytest.skip("a GPU is present")
    with pytest.raises(illumina.IlluminaError) as ei:
        illumina.createDepthModel(illumina.buildArchitecture(64))
    assert ei.value.status == _lib.NO_DEVICE


def test_model_create_rejects_bad_weights_before_touching_the_device():
    a = illumina.buildArchitecture(64)
    with pytest.raises(illumina.IlluminaError) as ei:
        illumina.createDepthModel(a, idm=b"\x01\x00")
    assert ei.value.status == _lib.BAD_WEIGHTS and "truncated" in str(ei.value)
