"""Pins the CPU oracle to the reference before it is trusted as the checker.

Each test compares the oracle's restatement with fixtures produced by the
reference's own Python twin and exporter (tests/golden/make_golden.py), on the
inputs the reference's own tests draw.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import arch as A
from oracle import arena as AR
from oracle import reference as R
from oracle import weights as W
from tests.golden import cases


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def _check(got, store, key, rtol_of_max):
    """Scale-relative comparison: |got - twin| <= rtol_of_max * max|twin| (+ a tiny abs floor)."""
    got = np.asarray(got, np.float64).ravel()
    s = store[f"{key}/sum"]
    scale = max(float(s[2]), 1e-30)
    if f"{key}/full" in store:
        want = store[f"{key}/full"].astype(np.float64)
        assert want.size == got.size
        err = np.abs(got - want).max()
        # fixtures store full arrays as float32: allow their rounding
        assert err <= rtol_of_max * scale + 1e-7 * scale + 1e-30, (key, err, scale)
    else:
        idx, want = store[f"{key}/idx"], store[f"{key}/val"]
        err = np.abs(got[idx] - want).max()
        assert err <= rtol_of_max * scale + 1e-30, (key, err, scale)
    # whole-tensor checksums
    assert abs(got.sum() - s[0]) <= 1e-5 * (np.abs(got).sum() + 1e-30) + 1e-6, key
    assert abs((got * got).sum() - s[1]) <= 1e-5 * s[1] + 1e-12, key


@pytest.mark.parametrize("size", [64, 448])
def test_arch_table_matches_twin(golden_dir, size):
    doc = json.load(open(os.path.join(golden_dir, "arch.json")))[str(size)]
    a = A.build_architecture(size)
    assert a.name == doc["name"] == "IlluminaDepth-448"
    assert [list(a.mean), list(a.std)] == [doc["mean"], doc["std"]]
    assert {n: [s.h, s.w, s.c] for n, s in a.tensors.items()} == doc["tensors"]
    assert len(a.ops) == len(doc["ops"]) == 40
    for op, want in zip(a.ops, doc["ops"]):
        got = {"kind": op.kind, "name": op.name, "out": op.out}
        for f in ("inp", "k", "stride", "act", "mid_act", "residual", "coarse", "skip"):
            if f in want:
                got[f] = getattr(op, f)
        assert got == want
    per_op, macs, params = A.cost_of(a)
    assert [(c["name"], c["macs"], c["params"]) for c in per_op] == \
        [(c["name"], c["macs"], c["params"]) for c in doc["cost"]]
    assert (macs, params) == (doc["total_macs"], doc["total_params"])
    assert [[n, list(s)] for n, s in A.weight_specs(a)] == doc["specs"]


def test_published_structure_448():
    """README.md:26-31 and network.test.ts:194-201."""
    a = A.build_architecture(448)
    _, macs, params = A.cost_of(a)
    assert abs(2 * macs / 1e9 - 2.198) < 0.0005
    assert params == 1_390_657
    assert len(A.weight_specs(a)) == 112
    assert 2 * macs < 3e9 and params < 2e6 and len(a.ops) == 40
    sizes, assign, total, naive = AR.plan_arena(a, {"depth"})
    assert len(sizes) == 7
    assert abs(total / 1e6 - 19.03) < 0.01 and abs(naive / 1e6 - 63.12) < 0.01


@pytest.mark.parametrize("size", [64, 448, 96])
def test_arena_valid(size):
    a = A.build_architecture(size)
    sizes, assign, total, naive = AR.plan_arena(a, {"depth"})
    AR.validate_arena(a, sizes, assign, {"depth"})
    assert total < naive


def test_arena_validation_catches_overlap():
    a = A.build_architecture(64)
    sizes, assign, _, _ = AR.plan_arena(a, {"depth"})
    bad = dict(assign)
    bad["s0"] = bad["stem"]  # s0 is produced while stem is still being read
    with pytest.raises(ValueError, match="overlap"):
        AR.validate_arena(a, sizes, bad, {"depth"})


def test_bad_input_size():
    with pytest.raises(ValueError, match="multiple of 32"):
        A.build_architecture(100)


def test_idm_serializer_is_byte_identical_to_reference_writer(golden_dir):
    """The reference exporter's container for the interop pattern (interop.test.ts:29-31)."""
    doc = json.load(open(os.path.join(golden_dir, "idm.json")))
    a = A.build_architecture(448)
    wts = {}
    for i, (n, shape) in enumerate(A.weight_specs(a)):
        cnt = int(np.prod(shape))
        j = np.arange(cnt, dtype=np.int64)
        wts[n] = (((i * 7919 + j * 31) % 1000) / 1000.0 - 0.5).astype(np.float32)
    raw = W.serialize_weights(a, wts)
    assert hashlib.sha256(raw).hexdigest() == doc["f32"]["sha256"]
    back = W.parse_weights(raw, a)
    for n, vals in doc["f32"]["samples"].items():
        np.testing.assert_array_equal(back[n][:8], np.array(vals, np.float32))


def test_half_decode_matches_reference_reader(golden_dir):
    doc = json.load(open(os.path.join(golden_dir, "idm.json")))["f16"]
    # rebuild the f16 container bytes from the reference header + pattern, parse with the oracle
    a = A.build_architecture(448)
    import struct
    header = json.dumps(doc["header"], separators=(",", ":")).encode()
    blob = []
    for i, (n, shape) in enumerate(A.weight_specs(a)):
        cnt = int(np.prod(shape))
        j = np.arange(cnt, dtype=np.int64)
        blob.append((((i * 7919 + j * 31) % 1000) / 1000.0 - 0.5).astype("<f2").tobytes())
    raw = struct.pack("<I", len(header)) + header + b"".join(blob)
    assert hashlib.sha256(raw).hexdigest() == doc["sha256"]
    # decode only the sampled tensors (pure-Python halfToFloat is slow)
    hdr = doc["header"]["tensors"]
    base = 4 + len(header)
    for n, vals in doc["samples"].items():
        off = hdr[n]["offset"]
        h = np.frombuffer(raw[base + off: base + off + 16], "<u2")
        got = [W.half_to_float(int(v)) for v in h]
        np.testing.assert_array_equal(np.array(got), np.array(vals))


def test_parse_errors_match_reference_messages():
    a = A.build_architecture(64)
    good = W.serialize_weights(a, W.synthesize_weights(a, 5))
    with pytest.raises(ValueError, match="truncated"):
        W.parse_weights(good[:3], a)
    with pytest.raises(ValueError, match="does not fit"):
        W.parse_weights(good[:40], a)
    import dataclasses
    other = dataclasses.replace(a, name="SomethingElse")
    with pytest.raises(ValueError, match="SomethingElse"):
        W.parse_weights(good, other)
    with pytest.raises(ValueError, match="extends past"):
        W.parse_weights(good[:-4], a)


def test_synthesized_weight_statistics():
    """Kaiming-normal: per-tensor std close to sqrt(2/fan_in); head scaled by 0.05; biases zero."""
    a = A.build_architecture(448)
    wts = W.synthesize_weights(a, 0)
    for n, shape in A.weight_specs(a):
        v = wts[n].astype(np.float64)
        if n.endswith("bias"):
            assert not v.any()
            continue
        fan = shape[1] * shape[2] if "dw_weight" in n else int(np.prod(shape[1:]))
        std = np.sqrt(2.0 / fan) * (0.05 if n.startswith("head") else 1.0)
        if v.size >= 2000:
            assert abs(v.std() / std - 1) < 0.08, n
    # seeds differ, runs repeat
    assert not np.array_equal(wts["stem.weight"], W.synthesize_weights(a, 1)["stem.weight"])
    np.testing.assert_array_equal(wts["e9c.dw_project.pw_weight"],
                                  W.synthesize_weights(a, 0)["e9c.dw_project.pw_weight"])


def test_mulberry32_integer_definition():
    import ctypes as C
    from oracle import lib
    out = np.empty(4, np.float64)
    lib().or_mulberry32(0x1234, 4, out.ctypes.data_as(C.POINTER(C.c_double)))
    ref = cases._mb32_stream(0x1234)
    np.testing.assert_array_equal(out, [ref() for _ in range(4)])


@pytest.mark.parametrize("case", cases.all_cases(), ids=lambda c: c["id"])
def test_ops_match_twin(golden_dir, case):
    store = _load(golden_dir, "ops.npz")
    data = cases.draw(case)
    got = cases.oracle_output(case, data)
    _check(got, store, case["id"], 2e-6)


def test_preprocess_matches_twin(golden_dir):
    g = _load(golden_dir, "preprocess.npz")
    rgba = cases.preprocess_image(32).astype(np.float32) / np.float32(255.0)
    inp, scene = R.preprocess(rgba, 32, A.MEAN, A.STD, True, cases.PREPROCESS_EXPOSURE)
    np.testing.assert_allclose(inp, g["input"], rtol=0, atol=2e-6)
    np.testing.assert_allclose(scene.reshape(-1, 4)[:, :3].ravel(), g["linear"], rtol=0, atol=2e-7)


def test_network64_matches_twin(golden_dir):
    """test/network.test.ts:45-113 at 64x64 with seed-20240819 weights, per tensor."""
    store = _load(golden_dir, "net64.npz")
    a = A.build_architecture(64)
    wts = W.synthesize_weights(a, cases.NET64_SEED)
    rgb = cases.rgba_bytes_to_planar(cases.test_image(64), 64)
    values, disp = R.forward_frame(a, wts, rgb)
    for name in a.tensors:
        if name == "depth":
            continue
        got = values[name]
        if name == "depth_low":  # the twin keeps one channel; the reference broadcasts to four
            got4 = got.reshape(-1, 4)
            assert (got4 == got4[:, :1]).all()
            got = got4[:, 0]
        _check(got, store, name, 2e-6)
    assert np.isfinite(disp).all() and disp.min() >= 0 and disp.max() <= 1
