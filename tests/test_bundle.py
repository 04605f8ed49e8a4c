"""ntb/1 activation bundles (scripts/ref-forward.ts:63-165) in the product
(illumina.bundle) against the oracle's restatement, and the ref-forward CLI's
weight dump, on the CPU."""
import json
import struct

import numpy as np
import pytest

import illumina
from illumina import bundle as B
from illumina import ref_forward
from oracle import weights as OW


def _tensors():
    rng = np.random.default_rng(3)
    return {"input": rng.random((4, 4, 4)).astype(np.float32), "e1": rng.standard_normal((2, 2, 24)).astype(np.float32),
            "depth_low": np.full((2, 2, 4), 0.25, np.float32)}


def test_written_bundle_reads_back_in_the_oracle():
    t = _tensors()
    got = OW.read_bundle(B.writeBundle(t))
    assert list(got) == list(t)
    for name, v in t.items():
        shape, data = got[name]
        assert tuple(shape) == v.shape
        np.testing.assert_array_equal(np.asarray(data, np.float32).reshape(v.shape), v)


def test_oracle_bundle_reads_in_the_product():
    t = _tensors()
    raw = OW.write_bundle({k: (v.shape, v.ravel()) for k, v in t.items()})
    got = B.readBundle(raw)
    assert list(got) == list(t)
    for k, v in t.items():
        np.testing.assert_array_equal(got[k], v)


def test_f16_tensors_decode_exactly():
    vals = np.array([0.0, 1.0, -2.5, 65504.0, 6.1035156e-05, 5.9604645e-08], np.float16)
    hdr = json.dumps({"format": "ntb/1", "tensors": {"h": {"dtype": "f16", "shape": [6], "offset": 0,
                                                            "length": 12}}}).encode()
    raw = struct.pack("<I", len(hdr)) + hdr + vals.tobytes()
    got = B.readBundle(raw)["h"]
    assert got.dtype == np.float32
    np.testing.assert_array_equal(got, [illumina.halfToFloat(int(h)) for h in vals.view(np.uint16)])


def test_validation_messages():
    raw = B.writeBundle({"x": np.zeros((2, 3), np.float32)})
    with pytest.raises(ValueError, match="truncated"):
        B.readBundle(raw[:3])
    with pytest.raises(ValueError, match="does not fit the file"):
        B.readBundle(struct.pack("<I", 10 ** 6) + raw[4:])
    with pytest.raises(ValueError, match="extends past the end"):
        B.readBundle(raw[:-4])
    hdr = json.loads(raw[4:4 + struct.unpack("<I", raw[:4])[0]])
    hdr["format"] = "ntb/2"
    hb = json.dumps(hdr).encode()
    with pytest.raises(ValueError, match="expected ntb/1"):
        B.readBundle(struct.pack("<I", len(hb)) + hb + raw[4 + struct.unpack("<I", raw[:4])[0]:])
    hdr["format"] = "ntb/1"
    hdr["tensors"]["x"]["length"] = 20
    hb = json.dumps(hdr).encode()
    with pytest.raises(ValueError, match="claims 20 bytes, shape needs 24"):
        B.readBundle(struct.pack("<I", len(hb)) + hb + raw[4 + struct.unpack("<I", raw[:4])[0]:])
    with pytest.raises(ValueError, match="needs 6 values"):
        B.writeBundle({"x": ((2, 3), np.zeros(5, np.float32))})


def test_cli_dumps_the_weights_it_uses(tmp_path):
    """ref-forward --dump-weights with no --input: the .idm of synthetic:0 at 64."""
    out = tmp_path / "w.idm"
    summary = ref_forward.run(["--weights", "synthetic:0", "--size", "64", "--dump-weights", str(out)])
    assert summary["tensors"] == 0 and summary["size"] == 64
    arch = illumina.buildArchitecture(64)
    assert out.read_bytes() == illumina.serializeWeights(arch, illumina.synthesizeWeights(arch, 0))
    # the dumped container loads back as --weights
    w = ref_forward.load_weights(str(out), arch)
    np.testing.assert_array_equal(w["stem.weight"], illumina.synthesizeWeights(arch, 0)["stem.weight"])
    with pytest.raises(ValueError, match="bad synthetic seed"):
        ref_forward.load_weights("synthetic:x", arch)
    with pytest.raises(ValueError, match="--size is required"):
        ref_forward.run(["--weights", "synthetic:0"])
