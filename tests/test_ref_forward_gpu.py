"""The ref-forward CLI on the CUDA path (python -m illumina.ref_forward): an
"rgba" bundle and an "input" bundle through the GPU forward, every dumped
activation read back with the oracle's bundle reader and compared with the
oracle's forwardReference of the same input (tolerances of the whole-network
tests: every conv output max|got - want| / max|want| <= 1e-4 and rel-L2 <=
5e-5; depth_low and the bilateral output max-abs <= 1.5e-3 on the tensor
engine; the preprocess outputs within 1e-5)."""
import numpy as np
import pytest

from tests.golden import cases
from tests.helpers import compare, scale_metrics

pytestmark = pytest.mark.gpu

FP32_MAXREL, FP32_L2, DISP_TC = 1e-4, 5e-5, 1.5e-3


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _check(dumped, values, skip=()):
    for name, want in values.items():
        if name in skip:
            continue
        shape, got = dumped[name]
        got = np.asarray(got, np.float32)
        if name in ("input", "scene_color"):
            _, _, worst = compare(got, want, 1e-5, 1e-5)
            assert worst == [], (name, worst)
        elif name == "depth_low":
            _, _, worst = compare(got, want, DISP_TC, 0)
            assert worst == [], (name, worst)
        else:
            mr, l2 = scale_metrics(got, want)
            assert mr <= FP32_MAXREL and l2 <= FP32_L2, (name, mr, l2)


@pytest.mark.parametrize("size", [64, 448])
def test_rgba_bundle_every_layer(torch, tmp_path, size):
    from illumina import ref_forward
    from oracle import arch as OA
    from oracle import frames
    from oracle import reference as R
    from oracle import weights as OW
    rgb = cases.rgba_bytes_to_planar(cases.test_image(size), size) if size == 64 else frames.blob_frame(7, size)
    rgba = R.rgb_planar_to_rgba(rgb, size).reshape(size, size, 4)
    inp = tmp_path / "in.ntb"
    inp.write_bytes(OW.write_bundle({"rgba": ((size, size, 4), rgba.ravel())}))
    out = tmp_path / "out.ntb"
    summary = ref_forward.run(["--weights", "synthetic:0", "--input", str(inp), "--out", str(out)])
    assert summary["size"] == size and summary["names"][0] == "input"
    a = OA.build_architecture(size)
    values, disp = R.forward_frame(a, OW.synthesize_weights(a, 0), rgb)
    dumped = OW.read_bundle(out.read_bytes())
    assert set(values) <= set(dumped) and "depth" in dumped
    _check(dumped, values)
    _, _, worst = compare(np.asarray(dumped["depth"][1]), disp, DISP_TC, 0)
    assert worst == []


def test_input_bundle_every_layer(torch, tmp_path):
    """An "input" bundle (the preprocess output) runs from the stem."""
    from illumina import ref_forward
    from oracle import arch as OA
    from oracle import reference as R
    from oracle import weights as OW
    size = 64
    rgb = cases.rgba_bytes_to_planar(cases.test_image(size), size)
    a = OA.build_architecture(size)
    values, disp = R.forward_frame(a, OW.synthesize_weights(a, 0), rgb)
    inp = tmp_path / "in.ntb"
    inp.write_bytes(OW.write_bundle({"input": ((size, size, 4), values["input"])}))
    out = tmp_path / "out.ntb"
    summary = ref_forward.run(["--weights", "synthetic:0", "--input", str(inp), "--out", str(out)])
    dumped = OW.read_bundle(out.read_bytes())
    assert "scene_color" not in dumped and summary["tensors"] == len(dumped)
    _check(dumped, values, skip=("scene_color",))
    # the guide is the input's luminance channel, so the bilateral output matches too
    _, _, worst = compare(np.asarray(dumped["depth"][1]), disp, DISP_TC, 0)
    assert worst == []
