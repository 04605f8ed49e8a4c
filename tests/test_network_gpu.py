"""Whole-network parity on the GPU through the C ABI (createDepthModel ->
forward), against the CPU oracle on the same seeded weights and inputs.

Tolerances (stated here, checked per layer, scale-relative because the
untrained seeded network grows activations to ~1e4 by the bottleneck):
  fp32 (both engines; the tensor engine is 3xTF32): every conv output
        max|got-want|/max|want| <= 1e-4 and rel-L2 <= 5e-5;
        final disparity and depth_low max-abs <= 2e-4 on the SIMT engine and
        <= 1.5e-3 on the tensor engine (the reference's own depth_low bound): the
        head's logits reach O(100) at 448 and 3xTF32 products accumulated in the
        tensor core drift ~1e-6 relative per layer, so the logit error reaches a
        few 1e-3 near the sigmoid's steep middle.
  bf16 (activations and weights stored in bf16, fp32 accumulation): every
        tensor rel-L2 <= 3e-2; final disparity max-abs <= 3e-2 and
        mean-abs <= 3e-3.
The reference's own end-to-end test (network.test.ts:95, :106) allows
abs 1.5e-3 / rel 5e-3 on depth_low and abs 2e-3 / rel 1e-2 on the depth map.
"""
import numpy as np
import pytest

from tests.golden import cases
from tests.helpers import compare, scale_metrics

pytestmark = pytest.mark.gpu

FP32_MAXREL, FP32_L2, FP32_DISP, FP32_DISP_TC = 1e-4, 5e-5, 2e-4, 1.5e-3
BF16_L2, BF16_DISP_MAX, BF16_DISP_MEAN = 3e-2, 3e-2, 3e-3


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def net64():
    """network.test.ts:45-113: 64x64, seed 20240819, testImage."""
    from oracle import arch as OA
    from oracle import reference as R
    from oracle import weights as OW
    a = OA.build_architecture(64)
    w = OW.synthesize_weights(a, cases.NET64_SEED)
    rgb = cases.rgba_bytes_to_planar(cases.test_image(64), 64)
    values, disp = R.forward_frame(a, w, rgb)
    return rgb, values, disp


def _model(size, seed, **kw):
    import illumina
    return illumina.createDepthModel(illumina.buildArchitecture(size), synthSeed=seed, **kw)


@pytest.mark.parametrize("engine", ["tensor", "simt"])
def test_network64_every_layer_fp32(torch, net64, engine):
    rgb, values, disp = net64
    m = _model(64, cases.NET64_SEED, keepIntermediates=True, engine=engine)
    assert m.stats.engine == engine
    low = np.empty((1, 32, 32), np.float32)
    got = m.forward(rgb[None], depthLow=low)
    for name, want in values.items():
        if name in ("scene_color",):
            continue
        t = m.debugTensor(name)
        assert t is not None, name
        data, live = t
        assert live, name
        if name == "depth_low":
            _, _, worst = compare(data[..., 0].ravel(), want.reshape(-1, 4)[:, 0], FP32_DISP, 0)
            assert worst == [], worst
            continue
        mr, l2 = scale_metrics(data.ravel(), want)
        assert mr <= FP32_MAXREL and l2 <= FP32_L2, (name, mr, l2)
    _, _, worst = compare(got.ravel(), disp, FP32_DISP, 0)
    assert worst == [], worst
    want_low = values["depth_low"].reshape(-1, 4)[:, 0]
    _, _, worst = compare(low.ravel(), want_low, FP32_DISP, 0)
    assert worst == [], worst
    # the reference's own tolerances hold with a wide margin
    _, _, worst = compare(got.ravel(), disp, 2e-3, 1e-2)
    assert worst == []
    m.destroy()


def test_network64_aliased_arena_live_at_end(torch, net64):
    """debugTensor liveAtEnd semantics (runner.ts:466-476) on the 7-buffer arena."""
    rgb, values, disp = net64
    m = _model(64, cases.NET64_SEED)
    got = m.forward(rgb[None])
    _, _, worst = compare(got.ravel(), disp, FP32_DISP, 0)
    assert worst == []
    data, live = m.debugTensor("depth_low")
    assert live
    np.testing.assert_allclose(data[..., 0].ravel(), values["depth_low"].reshape(-1, 4)[:, 0], atol=FP32_DISP)
    _, live_in = m.debugTensor("input")
    assert not live_in  # the arena recycles `input` right after the stem (network.test.ts:81-84)
    s = m.stats
    # 40 ops (the reference's dispatch count); the stem runs inside the
    # preprocess launch and the head inside d0.refine's, so 38 kernel launches
    assert s.dispatches == 40 and s.launches == 38 and s.deviceError == 0
    assert abs(s.arenaBytes - 19.03e6 / 49) < 1e5 or s.arenaBytes < s.naiveArenaBytes
    m.destroy()


def test_network448_single_frame_fp32(torch):
    """The single-frame workload: 448, seed-0 weights, uniform frame from seed 0."""
    from oracle import arch as OA
    from oracle import reference as R
    from oracle import weights as OW
    import ctypes as C
    from oracle import lib as olib
    a = OA.build_architecture(448)
    w = OW.synthesize_weights(a, 0)
    frame = np.empty(3 * 448 * 448, np.float32)
    olib().or_uniform_frame(0, frame.size, frame.ctypes.data_as(C.POINTER(C.c_float)))
    values, disp = R.forward_frame(a, w, frame)
    m = _model(448, 0, keepIntermediates=True)
    got = m.forward(frame.reshape(1, 3, 448, 448))
    tol = FP32_DISP_TC if m.stats.engine == "tensor" else FP32_DISP
    worst_layer = (None, 0, 0)
    for name, want in values.items():
        if name == "scene_color":
            continue
        data, _ = m.debugTensor(name)
        if name == "depth_low":
            _, _, worst = compare(data[..., 0].ravel(), want.reshape(-1, 4)[:, 0], tol, 0)
            assert worst == [], worst
            continue
        mr, l2 = scale_metrics(data.ravel(), want)
        if mr > worst_layer[1]:
            worst_layer = (name, mr, l2)
        assert mr <= FP32_MAXREL and l2 <= FP32_L2, (name, mr, l2)
    _, _, worst = compare(got.ravel(), disp, tol, 0)
    assert worst == [], worst
    m.destroy()


def test_device_frames_generator_matches_oracle_prng(torch):
    """Device-generated uniform frames equal the host mulberry32 stream bit for bit."""
    import ctypes as C
    from illumina import _lib
    from oracle import lib as olib
    out = torch.empty((2, 3, 64, 64), device="cuda")
    _lib.check(_lib.lib().illumina_generate_frames(0, 5, 2, 64, out.data_ptr(), None))
    torch.cuda.synchronize()
    for i in range(2):
        ref = np.empty(3 * 64 * 64, np.float32)
        olib().or_uniform_frame(5 + i, ref.size, ref.ctypes.data_as(C.POINTER(C.c_float)))
        np.testing.assert_array_equal(out[i].cpu().numpy().ravel(), ref)


def test_batched_forward_equals_per_frame(torch):
    """Frames are independent: a batch of 5 gives each frame's single-frame result."""
    from illumina import _lib
    m = _model(64, 7, maxBatch=5)
    frames = torch.empty((5, 3, 64, 64), device="cuda")
    _lib.check(_lib.lib().illumina_generate_frames(1, 100, 5, 64, frames.data_ptr(), None))
    batch = m.forward(frames).cpu().numpy()
    for i in range(5):
        one = m.forward(frames[i:i + 1].contiguous()).cpu().numpy()
        np.testing.assert_array_equal(batch[i], one[0])
    assert np.isfinite(batch).all() and batch.min() >= 0 and batch.max() <= 1
    m.destroy()


def test_graph_replay_retargets_caller_buffers(torch):
    """A captured forward replays with new frame / output / depth_low buffers (no stale pointers)."""
    from illumina import _lib
    m = _model(64, 3, maxBatch=2)
    a = torch.empty((2, 3, 64, 64), device="cuda")
    b = torch.empty((2, 3, 64, 64), device="cuda")
    _lib.check(_lib.lib().illumina_generate_frames(0, 10, 2, 64, a.data_ptr(), None))
    _lib.check(_lib.lib().illumina_generate_frames(1, 20, 2, 64, b.data_ptr(), None))
    x, y = torch.full((2, 64, 64), -1.0, device="cuda"), torch.full((2, 64, 64), -1.0, device="cuda")
    lx, ly = torch.full((2, 32, 32), -1.0, device="cuda"), torch.full((2, 32, 32), -1.0, device="cuda")
    want_a = m.forward(a.clone()).cpu().numpy()
    want_b = m.forward(b.clone()).cpu().numpy()
    for src, dst, low, want in [(a, x, lx, want_a), (b, y, ly, want_b), (a, y, lx, want_a), (b, x, ly, want_b)]:
        m.forward(src, disparity=dst, depthLow=low)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(dst.cpu().numpy(), want)
        assert (low.cpu().numpy() >= 0).all()
    m.destroy()


def test_host_and_device_buffers_agree(torch, net64):
    rgb, _, disp = net64
    m = _model(64, cases.NET64_SEED, maxBatch=2)
    host = m.forward(np.stack([rgb, rgb]))
    devo = m.forward(torch.from_numpy(np.stack([rgb, rgb])).cuda()).cpu().numpy()
    np.testing.assert_array_equal(host, devo)
    # interleaved RGBA frames give the same result
    rgba = np.ones((1, 64, 64, 4), np.float32)
    rgba[0, ..., :3] = np.transpose(rgb, (1, 2, 0))
    inter = m.forward(rgba)
    np.testing.assert_array_equal(inter[0], host[0])
    m.destroy()


def test_idm_weights_match_synthetic(torch, net64):
    import illumina
    rgb, _, disp = net64
    a = illumina.buildArchitecture(64)
    idm = illumina.serializeWeights(a, illumina.synthesizeWeights(a, cases.NET64_SEED))
    m = illumina.createDepthModel(a, idm=idm)
    got = m.forward(rgb[None])
    _, _, worst = compare(got.ravel(), disp, FP32_DISP, 0)
    assert worst == []
    m.destroy()


def test_bf16_variant_within_stated_tolerance(torch, net64):
    rgb, values, disp = net64
    m = _model(64, cases.NET64_SEED, keepIntermediates=True, precision="bf16")
    got = m.forward(rgb[None])
    for name, want in values.items():
        if name == "scene_color":
            continue
        data, _ = m.debugTensor(name)
        _, l2 = scale_metrics(data.ravel(), want)
        assert l2 <= BF16_L2, (name, l2)
    err = np.abs(got.ravel() - disp)
    assert err.max() <= BF16_DISP_MAX and err.mean() <= BF16_DISP_MEAN, (err.max(), err.mean())
    m.destroy()


def test_temporal_history_semantics(torch, net64):
    """record / swapHistory / parity (runner.ts:440-455, io.ts:259-274, frame.test.ts:305-352)."""
    rgb, _, disp = net64
    m = _model(64, cases.NET64_SEED)
    m.setTemporal(0.35, 3.0, 0.12)
    assert m.outputParity() == 1
    m.record(rgb)
    assert m.freshParity() == 1
    slot = m.debugDepth(1).cpu().numpy()
    # first frame: no history -> alpha 1 -> stabilised == raw == first-frame disparity
    np.testing.assert_allclose(slot[..., 0].ravel(), disp, atol=FP32_DISP)
    np.testing.assert_array_equal(slot[..., 0], slot[..., 1])
    assert (slot[..., 3] == 1).all()
    m.swapHistory()
    assert m.outputParity() == 0 and m.freshParity() == 1
    # second identical frame: change 0 -> alpha = base, stabilised stays put
    m.record(rgb)
    assert m.freshParity() == 0
    slot2 = m.debugDepth(0).cpu().numpy()
    np.testing.assert_allclose(slot2[..., 0], slot[..., 0], atol=1e-6)
    assert np.abs(slot2[..., 2]).max() <= 1e-6
    # a different frame: blend between history and the new raw value
    m.swapHistory()
    m.record(np.clip(rgb * 0.5, 0, 1))
    slot3 = m.debugDepth(1).cpu().numpy()
    raw, prev, change = slot3[..., 1], slot2[..., 0], slot3[..., 2]
    np.testing.assert_allclose(change, np.abs(raw - prev), atol=1e-6)
    alpha = np.clip(0.35 + change * 3.0, 0.35, 1.0)
    np.testing.assert_allclose(slot3[..., 0], prev + (raw - prev) * alpha, atol=1e-5)
    m.destroy()


def test_forward_rejects_bad_arguments(torch):
    import illumina
    m = _model(64, 1)
    with pytest.raises(illumina.IlluminaError, match="batch 2 outside"):
        m.forward(np.zeros((2, 3, 64, 64), np.float32))
    with pytest.raises(ValueError):
        m.forward(np.zeros((1, 3, 32, 32), np.float32))
    m.destroy()
