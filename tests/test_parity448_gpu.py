"""Parity at 448 on the configurations the benchmark times, through the C ABI.

* Batched fp32 (batch 256 of seeded blob frames, the throughput workload):
  frames 0, 127 and 255 of one batched forward against the oracle forward of
  the same frames -- every layer of a keep-intermediates model (read per frame
  with debugTensor) and the final disparity / depth_low of the default
  (aliased-arena) model. Tolerances as in the whole-network tests: every conv
  output max|got - want| / max|want| <= 1e-4 and rel-L2 <= 5e-5; disparity and
  depth_low max-abs <= 1.5e-3 on the tensor engine (3xTF32), 2e-4 on SIMT.
* BF16 (batch 64 of uniform frames at 448): frames 0 and 63 against the fp32
  oracle. Every conv output of frame 0 within rel-L2 3e-2 (measured <= 0.023,
  worst in the decoder). The depth head is a sigmoid of logits that reach
  O(100) in this untrained seeded network, so where a logit is near zero the
  ~2 % relative error of the bf16 activations moves the sigmoid a long way:
  measured on frames 0, 1, 63 the disparity has mean-abs <= 1.9e-3, 99th
  percentile <= 0.048, 0.38-0.52 % of pixels beyond 0.1 and single pixels up
  to 0.87. Stated BF16 tolerance at 448 for disparity and depth_low: mean-abs
  <= 3e-3, 99th percentile <= 6e-2, at most 1 % of pixels beyond 0.1, and
  rel-L2 <= 0.13 (the 64 x 64 test keeps the tighter max-abs 3e-2).
* The blob-frame generator bit for bit against the host generator.
* The bilinear disparity upsample to 1920x1080 (the relighting frame) bit for
  bit against the oracle.
* The joint-bilateral upsample against its closed forms (constant map,
  constant guide, step guide): within 5e-6 absolute on values in [0, 1] (the
  kernel forms its weights with the hardware exp2, relative error ~2^-22).
"""
import ctypes as C

import numpy as np
import pytest

from tests.bilateral_closed_form import separable_upsample
from tests.helpers import compare, scale_metrics

pytestmark = pytest.mark.gpu

S = 448
FP32_MAXREL, FP32_L2, FP32_DISP, FP32_DISP_TC = 1e-4, 5e-5, 2e-4, 1.5e-3
BF16_L2, BF16_DISP_MEAN, BF16_DISP_P99, BF16_FRAC_01, BF16_DISP_L2 = 3e-2, 3e-3, 6e-2, 1e-2, 0.13
BIL_ABS = 5e-6


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def net448():
    from oracle import arch as OA
    from oracle import weights as OW
    a = OA.build_architecture(S)
    return a, OW.synthesize_weights(a, 0)


def _generate(torch, kind, seed0, n, size=S):
    from illumina import _lib
    out = torch.empty((n, 3, size, size), device="cuda")
    _lib.check(_lib.lib().illumina_generate_frames(kind, seed0, n, size, out.data_ptr(), None))
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("size,seed0,n", [(S, 0, 2), (S, 255, 1), (37, 9, 3), (64, 1000, 2)])
def test_blob_generator_bit_exact(torch, size, seed0, n):
    from oracle import frames
    got = _generate(torch, 1, seed0, n, size).cpu().numpy()
    for i in range(n):
        np.testing.assert_array_equal(got[i], frames.blob_frame(seed0 + i, size))


@pytest.fixture(scope="module")
def b256(torch):
    """One batched forward of the bench's 256 blob frames (seeds 0..255)."""
    frames = _generate(torch, 1, 0, 256)
    return frames


CHECK_FRAMES = (0, 127, 255)


@pytest.fixture(scope="module")
def oracle_b256(net448):
    from oracle import frames
    from oracle import reference as R
    a, w = net448
    return {f: R.forward_frame(a, w, frames.blob_frame(f, S)) for f in CHECK_FRAMES}


def test_b256_blob_forward_final_outputs(torch, b256, oracle_b256):
    """Default model (7-buffer aliased arena, the bench's model): disparity and
    depth_low of frames 0, 127, 255 of a batch-256 forward."""
    import illumina
    m = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=0, maxBatch=256)
    tol = FP32_DISP_TC if m.stats.engine == "tensor" else FP32_DISP
    low = torch.empty((256, S // 2, S // 2), device="cuda")
    disp = m.forward(b256, depthLow=low)
    torch.cuda.synchronize()
    for f in CHECK_FRAMES:
        values, want = oracle_b256[f]
        _, _, worst = compare(disp[f].cpu().numpy().ravel(), want, tol, 0)
        assert worst == [], (f, worst)
        _, _, worst = compare(low[f].cpu().numpy().ravel(), values["depth_low"].reshape(-1, 4)[:, 0], tol, 0)
        assert worst == [], (f, worst)
    assert m.stats.deviceError == 0
    m.destroy()


def test_b256_blob_forward_every_layer(torch, b256, oracle_b256):
    """Keep-intermediates model at batch 256: every layer of frames 0, 127, 255."""
    import illumina
    m = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=0, maxBatch=256, keepIntermediates=True)
    m.forward(b256)
    torch.cuda.synchronize()
    for f in CHECK_FRAMES:
        values, _ = oracle_b256[f]
        for name, want in values.items():
            if name in ("scene_color", "depth_low"):
                continue
            data, live = m.debugTensor(name, frame=f)
            assert live, name
            mr, l2 = scale_metrics(data.ravel(), want)
            assert mr <= FP32_MAXREL and l2 <= FP32_L2, (f, name, mr, l2)
    m.destroy()


def test_debug_tensor_frame_range(torch):
    import illumina
    m = illumina.createDepthModel(illumina.buildArchitecture(64), synthSeed=0, maxBatch=2)
    with pytest.raises(illumina.IlluminaError, match="frame 2 outside"):
        m.debugTensor("s0", frame=2)
    m.destroy()


def _bf16_map_ok(got, want):
    e = np.abs(np.asarray(got, np.float64).ravel() - np.asarray(want, np.float64).ravel())
    stats = (e.mean(), np.percentile(e, 99), (e > 0.1).mean(), np.linalg.norm(e) / np.linalg.norm(want))
    ok = stats[0] <= BF16_DISP_MEAN and stats[1] <= BF16_DISP_P99 and stats[2] <= BF16_FRAC_01 and \
        stats[3] <= BF16_DISP_L2
    return ok, stats


def test_bf16_448_batch64(torch, net448):
    """The reduced-precision workload: BF16 weights and activations, fp32
    accumulation, batch 64 of uniform frames, against the fp32 oracle."""
    import illumina
    from oracle import frames
    from oracle import reference as R
    a, w = net448
    x = _generate(torch, 0, 0, 64)
    m = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=0, maxBatch=64, precision="bf16",
                                  keepIntermediates=True)
    disp = m.forward(x).cpu().numpy()
    for f in (0, 63):
        values, want = R.forward_frame(a, w, frames.uniform_frame(f, S))
        ok, stats = _bf16_map_ok(disp[f], want)
        assert ok, (f, "disparity", stats)
        low, _ = m.debugTensor("depth_low", frame=f)
        ok, stats = _bf16_map_ok(low[..., 0], values["depth_low"].reshape(-1, 4)[:, 0])
        assert ok, (f, "depth_low", stats)
        if f == 0:
            for name, v in values.items():
                if name in ("scene_color", "depth_low"):
                    continue
                data, _ = m.debugTensor(name, frame=f)
                _, l2 = scale_metrics(data.ravel(), v)
                assert l2 <= BF16_L2, (name, l2)
    m.destroy()


def test_resize_bilinear_1080p_bit_exact(torch):
    """The relighting frame's disparity upsample, 448 -> 1920x1080."""
    from illumina import _lib
    from oracle import frames
    from oracle import shade as OS
    src = frames.uniform_frame(3, S)[0]
    d_src = torch.from_numpy(src).cuda()
    dst = torch.empty((1080, 1920), device="cuda")
    _lib.check(_lib.lib().illumina_resize_bilinear(d_src.data_ptr(), S, S, dst.data_ptr(), 1920, 1080, None))
    want = OS.resize_bilinear(src, S, S, 1920, 1080)
    np.testing.assert_array_equal(dst.cpu().numpy().ravel(), want)
    # downsampling and odd sizes take the same formula
    dst2 = torch.empty((31, 45), device="cuda")
    _lib.check(_lib.lib().illumina_resize_bilinear(d_src.data_ptr(), S, S, dst2.data_ptr(), 45, 31, None))
    np.testing.assert_array_equal(dst2.cpu().numpy().ravel(), OS.resize_bilinear(src, S, S, 45, 31))


def _bilateral(torch, low, guide, sigma=0.12):
    from illumina import ops
    lh, lw = low.shape
    low4 = np.repeat(low[..., None], 4, axis=2).astype(np.float32)
    out = ops.bilateral(torch.from_numpy(low4).cuda(), lh, lw, 4, torch.from_numpy(guide).cuda(), 4, sigma)
    return out.cpu().numpy().reshape(2 * lh, 2 * lw)


def _grey_guide(cols, rows):
    g = np.ones((rows, cols.size, 4), np.float32)
    g[..., :3] = cols[None, :, None]
    return g


@pytest.mark.parametrize("lh", [7, 32, 224])
def test_bilateral_closed_forms(torch, lh):
    rng = np.random.default_rng(lh)
    # a constant map is reproduced whatever the guide
    got = _bilateral(torch, np.full((lh, lh), 0.37, np.float32), rng.random((2 * lh, 2 * lh, 4)).astype(np.float32))
    assert np.abs(got - 0.37).max() <= BIL_ABS
    # constant guide: the separable spatial filter
    low = rng.random((lh, lh)).astype(np.float32)
    got = _bilateral(torch, low, _grey_guide(np.full(2 * lh, 0.5, np.float32), 2 * lh))
    assert np.abs(got - separable_upsample(low.astype(np.float64))).max() <= BIL_ABS
    # vertical step in the guide: the range weight splits per column
    cols = np.where(np.arange(2 * lh) < lh, 0.2, 0.45).astype(np.float32)
    luma = 0.2126 * cols.astype(np.float64) + 0.7152 * cols + 0.0722 * cols
    got = _bilateral(torch, low, _grey_guide(cols, 2 * lh))
    assert np.abs(got - separable_upsample(low.astype(np.float64), luma, 0.12)).max() <= BIL_ABS
