"""8-bit source-texture path in front of the network: makePreprocess's texture
read with createDepthModel's uvScale/uvOffset (src/model/kernels/io.ts:64-118,
src/model/runner.ts:88-89, :177-182) and the blit's cropTransform/mirror
(src/scene/blit.ts:57-60, :80-86).

The sampler restatement (oracle/source.c) and the kernel evaluate the same
float32 expressions without contraction, so the sampled frames must be
bit-identical; the network after them keeps the whole-network tolerance of
the 64x64 smoke case (disparity max-abs <= 1e-5 of the oracle).
"""
import ctypes as C

import numpy as np
import pytest

from tests.golden import cases

F = C.POINTER(C.c_float)


def _oracle_sample(rgba8, sw, sh, scale, offset, mirror, size):
    from oracle import lib
    n = rgba8.shape[0]
    out = np.empty((n, 3, size, size), np.float32)
    sc = np.array(scale, np.float32)
    of = np.array(offset, np.float32)
    rgba8 = np.ascontiguousarray(rgba8, np.uint8)
    lib().or_sample_source(rgba8.ctypes.data_as(C.POINTER(C.c_uint8)), n, sw, sh, sc.ctypes.data_as(F),
                           of.ctypes.data_as(F), int(mirror), size, out.ctypes.data_as(F))
    return out


@pytest.mark.parametrize("w,h", [(1920, 1080), (480, 640), (448, 448), (0, 5), (7, 3)])
def test_crop_transform_matches_oracle(w, h):
    import illumina
    from oracle import lib
    o = (C.c_float * 4)()
    lib().or_crop_transform(w, h, o)
    assert illumina.cropTransform(w, h) == list(o)


def test_crop_transform_closed_form():
    import illumina
    assert illumina.cropTransform(1920, 1080) == [0.5625, 1.0, 0.21875, 0.0]
    assert illumina.cropTransform(480, 640) == [1.0, 0.75, 0.0, 0.125]


def test_oracle_identity_sampling_returns_the_texels():
    """Same-size source, identity transform: every sample lands on a texel centre."""
    S = 64
    px = cases.test_image(S).reshape(1, S, S, 4)
    got = _oracle_sample(px, S, S, (1, 1), (0, 0), False, S)
    np.testing.assert_allclose(got[0], cases.rgba_bytes_to_planar(px.ravel(), S), atol=2e-6, rtol=0)


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.mark.gpu
@pytest.mark.parametrize("sw,sh,scale,offset,mirror,size", [
    (640, 480, None, None, True, 64),               # camera frame, centre crop, mirrored
    (100, 37, (1.3, 0.7), (-0.2, 0.4), False, 96),  # uv leaving [0,1]: clamp-to-edge
    (64, 64, (1, 1), (0, 0), False, 64),            # identity
    (3, 2, (1, 1), (0, 0), False, 32),              # magnification of a tiny source
])
def test_sample_source_bit_exact(torch, sw, sh, scale, offset, mirror, size):
    import illumina
    if scale is None:
        t = illumina.cropTransform(sw, sh)
        scale, offset = t[:2], t[2:]
    rng = np.random.default_rng(sw * 7 + sh)
    px = rng.integers(0, 256, (2, sh, sw, 4), dtype=np.uint8)
    model = illumina.createDepthModel(illumina.buildArchitecture(size), synthSeed=1, maxBatch=2, device=0)
    got = model.sampleSource(torch.from_numpy(px).cuda(), scale, offset, mirror)
    torch.cuda.synchronize()
    model.destroy()
    want = _oracle_sample(px, sw, sh, scale, offset, mirror, size)
    np.testing.assert_array_equal(got.cpu().numpy(), want)


@pytest.mark.gpu
def test_forward_source_matches_oracle(torch):
    """forwardSource on the network test image (64x64 RGBA bytes) with the model's
    uv options, against the oracle forward of the oracle-sampled frame."""
    import illumina
    from oracle import arch as OA
    from oracle import reference as R
    from oracle import weights as OW
    S = 64
    px = cases.test_image(S).reshape(1, S, S, 4)
    scale, offset = (0.8, 0.9), (0.1, 0.05)
    model = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=cases.NET64_SEED, device=0,
                                      uvScale=scale, uvOffset=offset)
    disp = model.forwardSource(torch.from_numpy(px).cuda())
    torch.cuda.synchronize()
    got = disp.cpu().numpy().ravel()
    model.destroy()
    frame = _oracle_sample(px, S, S, scale, offset, False, S)[0]
    oa = OA.build_architecture(S)
    _, want = R.forward_frame(oa, OW.synthesize_weights(oa, cases.NET64_SEED), frame)
    assert float(np.abs(got - want).max()) <= 1e-5


@pytest.mark.gpu
def test_sample_source_rejects_bad_arguments(torch):
    import illumina
    from illumina import _lib
    bad = torch.zeros((1, 4, 4, 4), dtype=torch.uint8, device="cuda")
    frames = torch.empty((1, 3, 32, 32), dtype=torch.float32, device="cuda")
    lib = _lib.lib()
    assert lib.illumina_sample_source(bad.data_ptr(), 1, 0, 4, None, None, 0, 32, frames.data_ptr(), None) != 0
    assert "bad size" in lib.illumina_last_error().decode()
    assert lib.illumina_sample_source(bad.data_ptr() + 1, 1, 4, 4, None, None, 0, 32, frames.data_ptr(), None) != 0
    assert "aligned" in lib.illumina_last_error().decode()
    assert lib.illumina_sample_source(None, 1, 4, 4, None, None, 0, 32, frames.data_ptr(), None) != 0
    del illumina


def _device_path(torch, model, rgba8, scale, offset, mirror):
    """sampleSource + forward on device buffers: the unchunked reference for the host path."""
    frames = model.sampleSource(torch.from_numpy(rgba8).cuda(), scale, offset, mirror)
    disp = model.forward(frames)
    torch.cuda.synchronize()
    return disp.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("sw,sh,mirror", [(64, 64, False), (96, 80, True)])
def test_forward_source_host_chunks_bitwise(torch, sw, sh, mirror):
    """illumina_forward_source with host RGBA8 frames and a host disparity buffer: 40
    frames run as overlapped chunks (uploads, sampling, graphs, downloads); the
    96x80 source does not fit the staging room behind the planar frames and goes
    through the model's own source buffer. Equal to sampling and
    forwarding the whole batch on device buffers within the whole-network tolerance
    (1e-5), and bit-identical across calls."""
    import illumina
    S, n = 64, 40
    rng = np.random.default_rng(sw + sh)
    px = rng.integers(0, 256, (n, sh, sw, 4), dtype=np.uint8)
    scale, offset = (0.9, 0.8), (0.05, 0.1)
    model = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=cases.NET64_SEED, maxBatch=n)
    got = model.forwardSource(px, scale, offset, mirror)
    got2 = model.forwardSource(px, scale, offset, mirror)  # second call: staging and graphs reused
    want = _device_path(torch, model, px, scale, offset, mirror)
    assert model.stats.deviceError == 0
    model.destroy()
    assert got.shape == (n, S, S)
    np.testing.assert_array_equal(got2, got)
    # a chunk's forward equals a forward of those frames alone; the whole-batch
    # forward may split K differently (its own summation order)
    assert float(np.abs(got - want).max()) <= 1e-5


@pytest.mark.gpu
def test_forward_source_device_buffers(torch):
    """Device RGBA8 in, device disparity out: one asynchronous call, equal to the host path."""
    import illumina
    S, n = 64, 3
    px = np.random.default_rng(7).integers(0, 256, (n, S, S, 4), dtype=np.uint8)
    model = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=cases.NET64_SEED, maxBatch=n)
    dev = model.forwardSource(torch.from_numpy(px).cuda())
    torch.cuda.synchronize()
    host = model.forwardSource(px)
    model.destroy()
    np.testing.assert_array_equal(dev.cpu().numpy(), host)


@pytest.mark.gpu
def test_forward_source_rejects_bad_arguments(torch):
    import illumina
    from illumina import _lib
    model = illumina.createDepthModel(illumina.buildArchitecture(64), synthSeed=0, maxBatch=2)
    lib = _lib.lib()
    px = np.zeros((3, 8, 8, 4), np.uint8)
    h = model._h
    assert lib.illumina_forward_source(h, px.ctypes.data, 3, 8, 8, None, None, 0, None, None) != 0
    assert "outside [1, 2]" in lib.illumina_last_error().decode()
    assert lib.illumina_forward_source(h, px.ctypes.data, 1, 0, 8, None, None, 0, None, None) != 0
    assert "source size" in lib.illumina_last_error().decode()
    assert lib.illumina_forward_source(h, px.ctypes.data + 1, 1, 8, 8, None, None, 0, None, None) != 0
    assert "aligned" in lib.illumina_last_error().decode()
    assert lib.illumina_forward_source(h, None, 1, 8, 8, None, None, 0, None, None) != 0
    model.destroy()


@pytest.mark.gpu
def test_forward_source_fast_upload_schedule(torch):
    """200 host RGBA8 frames at the network resolution run as the chunks of the
    fast-upload schedule, 8, 48, 88, 48, 8 frames: bit-identical to sampling and
    forwarding those chunks one by one on device buffers (a chunk's forward is the
    forward of its frames alone), and across calls."""
    import illumina
    S, n = 64, 200
    px = np.random.default_rng(200).integers(0, 256, (n, S, S, 4), dtype=np.uint8)
    model = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=cases.NET64_SEED, maxBatch=n)
    got = model.forwardSource(px)
    got2 = model.forwardSource(px)
    want, f0 = [], 0
    for c in (8, 48, 88, 48, 8):
        want.append(_device_path(torch, model, px[f0:f0 + c], (1.0, 1.0), (0.0, 0.0), False))
        f0 += c
    assert model.stats.deviceError == 0
    model.destroy()
    np.testing.assert_array_equal(got2, got)
    np.testing.assert_array_equal(got, np.concatenate(want))
