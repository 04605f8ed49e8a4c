"""illumina_forward_async: the forward of pinned host buffers queued without
waiting (upload, one graph per call, download), consecutive calls alternating
two device staging slots. Every result must equal the synchronous forward of
the same frames bit for bit (same batch size, same graph)."""
import numpy as np
import pytest

from tests.golden import cases

pytestmark = pytest.mark.gpu
S = 64


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _frames(torch, n, seed):
    from illumina import _lib
    out = torch.empty((n, 3, S, S), device="cuda")
    _lib.check(_lib.lib().illumina_generate_frames(1, seed, n, S, out.data_ptr(), None))
    return out


def test_async_calls_equal_sync_forward(torch):
    import illumina
    n, calls = 6, 5
    m = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=cases.NET64_SEED, maxBatch=n)
    dev = [_frames(torch, n, 100 * i) for i in range(calls)]
    want = []
    for f in dev:
        want.append(m.forward(f).cpu().numpy())
    torch.cuda.synchronize()
    host_in = [torch.empty((n, 3, S, S), dtype=torch.float32, pin_memory=True) for _ in range(calls)]
    host_out = [torch.empty((n, S, S), dtype=torch.float32, pin_memory=True) for _ in range(calls)]
    for i in range(calls):
        host_in[i].copy_(dev[i].cpu())
    for i in range(calls):
        m.forwardAsync(host_in[i].numpy(), host_out[i].numpy())
    m.sync()
    assert m.stats.deviceError == 0
    for i in range(calls):
        np.testing.assert_array_equal(host_out[i].numpy(), want[i])
    # an asynchronous call, then a synchronous one on other buffers, then sync
    m.forwardAsync(host_in[1].numpy(), host_out[0].numpy())
    got = m.forward(host_in[2].numpy())
    m.sync()
    np.testing.assert_array_equal(host_out[0].numpy(), want[1])
    np.testing.assert_array_equal(got, want[2])
    m.destroy()


def test_async_rejects_pageable_buffers(torch):
    import illumina
    m = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=0, maxBatch=2)
    frames = np.zeros((2, 3, S, S), np.float32)
    out = np.zeros((2, S, S), np.float32)
    with pytest.raises(illumina.IlluminaError, match="pinned host memory"):
        m.forwardAsync(frames, out)
    pinned_in = torch.zeros((3, 3, S, S), dtype=torch.float32, pin_memory=True)
    pinned_out = torch.zeros((3, S, S), dtype=torch.float32, pin_memory=True)
    with pytest.raises(illumina.IlluminaError, match="outside"):
        m.forwardAsync(pinned_in.numpy(), pinned_out.numpy())
    m.destroy()


@pytest.mark.parametrize("sw,sh", [(S, S), (96, 80)])
def test_source_async_equals_source_forward(torch, sw, sh):
    """illumina_forward_source_async over three calls (a 96x80 source does not fit the
    slots' staging and uses the model's source buffers) equals the synchronous
    forwardSource of the same images bit for bit (same batch, same graph)."""
    import illumina
    n, calls = 4, 3
    rng = np.random.default_rng(sw)
    m = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=cases.NET64_SEED, maxBatch=n)
    src = [torch.from_numpy(rng.integers(0, 256, (n, sh, sw, 4), dtype=np.uint8)).pin_memory() for _ in range(calls)]
    want = [m.forwardSource(s.numpy(), (0.9, 0.8), (0.05, 0.1), True) for s in src]
    out = [torch.empty((n, S, S), dtype=torch.float32, pin_memory=True) for _ in range(calls)]
    for i in range(calls):
        m.forwardSourceAsync(src[i].numpy(), out[i].numpy(), (0.9, 0.8), (0.05, 0.1), True)
    m.sync()
    assert m.stats.deviceError == 0
    for i in range(calls):
        np.testing.assert_array_equal(out[i].numpy(), want[i])
    m.destroy()


def test_destroy_waits_for_async_work(torch):
    """Destroying the model right after an asynchronous call waits for that call:
    the disparity is complete afterwards."""
    import illumina
    n = 2
    m = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=cases.NET64_SEED, maxBatch=n)
    dev = _frames(torch, n, 7)
    want = m.forward(dev).cpu().numpy()
    torch.cuda.synchronize()
    host_in = torch.empty((n, 3, S, S), dtype=torch.float32, pin_memory=True)
    host_in.copy_(dev.cpu())
    host_out = torch.full((n, S, S), -1.0, dtype=torch.float32, pin_memory=True)
    m.forwardAsync(host_in.numpy(), host_out.numpy())
    m.destroy()
    np.testing.assert_array_equal(host_out.numpy(), want)
