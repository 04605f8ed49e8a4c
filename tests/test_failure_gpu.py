"""Failure surfacing on the GPU without a GPU fault.

The tensor-core kernels bound every wait on an mbarrier. Here the model's wait
limit is lowered to one cycle, so the pipeline waits give up at the first
probe that finds a phase incomplete (a consumer whose producer has not
delivered yet); each role that gives up records it in the model's error word
and leaves its loop, and the waits with which the producers drain their own
copies and the MMA thread its own MMAs keep the default limit, so nothing is
in flight when TMEM is released and the CTA leaves. The host reads the word
and reports ILLUMINA_TIMEOUT: a device-buffer forward at the next call or
illumina_model_sync, a host-buffer forward at its own return. Afterwards the
default limit gives the same results as before (the split-K arrival counters
that a unit that gave up may have left behind are reset by the report).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.mark.parametrize("size,batch", [(64, 2), (448, 1)])
def test_timeout_reported_and_model_recovers(torch, size, batch):
    import illumina
    from illumina import _lib
    m = illumina.createDepthModel(illumina.buildArchitecture(size), synthSeed=0, maxBatch=batch)
    assert m.stats.engine == "tensor"
    frames = torch.empty((batch, 3, size, size), device="cuda")
    _lib.check(_lib.lib().illumina_generate_frames(0, 40, batch, size, frames.data_ptr(), None))
    out = torch.empty((batch, size, size), device="cuda")
    m.forward(frames, disparity=out)
    m.sync()
    want = out.cpu().numpy()

    m.setWaitLimit(1)
    m.forward(frames, disparity=out)  # queued on device buffers: OK at the call
    with pytest.raises(illumina.IlluminaError, match="gave up a bounded wait") as e:
        m.sync()
    assert e.value.status == _lib.TIMEOUT
    assert m.stats.deviceError == 0  # the report cleared the word
    with pytest.raises(illumina.IlluminaError, match="in this call") as e:
        m.forward(frames.cpu().numpy())  # host buffers: synchronous, reports its own kernels
    assert e.value.status == _lib.TIMEOUT

    m.setWaitLimit(0)
    m.forward(frames, disparity=out)
    m.sync()
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    m.destroy()


def test_sync_without_error_is_ok(torch):
    import illumina
    m = illumina.createDepthModel(illumina.buildArchitecture(64), synthSeed=1)
    m.forward(np.zeros((1, 3, 64, 64), np.float32))
    m.sync()
    assert m.stats.deviceError == 0
    with pytest.raises(illumina.IlluminaError):
        m.setWaitLimit(-1)
    m.destroy()
