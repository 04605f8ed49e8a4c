"""The host-buffer forward runs in frame chunks (16, 32, 48, ..., then 16 frames, from 128 on), uploads and
downloads on their own streams overlapping the neighbouring chunks' graphs.
Frames are independent, so the result must equal, bit for bit, device-pointer
forwards over the same chunk sizes (the launch plan depends on the batch size,
so whole-batch forwards may round differently and are compared at the network
tolerance instead).
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


@pytest.mark.parametrize("n,chunks", [(40, [20, 20]), (33, [17, 16]), (130, [16, 32, 48, 18, 16]), (256, [16, 32, 48, 64, 80, 16])])
def test_chunked_host_forward_matches_device_chunks(torch, n, chunks):
    import illumina
    from illumina import _lib
    S = 64
    model = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=3, maxBatch=n, device=0)
    frames = torch.empty((n, 3, S, S), dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib().illumina_generate_frames(1, 11, n, S, frames.data_ptr(), None))
    host_in = frames.cpu().pin_memory()
    host_out = torch.empty((n, S, S), dtype=torch.float32).pin_memory()
    model.forward(host_in.numpy(), disparity=host_out.numpy())
    got = host_out.numpy().copy()
    # pageable output buffer and device input: the same path, same result
    pageable = np.empty((n, S, S), np.float32)
    model.forward(frames, disparity=pageable)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(pageable, got)
    want, f0 = [], 0
    for c in chunks:
        d = model.forward(frames[f0:f0 + c].contiguous())
        torch.cuda.synchronize()
        want.append(d.cpu().numpy())
        f0 += c
    np.testing.assert_array_equal(got, np.concatenate(want))
    whole = model.forward(frames)
    torch.cuda.synchronize()
    assert float(np.abs(whole.cpu().numpy() - got).max()) <= 1e-5
    model.destroy()


def test_frames_at_any_4_byte_offset_match_aligned(torch):
    """The fused preprocess+stem reads planar frames as float4 groups when the
    pointer is 16-byte aligned and pixel by pixel otherwise; both give the same bits."""
    import illumina
    from illumina import _lib
    S, n = 64, 3
    model = illumina.createDepthModel(illumina.buildArchitecture(S), synthSeed=5, maxBatch=n, device=0)
    frames = torch.empty((n, 3, S, S), dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib().illumina_generate_frames(0, 7, n, S, frames.data_ptr(), None))
    want = model.forward(frames).cpu().numpy()
    for off in (1, 2, 3):
        buf = torch.zeros(n * 3 * S * S + 4, dtype=torch.float32, device="cuda")
        view = buf[off:off + n * 3 * S * S].view(n, 3, S, S)
        view.copy_(frames)
        assert view.data_ptr() % 16 != 0
        got = model.forward(view)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got.cpu().numpy(), want)
    model.destroy()
