"""illumina_op_dwpw_noalloc: the fused depthwise -> pointwise op for callers
that cannot allocate device memory (a real-time frame loop with a fixed
memory budget, or a host whose memory manager owns the device heap). It
repacks the depthwise weights into a fixed array compiled into the library
instead of a temporary allocation.

Checked through the C ABI against illumina_op_dwpw (the allocating entry
point) on two calls in a row that reuse the shared array with different
shapes, with the reference kernel tolerance (2e-4 / 2e-3), and for the
size limit. This file is collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest

from tests.golden import cases
from tests.helpers import compare

pytestmark = pytest.mark.gpu

MAX_FLOATS = 65536  # ILLUMINA_NOALLOC_DW_MAX_FLOATS in include/illumina.h


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _call(fn, torch, case, data):
    from illumina import _lib
    pad = (case["k"] - 1) >> 1
    oh = (case["inH"] + 2 * pad - case["k"]) // case["stride"] + 1
    ow = (case["inW"] + 2 * pad - case["k"]) // case["stride"] + 1
    d = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)).cuda()
         for k, v in data.items() if isinstance(v, np.ndarray)}
    dst = torch.full((oh * ow * case["outC"],), -5.0, device="cuda")
    act = _lib.ACT
    status = fn(d["src"].data_ptr(), case["inH"], case["inW"], case["inC"], d["dw_w"].data_ptr(),
                d["dw_b"].data_ptr(), act[case["midAct"]], d["pw_w"].data_ptr(), d["pw_b"].data_ptr(),
                case["outC"], case["k"], case["stride"], act[case["act"]],
                d["res"].data_ptr() if case["residual"] else None, dst.data_ptr(), None)
    _lib.check(status)
    torch.cuda.synchronize()
    return dst.cpu().numpy()


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls(torch):
    from illumina import _lib
    lib = _lib.lib()
    by_id = {c["id"]: c for c in cases.all_cases()}
    # a wide case first (704*25 packed floats), then a narrow one that reuses the
    # array's first 16*9 floats while stale weights from the first call remain beyond
    for cid in ("s_dwpw10", "k_dwpw0"):
        case = by_id[cid]
        data = cases.draw(case)
        got = _call(lib.illumina_op_dwpw_noalloc, torch, case, data)
        want = _call(lib.illumina_op_dwpw, torch, case, data)
        _, _, worst = compare(got, want, 2e-4, 2e-3)
        assert worst == [], (cid, worst)
        _, _, worst = compare(got, cases.oracle_output(case, data), *case["tol"])
        assert worst == [], (cid, worst)


def test_noalloc_runs_simt_whatever_engine_the_thread_selected(torch):
    """With the tensor engine selected for the thread, illumina_op_dwpw runs
    tcgen05 while the no-alloc variant still runs the SIMT kernel: both match
    the oracle within the kernel tolerance and each other within it too."""
    from illumina import _lib
    lib = _lib.lib()
    case = {c["id"]: c for c in cases.all_cases()}["s_dwpw10"]
    data = cases.draw(case)
    lib.illumina_set_op_engine(_lib.ENGINE["tensor"])
    try:
        got = _call(lib.illumina_op_dwpw_noalloc, torch, case, data)
        tc = _call(lib.illumina_op_dwpw, torch, case, data)
    finally:
        lib.illumina_set_op_engine(_lib.ENGINE["simt"])
    want = cases.oracle_output(case, data)
    for out in (got, tc):
        _, _, worst = compare(out, want, *case["tol"])
        assert worst == [], worst
    _, _, worst = compare(got, tc, *case["tol"])
    assert worst == []


def test_noalloc_rejects_weights_beyond_the_fixed_scratch(torch):
    from illumina import _lib
    lib = _lib.lib()
    in_c = (MAX_FLOATS // 25 + 4) // 4 * 4  # in_c * 25 > MAX_FLOATS
    x = torch.zeros(in_c * 4, device="cuda")
    status = lib.illumina_op_dwpw_noalloc(x.data_ptr(), 1, 1, in_c, x.data_ptr(), x.data_ptr(), 0, x.data_ptr(),
                                          x.data_ptr(), 4, 5, 1, 0, None, x.data_ptr(), None)
    assert status == _lib.INVALID_ARG
    assert b"exceeds the fixed scratch" in lib.illumina_last_error()
