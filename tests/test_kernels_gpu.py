"""Per-kernel parity on the GPU: every case of the reference's
test/kernels.test.ts and test/shapes.test.ts, run through the C ABI's kernel
entry points and compared with the CPU oracle on identical seeded inputs,
with the reference's tolerances (kernels 2e-4/2e-3, shapes 3e-4/3e-3), plus
the out-of-bounds guard-band checks (kernels.test.ts:101-133,
shapes.test.ts:57-88).
"""
import numpy as np
import pytest

from tests.golden import cases
from tests.helpers import compare

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def run_case(torch, case, data, guard=0):
    from illumina import ops
    kind = case["kind"]
    if kind == "pw":
        n = case["h"] * case["w"] * case["outC"]
        dst = torch.full((n + guard,), -98765.0, device="cuda")
        ops.pointwise(dev(torch, data["src"]), case["h"], case["w"], case["inC"], dev(torch, data["w"]),
                      dev(torch, data["b"]), case["outC"], case["act"],
                      dev(torch, data["res"]) if case["residual"] else None, dst=dst)
    elif kind == "dwpw":
        n = data["outH"] * data["outW"] * case["outC"]
        dst = torch.full((n + guard,), -98765.0, device="cuda")
        ops.dwpw(dev(torch, data["src"]), case["inH"], case["inW"], case["inC"], dev(torch, data["dw_w"]),
                 dev(torch, data["dw_b"]), case["midAct"], dev(torch, data["pw_w"]), dev(torch, data["pw_b"]),
                 case["outC"], case["k"], case["stride"], case["act"],
                 dev(torch, data["res"]) if case["residual"] else None, dst=dst)
    elif kind == "conv":
        n = data["outH"] * data["outW"] * case["outC"]
        dst = torch.full((n + guard,), -98765.0, device="cuda")
        ops.conv(dev(torch, data["src"]), case["inH"], case["inW"], case["inC"], dev(torch, data["w"]),
                 dev(torch, data["b"]), case["outC"], case["k"], case["stride"], case["act"], dst=dst)
    else:
        n = 4 * case["ch"] * case["cw"] * case["outC"]
        dst = torch.full((n + guard,), -98765.0, device="cuda")
        ops.lateral(dev(torch, data["coarse"]), case["ch"], case["cw"], dev(torch, data["skip"]), case["skipC"],
                    dev(torch, data["w"]), dev(torch, data["b"]), case["outC"], case["act"], dst=dst)
    torch.cuda.synchronize()
    out = dst.cpu().numpy()
    return out[:n], out[n:]


@pytest.mark.parametrize("engine", ["simt", "tensor"])
@pytest.mark.parametrize("case", cases.all_cases(), ids=lambda c: c["id"])
def test_kernel_matches_oracle(torch, case, engine):
    """Every case on both engines; the tensor engine (tcgen05, 3xTF32) meets the same tolerances."""
    from illumina import ops
    if engine == "tensor" and case["kind"] == "conv":
        pytest.skip("the stem conv has one engine")
    data = cases.draw(case)
    want = cases.oracle_output(case, data)
    ops.set_engine(engine)
    try:
        got, tail = run_case(torch, case, data, guard=64)
    finally:
        ops.set_engine("simt")
    max_abs, max_rel, worst = compare(got, want, *case["tol"])
    assert worst == [], f"maxAbs={max_abs:.3e} maxRel={max_rel:.3e} worst={worst}"
    assert (tail == -98765.0).all(), "kernel wrote past the end of its output"


def test_pointwise_writes_nothing_outside_destination(torch):
    """kernels.test.ts:101-133: 13x13 px, 8->12 ch, tiles never divide evenly."""
    from illumina import ops
    st = 7
    src, st = cases.random_floats(st, 13 * 13 * 8, 1)
    w, st = cases.random_floats(st, 12 * 8, 0.25)
    b, st = cases.random_floats(st, 12, 0.5)
    n = 13 * 13 * 12
    dst = torch.full((n + 64,), -12345.0, device="cuda")
    ops.pointwise(dev(torch, src), 13, 13, 8, dev(torch, w), dev(torch, b), 12, "linear", dst=dst)
    out = dst.cpu().numpy()
    assert (out[n:] == -12345.0).all()
    from oracle import reference as R
    _, _, worst = compare(out[:n], R.pointwise(src, 13, 13, 8, w, b, 12, "linear"), 2e-4, 2e-3)
    assert worst == []


def test_preprocess_matches_oracle(torch):
    """kernels.test.ts preprocess case: input tolerance 1e-5; sceneColor exact-ish (f32 here, not fp16)."""
    from illumina import ops
    from oracle import reference as R
    from oracle.arch import MEAN, STD
    px = cases.preprocess_image(32)
    rgba = px.astype(np.float32) / np.float32(255.0)
    want_in, want_scene = R.preprocess(rgba, 32, MEAN, STD, True, cases.PREPROCESS_EXPOSURE)
    frames = dev(torch, rgba)  # interleaved layout (S x S x 4)
    got_in, got_scene = ops.preprocess(frames, 1, 1, 32, True, cases.PREPROCESS_EXPOSURE)
    _, _, worst = compare(got_in.cpu().numpy(), want_in, 1e-5, 1e-5)
    assert worst == []
    _, _, worst = compare(got_scene.cpu().numpy(), want_scene, 1e-6, 1e-6)
    assert worst == []
    # planar layout gives the same tensor
    planar = dev(torch, cases.rgba_bytes_to_planar(px, 32))
    got2, _ = ops.preprocess(planar, 1, 0, 32, True, cases.PREPROCESS_EXPOSURE)
    np.testing.assert_array_equal(got2.cpu().numpy(), got_in.cpu().numpy())


@pytest.mark.parametrize("lh,lw", [(16, 16), (32, 32), (7, 7)])
def test_bilateral_matches_oracle(torch, lh, lw):
    from illumina import ops
    from oracle import reference as R
    st = 0xB11A + lh
    low, st = cases.random_floats(st, lh * lw * 4, 0.5)
    low = (low + 0.5).astype(np.float32)
    guide, st = cases.random_floats(st, 4 * lh * lw * 4, 0.5)
    guide = (guide + 0.5).astype(np.float32)
    want = R.bilateral_upsample(low, lh, lw, 4, guide, 2 * lw, 4, 0.12)
    got = ops.bilateral(dev(torch, low), lh, lw, 4, dev(torch, guide), 4, 0.12)
    _, _, worst = compare(got.cpu().numpy(), want, 1e-5, 1e-5)
    assert worst == []


def test_head_matches_oracle(torch):
    from illumina import ops
    from oracle import reference as R
    st = 0x4EAD
    src, st = cases.random_floats(st, 37 * 32, 2.0)
    w, st = cases.random_floats(st, 32, 0.3)
    got = ops.head(dev(torch, src), 37, 32, dev(torch, w), 0.25)
    want = R.head(src, 37, 32, w, np.float32(0.25))
    _, _, worst = compare(got.cpu().numpy(), want, 1e-6, 1e-6)
    assert worst == []


def test_op_argument_errors(torch):
    import illumina
    from illumina import ops
    x = torch.zeros(64, device="cuda")
    with pytest.raises(illumina.IlluminaError, match="multiples of 4"):
        ops.pointwise(x, 2, 2, 6, x, x, 4, "linear")
    with pytest.raises(illumina.IlluminaError, match="kernel size must be 3 or 5"):
        ops.dwpw(x, 2, 2, 4, x, x, "linear", x, x, 4, 7, 1, "linear")


@pytest.mark.gpu
@pytest.mark.parametrize("which,name", [(0, "tf32_round vs cvt.rna.tf32.f32"), (1, "div6 vs IEEE a / 6.0f")])
def test_arith_helpers_exhaustive(which, name):
    """The tensor-core kernels replace two compiler operations by short
    branch-free sequences (the TF32 rounding of the 3xTF32 split, hardswish's
    division by 6); both must equal the replaced operation bit for bit on
    every non-NaN binary32 input."""
    import ctypes as C
    from illumina import _lib
    out = (C.c_ulonglong * 3)()
    _lib.check(_lib.lib().illumina_selftest(which, out))
    assert out[0] == (1 << 32) - 2 * ((1 << 23) - 1), name   # every pattern but the NaNs
    assert out[1] == 0, f"{name}: {out[1]} mismatches, e.g. input bits {out[2]:#010x}"


@pytest.mark.parametrize("h,w,in_c,out_c,res", [(14, 14, 416, 176, False), (7, 9, 352, 24, True)])
def test_pointwise_split_k_matches_oracle(torch, h, w, in_c, out_c, res):
    """Pointwise ops with a long K walk and few 128-pixel tiles (the bottleneck
    shapes at small batches) take the split-K path of the tensor engine: fp32
    partials per K split, summed in split order by a reduction launch; compared
    with the oracle at the kernel tolerance (2e-4 / 2e-3)."""
    from illumina import _lib, ops
    from oracle import reference as R
    st = 0x5B17 + in_c
    src, st = cases.random_floats(st, h * w * in_c, 1.0)
    wt, st = cases.random_floats(st, out_c * in_c, 0.1)
    b, st = cases.random_floats(st, out_c, 0.5)
    r, st = cases.random_floats(st, h * w * out_c, 1.0)
    want = R.pointwise(src, h, w, in_c, wt, b, out_c, "hardswish", r if res else None)
    lib = _lib.lib()
    lib.illumina_set_op_engine(_lib.ENGINE["tensor"])
    try:
        got = ops.pointwise(dev(torch, src), h, w, in_c, dev(torch, wt), dev(torch, b), out_c, "hardswish",
                            dev(torch, r) if res else None)
        torch.cuda.synchronize()
    finally:
        lib.illumina_set_op_engine(_lib.ENGINE["simt"])
    _, _, worst = compare(got.cpu().numpy(), want, 2e-4, 2e-3)
    assert worst == [], worst
