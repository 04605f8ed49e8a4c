"""The procedural scene and its depth metrics: the Python face of
src/scene/procedural.ts (createProceduralScene -> ProceduralScene with
record / update / destroy) and src/scene/metrics.ts (evaluateDepth ->
DepthMetrics).

The reference draws the scene into an rgba8unorm colour texture and an
rgba16float truth texture and scores a prediction by reading both back to the
CPU. Here both run as native kernels on device buffers (torch tensors): the
scene renders a batch of frames straight into the planar float layout the
network takes, plus (depth, hit) truth pairs in float32, and the metrics are
reduced on the device, one block per frame, with only the 64-byte result per
frame copied back.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from ._lib import DepthMetricsC, SceneParamsC, check, lib, ptr, stream_handle


@dataclass(frozen=True)
class DepthMetrics:
    """DepthMetrics (metrics.ts:17-32)."""
    samples: int
    absRel: float
    rmse: float
    delta1: float
    delta2: float
    delta3: float
    scale: float
    shift: float


def sceneParams(timeSeconds: float | None = None, orbit: bool = False) -> SceneParamsC:
    """The scene uniforms: the initial block of createProceduralScene when
    timeSeconds is None (procedural.ts:295-299), else update(time, orbit) (:310-318)."""
    p = SceneParamsC()
    if timeSeconds is None:
        lib().illumina_scene_params_initial(C.byref(p))
    else:
        lib().illumina_scene_params_update(C.byref(p), float(timeSeconds), int(bool(orbit)))
    return p


def _check_out(t, shape, what):
    if t is None:
        return
    if tuple(t.shape) != tuple(shape) or not t.is_contiguous() or not t.is_cuda:
        raise ValueError(f"{what} must be a contiguous CUDA tensor of shape {tuple(shape)}")


def renderScenes(params, width: int, height: int, rgb=None, rgba8=None, truth=None, stream=None):
    """Renders len(params) frames (one SceneParams each) into the given device
    tensors: rgb [n, 3, H, W] float32, rgba8 [n, H, W, 4] uint8, truth [n, H, W, 2]
    float32 (any may be None)."""
    n = len(params)
    _check_out(rgb, (n, 3, height, width), "rgb")
    _check_out(rgba8, (n, height, width, 4), "rgba8")
    _check_out(truth, (n, height, width, 2), "truth")
    arr = (SceneParamsC * max(n, 1))(*params)
    check(lib().illumina_scene_render(arr, n, width, height, ptr(rgb), ptr(rgba8), ptr(truth),
                                      stream_handle(stream)))


class ProceduralScene:
    """ProceduralScene (procedural.ts:275-282). record() renders one frame into
    caller-owned buffers, as the reference draws into caller-owned targets."""

    def __init__(self):
        self.params = sceneParams()

    def update(self, timeSeconds: float, orbit: bool) -> None:
        self.params = sceneParams(timeSeconds, orbit)

    def record(self, width: int, height: int, rgb=None, rgba8=None, truth=None, stream=None) -> None:
        """rgb [1, 3, H, W] float32, rgba8 [1, H, W, 4] uint8, truth [1, H, W, 2] float32."""
        renderScenes([self.params], width, height, rgb=rgb, rgba8=rgba8, truth=truth, stream=stream)

    def destroy(self) -> None:
        """The caller owns the render targets; nothing to free."""


def createProceduralScene() -> ProceduralScene:
    """createProceduralScene (procedural.ts:292-330)."""
    return ProceduralScene()


def evaluateDepth(predicted, truth, width: int, height: int | None = None, predChannels: int = 1, stream=None):
    """evaluateDepth (metrics.ts:66-161) on device tensors: predicted [n, H, W(, C)]
    disparity (channel 0 of predChannels), truth [n, H, W, 2] (depth, hit).
    Returns a DepthMetrics, or a list of them when n > 1."""
    import torch

    height = width if height is None else height
    n = truth.shape[0] if truth.dim() == 4 else 1
    if truth.numel() != n * height * width * 2 or predicted.numel() != n * height * width * predChannels:
        raise ValueError("evaluateDepth: predicted/truth sizes do not match the frame size")
    if not (predicted.is_cuda and truth.is_cuda and predicted.is_contiguous() and truth.is_contiguous()):
        raise ValueError("evaluateDepth: predicted and truth must be contiguous CUDA tensors")
    out = torch.empty((n, C.sizeof(DepthMetricsC)), dtype=torch.uint8, device=truth.device)
    check(lib().illumina_evaluate_depth(ptr(predicted), predChannels, ptr(truth), n, width, height, ptr(out),
                                        stream_handle(stream)))
    if stream is not None and not isinstance(stream, int):
        stream.synchronize()
    else:
        torch.cuda.synchronize(truth.device)
    raw = out.cpu().numpy().tobytes()
    res = []
    for i in range(n):
        m = DepthMetricsC.from_buffer_copy(raw, i * C.sizeof(DepthMetricsC))
        res.append(DepthMetrics(int(m.samples), m.abs_rel, m.rmse, m.delta1, m.delta2, m.delta3, m.scale,
                                m.shift))
    return res[0] if n == 1 and truth.dim() != 4 else res
