"""The frame graph: the Python face of src/engine/frame.ts (renderFrame).

A frame is inference (one CUDA-graph launch of the 40 ops) followed by one
shading + tone-map kernel, all on one stream: the CUDA analogue of the
reference's single encoder and single submit.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class FrameResult:
    """FrameResult (frame.ts:62-71)."""
    dispatches: int   # logical compute dispatches, including shading
    draws: int        # the composite (fused into the shading kernel here)
    encoders: int
    submits: int      # graph launches + the shading launch, on one stream
    launches: int     # kernels actually launched


def renderFrame(model, renderer, frame=None, skipInference: bool = False, stream=None) -> FrameResult:
    """renderFrame (frame.ts:80-167).

    With skipInference the shading reads freshParity(), the slot last written,
    and the temporal ping-pong does not advance (frame.ts:108-164).
    """
    parity = model.freshParity() if skipInference else model.outputParity()
    launches = 0
    if not skipInference:
        if frame is None:
            raise ValueError("renderFrame needs a frame unless skipInference is set")
        model.record(frame, stream=stream)
        launches += model.stats.launches
    renderer.recordShade(parity, stream=stream)
    launches += 1
    if not skipInference:
        model.swapHistory()
    dispatches = 1 if skipInference else model.stats.dispatches + 1
    return FrameResult(dispatches=dispatches, draws=1, encoders=1, submits=1, launches=launches)
