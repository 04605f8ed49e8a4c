"""The depth model: the Python face of src/model/runner.ts
(createDepthModel / DepthModel) over the native runtime.

Frames are [n, 3, S, S] (or [3, S, S]) float32 in [0, 1], sRGB-encoded by
default, given as numpy arrays (host) or torch CUDA tensors (device). Device
memory, streams and the optional torch views are plumbing; every kernel is
the library's.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import (ENGINE, FRAME_RGB_PLANAR, FRAME_RGBA_INTERLEAVED, PRECISION_BF16, PRECISION_F32, ModelOptions, Stats,
                   check, lib, ptr, stream_handle)
from .arch import Architecture, buildArchitecture
from .weights import flatten


class _DeviceView:
    """Exposes a raw device buffer through __cuda_array_interface__ (for torch.as_tensor)."""

    def __init__(self, address: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"data": (address, False), "shape": shape, "typestr": typestr,
                                          "version": 3, "strides": None, "stream": None}


@dataclass(frozen=True)
class DepthModelStats:
    dispatches: int
    launches: int
    arenaBytes: int
    naiveArenaBytes: int
    weightBytes: int
    deviceBytes: int
    maxBatch: int
    precision: str
    inputSize: int
    engine: str
    deviceError: int


def _is_torch(x) -> bool:
    return hasattr(x, "data_ptr") and hasattr(x, "is_cuda")


class DepthModel:
    """DepthModel (runner.ts:103-146). Create with createDepthModel."""

    def __init__(self, handle: int, arch: Architecture, max_batch: int, uvScale=(1.0, 1.0), uvOffset=(0.0, 0.0)):
        self._h = C.c_void_p(handle)
        self.arch = arch
        self.maxBatch = max_batch
        self.uvScale = tuple(uvScale)
        self.uvOffset = tuple(uvOffset)

    # -- inference --------------------------------------------------------
    def _layout(self, frames):
        shape = tuple(frames.shape)
        S = self.arch.inputSize
        if shape[-3:] == (3, S, S):
            return FRAME_RGB_PLANAR, (1 if len(shape) == 3 else shape[0])
        if shape[-3:] == (S, S, 4):
            return FRAME_RGBA_INTERLEAVED, (1 if len(shape) == 3 else shape[0])
        raise ValueError(f"frames must be [n,3,{S},{S}] or [n,{S},{S},4], got {list(shape)}")

    def forward(self, frames, disparity=None, depthLow=None, stream=None):
        """The hot path for n independent frames (preprocess -> 38 convs -> head -> bilateralUp).

        Returns the disparity [n, S, S] (numpy for host input, torch for device
        input) and writes depth_low [n, S/2, S/2] into `depthLow` when given.
        """
        layout, n = self._layout(frames)
        S = self.arch.inputSize
        if _is_torch(frames):
            import torch
            if not frames.is_contiguous() or frames.dtype != torch.float32:
                raise ValueError("frames must be a contiguous float32 tensor")
            if disparity is None:
                disparity = torch.empty((n, S, S), dtype=torch.float32, device=frames.device)
        else:
            frames = np.ascontiguousarray(frames, np.float32)
            if disparity is None:
                disparity = np.empty((n, S, S), np.float32)
        check(lib().illumina_forward(self._h, ptr(frames), n, layout, ptr(disparity), ptr(depthLow),
                                     stream_handle(stream)))
        return disparity

    def forwardAsync(self, frames, disparity, stream=None):
        """forward() without waiting (illumina_forward_async): `frames` and `disparity` are
        pinned host buffers (numpy views of pinned torch tensors, or pinned CPU tensors) that
        must stay untouched until sync(); the whole batch runs as one graph while the
        neighbouring calls' transfers overlap it. Returns `disparity`."""
        layout, n = self._layout(frames)
        S = self.arch.inputSize
        if tuple(disparity.shape) != (n, S, S):
            raise ValueError(f"disparity must be [{n}, {S}, {S}]")
        check(lib().illumina_forward_async(self._h, ptr(frames), n, layout, ptr(disparity), stream_handle(stream)))
        return disparity

    def forwardSourceAsync(self, rgba8, disparity, uvScale=None, uvOffset=None, mirror: bool = False, stream=None):
        """forwardSource() without waiting (illumina_forward_source_async): `rgba8` [n, h, w, 4]
        uint8 and `disparity` [n, S, S] float32 are pinned host buffers that must stay untouched
        until sync(). Returns `disparity`."""
        if rgba8.ndim == 3:
            rgba8 = rgba8[None]
        n, h, w = int(rgba8.shape[0]), int(rgba8.shape[1]), int(rgba8.shape[2])
        S = self.arch.inputSize
        if rgba8.shape[-1] != 4 or tuple(disparity.shape) != (n, S, S):
            raise ValueError(f"rgba8 must be [n, h, w, 4] and disparity [{n}, {S}, {S}]")
        sc = (C.c_float * 2)(*(uvScale if uvScale is not None else self.uvScale))
        of = (C.c_float * 2)(*(uvOffset if uvOffset is not None else self.uvOffset))
        check(lib().illumina_forward_source_async(self._h, ptr(rgba8), n, w, h, sc, of, int(bool(mirror)),
                                                  ptr(disparity), stream_handle(stream)))
        return disparity

    def forwardInput(self, inputs, disparity=None, depthLow=None):
        """forwardReference from given network inputs (ref-forward.ts with an "input" bundle):
        [n, S, S, 4] float32 channels-last preprocess outputs. Synchronous; returns the disparity
        [n, S, S] (numpy unless `disparity` is given). fp32 models only."""
        S = self.arch.inputSize
        x = inputs if _is_torch(inputs) else np.ascontiguousarray(inputs, np.float32)
        shape = tuple(x.shape)
        if len(shape) == 3:
            shape = (1,) + shape
        if shape[1:] != (S, S, 4):
            raise ValueError(f"inputs must be [n,{S},{S},4], got {list(x.shape)}")
        n = shape[0]
        if disparity is None:
            disparity = np.empty((n, S, S), np.float32)
        check(lib().illumina_forward_input(self._h, ptr(x), n, ptr(disparity), ptr(depthLow)))
        return disparity

    def sampleSource(self, rgba8, uvScale=None, uvOffset=None, mirror: bool = False, frames=None, stream=None):
        """The source-texture read of makePreprocess (io.ts:64-118): n 8-bit RGBA
        images [n, h, w, 4] (CUDA uint8 tensor, any size) sampled at the network
        resolution with uv * uvScale + uvOffset (the model's createDepthModel
        options unless given), linear filtering, clamp-to-edge. Returns the planar
        float frames [n, 3, S, S] that forward() takes."""
        import torch
        if rgba8.dim() == 3:
            rgba8 = rgba8[None]
        if rgba8.dtype != torch.uint8 or not rgba8.is_cuda or not rgba8.is_contiguous() or rgba8.shape[-1] != 4:
            raise ValueError("rgba8 must be a contiguous CUDA uint8 tensor [n, h, w, 4]")
        n, h, w = rgba8.shape[0], rgba8.shape[1], rgba8.shape[2]
        S = self.arch.inputSize
        if frames is None:
            frames = torch.empty((n, 3, S, S), dtype=torch.float32, device=rgba8.device)
        sc = (C.c_float * 2)(*(uvScale if uvScale is not None else self.uvScale))
        of = (C.c_float * 2)(*(uvOffset if uvOffset is not None else self.uvOffset))
        check(lib().illumina_sample_source(ptr(rgba8), n, w, h, sc, of, int(bool(mirror)), S, ptr(frames),
                                           stream_handle(stream)))
        return frames

    def forwardSource(self, rgba8, uvScale=None, uvOffset=None, mirror: bool = False, disparity=None, stream=None):
        """forward() on 8-bit RGBA source images [n, h, w, 4] (numpy uint8 on the host or a CUDA
        uint8 tensor): the source read of makePreprocess, then the hot path, in one call
        (illumina_forward_source). Returns the disparity [n, S, S] (numpy for a host source,
        a CUDA tensor for a device source, or `disparity` when given)."""
        host = not _is_torch(rgba8)
        if host:
            rgba8 = np.ascontiguousarray(rgba8, np.uint8)
        else:
            import torch
            if rgba8.dtype != torch.uint8 or not rgba8.is_cuda or not rgba8.is_contiguous():
                raise ValueError("rgba8 must be a contiguous uint8 array or CUDA tensor [n, h, w, 4]")
        if rgba8.ndim == 3:
            rgba8 = rgba8[None]
        if rgba8.shape[-1] != 4:
            raise ValueError(f"rgba8 must be [n, h, w, 4], got {list(rgba8.shape)}")
        n, h, w = int(rgba8.shape[0]), int(rgba8.shape[1]), int(rgba8.shape[2])
        S = self.arch.inputSize
        if disparity is None:
            if host:
                disparity = np.empty((n, S, S), np.float32)
            else:
                import torch
                disparity = torch.empty((n, S, S), dtype=torch.float32, device=rgba8.device)
        sc = (C.c_float * 2)(*(uvScale if uvScale is not None else self.uvScale))
        of = (C.c_float * 2)(*(uvOffset if uvOffset is not None else self.uvOffset))
        check(lib().illumina_forward_source(self._h, ptr(rgba8), n, w, h, sc, of, int(bool(mirror)), ptr(disparity),
                                            stream_handle(stream)))
        return disparity

    def record(self, frame, stream=None):
        """record (runner.ts:440-449): one streaming frame blended with the temporal history."""
        layout, n = self._layout(frame)
        if n != 1:
            raise ValueError("record takes one frame")
        if not _is_torch(frame):
            frame = np.ascontiguousarray(frame, np.float32)
        check(lib().illumina_model_record(self._h, ptr(frame), layout, stream_handle(stream)))

    def sync(self):
        """Waits for this model's queued work; raises IlluminaError (status TIMEOUT) when a
        kernel gave up a bounded wait since the last check."""
        check(lib().illumina_model_sync(self._h))

    def setWaitLimit(self, cycles: int):
        """Cycles a tensor-core pipeline wait may take before the kernel gives up (0 = default)."""
        check(lib().illumina_model_set_wait_limit(self._h, int(cycles)))

    def swapHistory(self):
        check(lib().illumina_model_swap_history(self._h))

    def outputParity(self) -> int:
        return lib().illumina_model_output_parity(self._h)

    def freshParity(self) -> int:
        return lib().illumina_model_fresh_parity(self._h)

    def debugDepth(self, index: int):
        """Depth slot `index` as a torch CUDA tensor view [S, S, 4] (stabilised, raw, change, valid)."""
        import torch
        p = C.c_void_p()
        check(lib().illumina_model_depth_slot(self._h, index, C.byref(p)))
        S = self.arch.inputSize
        return torch.as_tensor(_DeviceView(p.value, (S, S, 4)), device="cuda")

    def currentDepth(self):
        return self.debugDepth(self.freshParity())

    def depthSlotPointer(self, index: int) -> int:
        p = C.c_void_p()
        check(lib().illumina_model_depth_slot(self._h, index, C.byref(p)))
        return p.value

    def setExposure(self, exposure: float):
        check(lib().illumina_model_set_exposure(self._h, float(exposure)))

    def setTemporal(self, baseAlpha: float, motionSensitivity: float, rangeSigma: float):
        check(lib().illumina_model_set_temporal(self._h, float(baseAlpha), float(motionSensitivity),
                                                float(rangeSigma)))

    @property
    def stats(self) -> DepthModelStats:
        s = Stats()
        check(lib().illumina_model_stats(self._h, C.byref(s)))
        return DepthModelStats(s.dispatches, s.launches, s.arena_bytes, s.naive_arena_bytes, s.weight_bytes,
                               s.device_bytes, s.max_batch, "bf16" if s.precision == PRECISION_BF16 else "f32",
                               s.input_size, "tensor" if s.gemm_engine == 0 else "simt", s.device_error)

    def profile(self, frames, reps: int = 3):
        """Per-op mean device time in ms (GpuProfiler analogue), frames on the device."""
        layout, n = self._layout(frames)
        out = np.zeros(len(self.arch.ops), np.float32)
        check(lib().illumina_model_profile(self._h, ptr(frames), n, layout, reps, out.ctypes.data, out.size))
        return {op.name: float(t) for op, t in zip(self.arch.ops, out)}

    def debugTensor(self, name: str, frame: int = 0):
        """debugTensor (runner.ts:466-476): (data [h, w, c] float32 numpy of batch frame `frame` of the
        last forward, liveAtEnd) or None. "scene_color" (the preprocess's linear colour) is kept by a
        keepIntermediates model."""
        if name == "scene_color":
            S = self.arch.inputSize
            out = np.empty((S, S, 4), np.float32)
        elif name not in self.arch.tensors or name == "depth":
            return None
        else:
            s = self.arch.tensors[name]
            out = np.empty((s.h, s.w, s.c), np.float32)
        h, w, c, live = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        check(lib().illumina_model_debug_tensor_frame(self._h, name.encode(), int(frame), out.ctypes.data, out.size,
                                                      C.byref(h), C.byref(w), C.byref(c), C.byref(live)))
        return out, bool(live.value)

    def destroy(self):
        if self._h:
            lib().illumina_model_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.destroy()
        except Exception:  # noqa: BLE001
            pass


def createDepthModel(arch: Architecture | None = None, weights: dict | None = None, idm: bytes | None = None,
                     decodeSrgb: bool = True, exposure: float = 1.0, device: int = 0, maxBatch: int = 1,
                     precision: str = "f32", keepIntermediates: bool = False, synthSeed: int = 1,
                     rangeSigma: float = 0.12, temporalBase: float = 0.35,
                     temporalSensitivity: float = 3.0, engine: str = "tensor", uvScale=(1.0, 1.0),
                     uvOffset=(0.0, 0.0)) -> DepthModel:
    """createDepthModel (runner.ts:160-485).

    Weights: a WeightMap (`weights`), or an .idm container (`idm`), else the
    seeded Kaiming fallback synthesizeWeights(arch, synthSeed) (main.ts:61).
    `engine` selects the pointwise-shaped ops' engine: "tensor" (tcgen05) or "simt".
    `uvScale`/`uvOffset` (runner.ts:88-89) transform the source uv of sampleSource /
    forwardSource.
    """
    arch = arch or buildArchitecture(448)
    o = ModelOptions()
    lib().illumina_model_options_default(C.byref(o))
    o.input_size = arch.inputSize
    o.device = device
    o.max_batch = maxBatch
    o.precision = {"f32": PRECISION_F32, "bf16": PRECISION_BF16}[precision]
    o.decode_srgb = 1 if decodeSrgb else 0
    o.exposure = exposure
    o.range_sigma = rangeSigma
    o.temporal_base = temporalBase
    o.temporal_sensitivity = temporalSensitivity
    o.keep_intermediates = 1 if keepIntermediates else 0
    o.synth_seed = synthSeed & 0xFFFFFFFF
    o.gemm_engine = ENGINE[engine]
    keep = []
    if weights is not None:
        blob = flatten(arch, weights)
        keep.append(blob)
        o.weights = blob.ctypes.data_as(C.POINTER(C.c_float))
        o.weights_count = blob.size
    elif idm is not None:
        buf = C.create_string_buffer(bytes(idm), len(idm))
        keep.append(buf)
        o.idm_bytes = C.cast(buf, C.c_void_p)
        o.idm_len = len(idm)
    h = C.c_void_p()
    check(lib().illumina_model_create(C.byref(o), C.byref(h)))
    return DepthModel(h.value, arch, maxBatch, uvScale, uvOffset)


def cropTransform(width: int, height: int):
    """cropTransform (scene/blit.ts:80-86): [scaleX, scaleY, offsetX, offsetY] of the
    largest centred square, for uvScale = out[:2], uvOffset = out[2:]."""
    out = (C.c_float * 4)()
    lib().illumina_crop_transform(int(width), int(height), out)
    return list(out)
