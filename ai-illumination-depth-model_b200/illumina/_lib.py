"""ctypes binding of libillumina.so (the C ABI in include/illumina.h).

The library is the product: there is no Python or CPU fallback. Loading fails
loudly when the shared library has not been built.
"""
from __future__ import annotations

import ctypes as C
import os

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_DIR, "libillumina.so")

OK, INVALID_ARG, BAD_WEIGHTS, ARCH_MISMATCH, CUDA_ERROR, TIMEOUT, NO_DEVICE = range(7)
PRECISION_F32, PRECISION_BF16 = 0, 1
FRAME_RGB_PLANAR, FRAME_RGBA_INTERLEAVED = 0, 1
ENGINE = {"tensor": 0, "simt": 1}
ACT = {"linear": 0, "relu": 1, "relu6": 2, "hardswish": 3}


class IlluminaError(RuntimeError):
    """A non-OK status from the library, carrying illumina_last_error()."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class ModelOptions(C.Structure):
    _fields_ = [
        ("input_size", C.c_int), ("device", C.c_int), ("max_batch", C.c_int), ("precision", C.c_int),
        ("decode_srgb", C.c_int), ("exposure", C.c_float), ("range_sigma", C.c_float),
        ("temporal_base", C.c_float), ("temporal_sensitivity", C.c_float),
        ("keep_intermediates", C.c_int), ("weights", C.POINTER(C.c_float)), ("weights_count", C.c_size_t),
        ("idm_bytes", C.c_void_p), ("idm_len", C.c_size_t), ("idm_path", C.c_char_p),
        ("synth_seed", C.c_uint32), ("gemm_engine", C.c_int),
    ]


class Stats(C.Structure):
    _fields_ = [
        ("dispatches", C.c_int), ("launches", C.c_int), ("arena_bytes", C.c_size_t),
        ("naive_arena_bytes", C.c_size_t), ("weight_bytes", C.c_size_t), ("device_bytes", C.c_size_t),
        ("max_batch", C.c_int), ("precision", C.c_int), ("input_size", C.c_int), ("gemm_engine", C.c_int),
        ("device_error", C.c_int),
    ]


class SceneParamsC(C.Structure):
    _fields_ = [("camera", C.c_float * 4), ("focus", C.c_float * 4), ("options", C.c_float * 4)]


class DepthMetricsC(C.Structure):
    _fields_ = [("samples", C.c_longlong), ("abs_rel", C.c_double), ("rmse", C.c_double),
                ("delta1", C.c_double), ("delta2", C.c_double), ("delta3", C.c_double),
                ("scale", C.c_double), ("shift", C.c_double)]


class Light(C.Structure):
    _fields_ = [("position", C.c_float * 4), ("color", C.c_float * 4), ("direction", C.c_float * 4),
                ("params", C.c_float * 4)]


class ShadingSettingsC(C.Structure):
    _fields_ = [
        ("fov_y", C.c_float), ("near_m", C.c_float), ("far_m", C.c_float),
        ("ao_strength", C.c_float), ("shadow_strength", C.c_float), ("volumetric", C.c_float),
        ("exposure", C.c_float), ("ambient", C.c_float * 3), ("ambient_intensity", C.c_float),
        ("roughness", C.c_float), ("fog_density", C.c_float), ("fog_color", C.c_float * 3),
        ("specular", C.c_float), ("normal_strength", C.c_float), ("albedo_mix", C.c_float),
        ("contact_shadow_length", C.c_float), ("ao_radius_pixels", C.c_float), ("tone_map", C.c_int),
        ("contrast", C.c_float), ("saturation", C.c_float), ("vignette", C.c_float),
        ("debug_view", C.c_int),
    ]


class ShadeSteps(C.Structure):
    _fields_ = [("contact", C.c_int), ("ao_dirs", C.c_int), ("ao_steps", C.c_int), ("volumetric", C.c_int)]


_F = C.POINTER(C.c_float)
_V = C.c_void_p
_S = C.c_int  # status

SIGNATURES = {
    "illumina_last_error": (C.c_char_p, []),
    "illumina_version": (C.c_char_p, []),
    "illumina_device_count": (C.c_int, []),
    "illumina_arch_json": (_S, [C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "illumina_arena_json": (_S, [C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "illumina_weights_count": (_S, [C.c_int, C.POINTER(C.c_size_t)]),
    "illumina_weights_synthesize": (_S, [C.c_int, C.c_uint32, _V, C.c_size_t]),
    "illumina_weights_parse": (_S, [C.c_int, _V, C.c_size_t, _V, C.c_size_t]),
    "illumina_weights_serialize": (_S, [C.c_int, _V, C.c_size_t, _V, C.c_size_t, C.POINTER(C.c_size_t)]),
    "illumina_half_to_float": (C.c_double, [C.c_uint16]),
    "illumina_model_options_default": (None, [C.POINTER(ModelOptions)]),
    "illumina_model_create": (_S, [C.POINTER(ModelOptions), C.POINTER(C.c_void_p)]),
    "illumina_model_destroy": (_S, [_V]),
    "illumina_model_set_exposure": (_S, [_V, C.c_float]),
    "illumina_model_set_temporal": (_S, [_V, C.c_float, C.c_float, C.c_float]),
    "illumina_forward": (_S, [_V, _V, C.c_int, C.c_int, _V, _V, _V]),
    "illumina_model_record": (_S, [_V, _V, C.c_int, _V]),
    "illumina_forward_input": (_S, [_V, _V, C.c_int, _V, _V]),
    "illumina_forward_async": (_S, [_V, _V, C.c_int, C.c_int, _V, _V]),
    "illumina_forward_source_async": (_S, [_V, _V, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_float),
                                          C.POINTER(C.c_float), C.c_int, _V, _V]),
    "illumina_forward_source": (_S, [_V, _V, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_float),
                                    C.c_int, _V, _V]),
    "illumina_model_swap_history": (_S, [_V]),
    "illumina_model_sync": (_S, [_V]),
    "illumina_model_set_wait_limit": (_S, [_V, C.c_longlong]),
    "illumina_model_output_parity": (C.c_int, [_V]),
    "illumina_model_fresh_parity": (C.c_int, [_V]),
    "illumina_model_depth_slot": (_S, [_V, C.c_int, C.POINTER(C.c_void_p)]),
    "illumina_model_debug_tensor": (_S, [_V, C.c_char_p, _V, C.c_size_t, C.POINTER(C.c_int),
                                         C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "illumina_model_debug_tensor_frame": (_S, [_V, C.c_char_p, C.c_int, _V, C.c_size_t, C.POINTER(C.c_int),
                                               C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "illumina_model_stats": (_S, [_V, C.POINTER(Stats)]),
    "illumina_model_profile": (_S, [_V, _V, C.c_int, C.c_int, C.c_int, _V, C.c_int]),
    "illumina_set_op_engine": (_S, [C.c_int]),
    "illumina_op_pointwise": (_S, [_V, C.c_long, C.c_int, _V, _V, C.c_int, C.c_int, _V, _V, _V]),
    "illumina_op_dwpw": (_S, [_V, C.c_int, C.c_int, C.c_int, _V, _V, C.c_int, _V, _V, C.c_int, C.c_int,
                              C.c_int, C.c_int, _V, _V, _V]),
    "illumina_op_dwpw_noalloc": (_S, [_V, C.c_int, C.c_int, C.c_int, _V, _V, C.c_int, _V, _V, C.c_int,
                                      C.c_int, C.c_int, C.c_int, _V, _V, _V]),
    "illumina_selftest": (_S, [C.c_int, _V]),
    "illumina_op_conv": (_S, [_V, C.c_int, C.c_int, C.c_int, _V, _V, C.c_int, C.c_int, C.c_int, C.c_int,
                              _V, _V]),
    "illumina_op_lateral": (_S, [_V, C.c_int, C.c_int, _V, C.c_int, _V, _V, C.c_int, C.c_int, _V, _V]),
    "illumina_op_head": (_S, [_V, C.c_long, C.c_int, _V, C.c_float, _V, _V]),
    "illumina_op_preprocess": (_S, [_V, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _V, _V, _V]),
    "illumina_op_bilateral": (_S, [_V, C.c_int, C.c_int, C.c_int, _V, C.c_int, C.c_float, _V, _V]),
    "illumina_shading_settings_default": (None, [C.POINTER(ShadingSettingsC)]),
    "illumina_shade": (_S, [_V, C.c_int, C.c_int, C.c_int, _V, C.c_int, C.c_int, C.POINTER(Light),
                            C.POINTER(ShadingSettingsC), C.c_uint32, C.POINTER(ShadeSteps), C.c_int,
                            C.c_int, _V, _V, _V]),
    "illumina_resize_bilinear": (_S, [_V, C.c_int, C.c_int, _V, C.c_int, C.c_int, _V]),
    "illumina_sample_source": (_S, [_V, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_float),
                                     C.c_int, C.c_int, _V, _V]),
    "illumina_crop_transform": (None, [C.c_int, C.c_int, C.POINTER(C.c_float)]),
    "illumina_scene_params_initial": (None, [C.POINTER(SceneParamsC)]),
    "illumina_scene_params_update": (None, [C.POINTER(SceneParamsC), C.c_double, C.c_int]),
    "illumina_scene_render": (_S, [C.POINTER(SceneParamsC), C.c_int, C.c_int, C.c_int, _V, _V, _V, _V]),
    "illumina_evaluate_depth": (_S, [_V, C.c_int, _V, C.c_int, C.c_int, C.c_int, _V, _V]),
    "illumina_generate_frames": (_S, [C.c_int, C.c_uint32, C.c_int, C.c_int, _V, _V]),
    "illumina_checksums": (_S, [_V, C.c_int, C.c_long, _V, _V, _V]),
}

_lib = None


def lib() -> C.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libillumina.so not found at {LIB_PATH}; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` or `make -C ai-illumination-depth-model_b200/csrc`")
        handle = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int) -> None:
    if status != OK:
        raise IlluminaError(status, lib().illumina_last_error().decode("utf-8", "replace"))


def ptr(x) -> int | None:
    """Raw address of a numpy array or torch tensor (None passes through)."""
    if x is None:
        return None
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    if isinstance(x, int):
        return x
    raise TypeError(f"cannot take the address of {type(x).__name__}")


def stream_handle(stream) -> int | None:
    """cudaStream_t of a torch stream (or an int handle); None = legacy default stream."""
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream
