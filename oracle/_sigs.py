"""ctypes signatures for liboracle.so (test infrastructure only)."""
import ctypes as C

F = C.POINTER(C.c_float)
D = C.POINTER(C.c_double)
L = C.POINTER(C.c_long)
I = C.POINTER(C.c_int)
U8 = C.POINTER(C.c_uint8)


class Light(C.Structure):
    _fields_ = [("position", C.c_float * 4), ("color", C.c_float * 4),
                ("direction", C.c_float * 4), ("params", C.c_float * 4)]


class ShadeParams(C.Structure):
    _fields_ = [(n, C.c_float * 4) for n in
                ("camera", "toggles", "ambient", "misc", "fog", "size", "debug", "grade")]


class Steps(C.Structure):
    _fields_ = [("contact_steps", C.c_int), ("ao_dirs", C.c_int), ("ao_steps", C.c_int),
                ("vol_steps", C.c_int)]


def declare(lib):
    sig = {
        "or_activation": (C.c_double, [C.c_int, C.c_double]),
        "or_out_extent": (C.c_int, [C.c_int, C.c_int, C.c_int]),
        "or_pointwise": (None, [F, C.c_long, C.c_int, F, F, C.c_int, C.c_int, F, F]),
        "or_conv": (None, [F, C.c_int, C.c_int, C.c_int, F, F, C.c_int, C.c_int, C.c_int, C.c_int, F]),
        "or_depthwise": (None, [F, C.c_int, C.c_int, C.c_int, F, F, C.c_int, C.c_int, C.c_int, F]),
        "or_dwpw": (C.c_int, [F, C.c_int, C.c_int, C.c_int, F, F, C.c_int, F, F, C.c_int, C.c_int,
                              C.c_int, C.c_int, F, F]),
        "or_upsample2": (None, [F, C.c_int, C.c_int, C.c_int, F]),
        "or_lateral": (C.c_int, [F, C.c_int, C.c_int, C.c_int, F, C.c_int, C.c_int, C.c_int, F, F,
                                 C.c_int, C.c_int, F]),
        "or_head": (None, [F, C.c_long, C.c_int, F, C.c_float, F]),
        "or_head_logit": (None, [F, C.c_long, C.c_int, F, C.c_float, D]),
        "or_preprocess": (None, [F, C.c_int, D, D, C.c_int, C.c_double, F, F]),
        "or_bilateral": (None, [F, C.c_int, C.c_int, C.c_int, F, C.c_int, C.c_int, C.c_double, F]),
        "or_mulberry32": (None, [C.c_uint32, C.c_long, D]),
        "or_synthesize": (None, [C.c_uint32, C.c_int, L, L, I, I, F]),
        "or_random_floats": (C.c_uint32, [C.c_uint32, C.c_long, C.c_double, F]),
        "or_uniform_frame": (None, [C.c_uint32, C.c_long, F]),
        "or_half_to_float": (C.c_double, [C.c_uint32]),
        "or_ggx_d": (C.c_float, [C.c_float, C.c_float]),
        "or_smith_g": (C.c_float, [C.c_float, C.c_float, C.c_float]),
        "or_composite_px": (None, [F, F, C.c_float, C.c_float, F]),
        "or_shade": (None, [F, C.c_int, C.c_int, F, C.c_int, C.c_int, C.POINTER(Light), C.c_int,
                            C.POINTER(ShadeParams), C.POINTER(Steps), C.c_int, C.c_int, C.c_int,
                            C.c_int, F, U8]),
        "or_sample_source": (None, [U8, C.c_int, C.c_int, C.c_int, F, F, C.c_int, C.c_int, F]),
        "or_crop_transform": (None, [C.c_int, C.c_int, F]),
        "or_scene_params": (None, [C.c_double, C.c_int, C.c_int, F]),
        "or_scene_render": (None, [F, C.c_int, C.c_int, F, U8, F]),
        "or_evaluate_depth": (None, [F, C.c_int, F, C.c_int, C.c_int, D]),
        "or_resize_bilinear": (None, [F, C.c_int, C.c_int, F, C.c_int, C.c_int]),
        "or_blob_frame": (None, [C.c_uint32, C.c_int, F]),
        "or_det_exp": (C.c_double, [C.c_double]),
        "or_det_log": (C.c_double, [C.c_double]),
        "or_det_cos2pi": (C.c_double, [C.c_double]),
        "or_det_sincos": (None, [C.c_double, D, D]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
