"""ctypes binding of the C ABI in include/flare_b200.h (libflare_b200.so, built in-tree).

The library is required: importing the renderer without it raises, there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libflare_b200.so")

c_float_p = ctypes.POINTER(ctypes.c_float)
c_int_p = ctypes.POINTER(ctypes.c_int)
vp = ctypes.c_void_p

FWD_TRAINING, FWD_INFERENCE, FWD_INFERENCE_GEOMETRY, FWD_PCA, FWD_MEDIAN = range(5)


class Scene(ctypes.Structure):
    _fields_ = [("m", vp), ("s", vp), ("q", vp), ("RGBA", vp), ("k", vp), ("n", ctypes.c_int),
                ("cond", vp), ("features", vp), ("A1", vp), ("A2", vp), ("A3", vp),
                ("b1", vp), ("b2", vp), ("b3", vp), ("decoder", ctypes.c_int)]


class ForwardArgs(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_int), ("O", vp), ("v", vp), ("n_rays", ctypes.c_int),
                ("bg", ctypes.c_float * 3), ("T_threshold", ctypes.c_float), ("bitmap", vp),
                ("depth_reg_accums", vp), ("reg_a", ctypes.c_float), ("reg_b", ctypes.c_float),
                ("depth_and_index", vp), ("surface_normal", vp), ("normal_reg_accums", vp),
                ("normal", vp), ("alpha", vp), ("expected_depth_numerator", vp), ("override_colors", vp)]


class BackwardArgs(ctypes.Structure):
    _fields_ = [("O", vp), ("v", vp), ("n_rays", ctypes.c_int), ("bg", ctypes.c_float * 3),
                ("T_threshold", ctypes.c_float), ("I", vp), ("dL_dI", vp),
                ("dL_dRGB", vp), ("dL_dA", vp), ("dL_dk", vp), ("dL_dm", vp), ("dL_ds", vp), ("dL_dq", vp),
                ("dL_dcond", vp), ("dL_dfeatures", vp),
                ("dL_dw1", vp), ("dL_db1", vp), ("dL_dw2", vp), ("dL_db2", vp), ("dL_dw3", vp), ("dL_db3", vp),
                ("depth_reg_accums", vp), ("depth_normal_reg_prefix_sums", vp), ("lambda_depth", ctypes.c_float),
                ("reg_a", ctypes.c_float), ("reg_b", ctypes.c_float), ("surface_normal", vp),
                ("lambda_normal", ctypes.c_float), ("prim_rows", vp)]


class ViewerArgs(ctypes.Structure):
    _fields_ = [("O", vp), ("v", vp), ("bitmap", vp), ("n_rays", ctypes.c_int), ("bg", ctypes.c_float * 3),
                ("T_threshold", ctypes.c_float), ("spheres", vp), ("materials", vp), ("n_spheres", ctypes.c_int),
                ("lights", vp), ("n_lights", ctypes.c_int), ("epsilon", ctypes.c_float),
                ("shadow_multiplier", ctypes.c_float), ("ambient", ctypes.c_float * 3),
                ("max_recursion_depth", ctypes.c_int)]


VIEWER_MAX_SPHERES, VIEWER_MAX_LIGHTS = 16, 8
ADAM_MAX_SEGMENTS = 24


class AdamSegment(ctypes.Structure):
    _fields_ = [("param", vp), ("grad", vp), ("exp_avg", vp), ("exp_avg_sq", vp), ("param_f16", vp),
                ("rows", ctypes.c_longlong), ("width", ctypes.c_int), ("p_stride", ctypes.c_int),
                ("p_offset", ctypes.c_int), ("lr", ctypes.c_float), ("scale_reg", ctypes.c_float)]


class AdamArgs(ctypes.Structure):
    _fields_ = [("n_segments", ctypes.c_int), ("seg", AdamSegment * ADAM_MAX_SEGMENTS), ("beta1", ctypes.c_float),
                ("beta2", ctypes.c_float), ("eps", ctypes.c_float), ("step", ctypes.c_int)]


GATHER_MAX_TENSORS = 32


class GatherTensor(ctypes.Structure):
    _fields_ = [("src", vp), ("src_alt", vp), ("dst", vp), ("row_bytes", ctypes.c_int)]


class Stats(ctypes.Structure):
    _fields_ = [("rays", ctypes.c_longlong), ("passes", ctypes.c_longlong), ("hits_composited", ctypes.c_longlong),
                ("prim_tests", ctypes.c_longlong), ("node_visits", ctypes.c_longlong),
                ("decoder_tiles", ctypes.c_longlong)]


class KernelTimes(ctypes.Structure):
    _fields_ = [("ms", ctypes.c_double * 4), ("launches", ctypes.c_longlong * 4)]


KERNEL_NAMES = ("build", "trace", "shade_forward", "shade_backward")

# every entry point declared in include/flare_b200.h
EXPORTS = {
    "flare_last_error": (ctypes.c_char_p, []),
    "flare_version": (ctypes.c_char_p, []),
    "flare_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.POINTER(vp)]),
    "flare_destroy": (ctypes.c_int, [vp]),
    "flare_set_geometry": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, ctypes.c_int, vp]),
    "flare_render_hits": (ctypes.c_int, [vp, vp, vp, vp, ctypes.c_int, vp, vp, vp]),
    "flare_generate_rays": (ctypes.c_int, [vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float, vp,
                                           vp]),
    "flare_forward": (ctypes.c_int, [vp, ctypes.POINTER(Scene), ctypes.POINTER(ForwardArgs), vp]),
    "flare_backward": (ctypes.c_int, [vp, ctypes.POINTER(Scene), ctypes.POINTER(BackwardArgs), vp]),
    "flare_viewer_forward": (ctypes.c_int, [vp, ctypes.POINTER(Scene), ctypes.POINTER(ViewerArgs), vp]),
    "flare_adam_step": (ctypes.c_int, [ctypes.POINTER(AdamArgs), vp]),
    "flare_gather_rows": (ctypes.c_int, [ctypes.POINTER(GatherTensor), ctypes.c_int, vp, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, vp]),
    "flare_get_stats": (ctypes.c_int, [vp, ctypes.POINTER(Stats)]),
    "flare_get_frames": (ctypes.c_int, [vp, vp, vp]),
    "flare_scatter_prim_rows": (ctypes.c_int, [vp, ctypes.c_int, vp, ctypes.c_int] + [vp] * 8),
    "flare_get_pass_hits": (ctypes.c_int, [vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int), vp, vp, vp, vp]),
    "flare_profile": (ctypes.c_int, [vp, ctypes.c_int]),
    "flare_get_kernel_times": (ctypes.c_int, [vp, ctypes.POINTER(KernelTimes)]),
    "flare_selftest_mlp": (ctypes.c_int, [vp, ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp]),
    "flare_render_hits_noalloc": (ctypes.c_int, [ctypes.c_int, vp, vp, vp, vp, vp, ctypes.c_int, vp, vp, vp,
                                                 ctypes.c_int, vp, vp, vp]),
}

_lib = None


def load(path: str = None):
    """Loads libflare_b200.so (or the file named by $FLARE_B200_LIB) and declares every exported
    signature.  Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("FLARE_B200_LIB") or LIB_PATH
    if not os.path.exists(path):
        raise RuntimeError(f"flare_b200: native library not found at {path}; run `python -m flare_b200.build`")
    lib = ctypes.CDLL(path)
    for name, (res, args) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class FlareError(RuntimeError):
    pass


def check(code: int, what: str = ""):
    if code != 0:
        msg = _lib.flare_last_error().decode(errors="replace") if _lib is not None else ""
        raise FlareError(f"{what} failed (code {code}): {msg}")
