"""CPU tests of the C-ABI boundary: the library loads, exports every declared entry point, and
rejects bad arguments with a message (no compute call needs a GPU here)."""
import ctypes
import os
import re

import pytest
import torch

from flare_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flare_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(flare_[a-z_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.EXPORTS), "ctypes table and header disagree"


def test_version_and_error_string():
    lib = _lib.load()
    assert b"sm_100a" in lib.flare_version()
    assert isinstance(lib.flare_last_error(), bytes)


def test_create_rejects_bad_arguments_without_gpu():
    lib = _lib.load()
    h = ctypes.c_void_p()
    assert lib.flare_create(2, 11.3449, 16, 0, ctypes.byref(h)) == 1
    assert b"number_of_sides" in lib.flare_last_error()
    assert lib.flare_create(8, 11.3449, -1, 0, ctypes.byref(h)) == 1
    assert lib.flare_destroy(None) == 0


def test_null_arguments_are_rejected():
    lib = _lib.load()
    assert lib.flare_set_geometry(None, None, None, None, None, None, 0, None) == 1
    assert lib.flare_generate_rays(None, None, None, 4, 4, 1.0, 1.0, None, None) == 1
    assert b"NULL" in lib.flare_last_error()


def test_host_layer_validates_tensors():
    from flare_b200.renderer import GenerateRays
    with pytest.raises(ValueError):
        GenerateRays(torch.zeros(3), torch.zeros(3), torch.zeros(3), 4, 4, 1.0, 1.0)


def test_drop_in_module_names():
    import importlib.util
    p = os.path.join(ROOT, "flare_b200", "compat", "PYOPTIXFLARERENDERER.py")
    spec = importlib.util.spec_from_file_location("PYOPTIXFLARERENDERER", p)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    cls = mod.CPyOptiXFLARERenderer
    for name in ["SetGeometry", "Render", "GetMedianDepth_base", "Forward_training_base", "Forward_inference_base",
                 "Forward_inference_base_with_geometry", "Backward_base", "GetMedianDepth", "Forward_training",
                 "Forward_inference", "Forward_pca", "Forward_inference_with_geometry", "Backward"]:
        assert callable(getattr(cls, name)), name
    assert callable(mod.GenerateRays)
