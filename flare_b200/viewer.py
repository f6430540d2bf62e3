"""Secondary-ray renderer: the reference viewer's recursive forward (reflection, refraction, shadows) with
analytic spheres in place of its triangle meshes.

Mirrors `CPyOptiXFLAREVIEWERRenderer` (source/viewer_renderer/CPyOptiXFLAREVIEWERRenderer.h:12-64):
the constructor takes the same four arguments; `SetGeometry` takes the activated primitive tensors and,
instead of mesh instances / hitgroup records, a (S,4) tensor of spheres (centre, radius); `Forward`
takes the reference's arguments minus the mesh normal matrices (`M4N`), which spheres do not need.
Materials are the reference's rows (Id rgb, kd, eta, n) and lights its rows (Is rgb, direction L).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .renderer import F32, CPyOptiXFLARERenderer, _need, _ptr


def _host_table(t, name, width, max_rows):
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name}: expected a torch.Tensor")
    if t.dim() != 2 or t.shape[1] != width:
        raise ValueError(f"{name}: shape {tuple(t.shape)}, expected (rows, {width})")
    if t.shape[0] > max_rows:
        raise ValueError(f"{name}: {t.shape[0]} rows, at most {max_rows}")
    return t.detach().to("cpu", torch.float32).contiguous()


class CPyFlareViewerRenderer(CPyOptiXFLARERenderer):
    """B200 replacement of the reference viewer renderer (spheres instead of meshes)."""

    def __init__(self, number_of_sides: int, chi_square_squared_radius: float, max_batch_size: int,
                 max_recursion_depth: int):
        super().__init__(number_of_sides, chi_square_squared_radius, max_batch_size)
        if not 0 <= int(max_recursion_depth) <= 64:
            raise ValueError(f"max_recursion_depth {max_recursion_depth} not in [0, 64]")
        self.max_recursion_depth = int(max_recursion_depth)
        self._spheres = torch.zeros(0, 4)

    def SetGeometry(self, m, s, q, opacity, kappa, spheres=None):
        super().SetGeometry(m, s, q, opacity, kappa)
        self._spheres = (_host_table(spheres, "spheres", 4, _lib.VIEWER_MAX_SPHERES) if spheres is not None
                         else torch.zeros(0, 4))

    def Forward(self, conditioning_variable, features_P_hit_object, RGB, A1, b1, A2, b2, A3, b3, O, v, bitmap,
                bg_color_R, bg_color_G, bg_color_B, m, s, q, A, kappa, T_threshold, materials, lights, epsilon,
                shadow_multiplier, Ia_R, Ia_G, Ia_B):
        n = m.shape[0]
        _need(RGB, "RGB", F32, (n, 3), self.device)
        if A.numel() != n:
            raise ValueError(f"A: {A.numel()} elements, expected {n}")
        RGBA = torch.cat([RGB, A.reshape(n, 1).to(torch.float32)], 1).contiguous()
        sc = self._scene(m, s, q, RGBA, kappa, (conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3))
        R = self._rays(O, v)
        mats = _host_table(materials, "materials", 6, _lib.VIEWER_MAX_SPHERES)
        if mats.shape[0] < self._spheres.shape[0]:
            raise ValueError(f"materials: {mats.shape[0]} rows for {self._spheres.shape[0]} spheres")
        lts = _host_table(lights, "lights", 6, _lib.VIEWER_MAX_LIGHTS)
        a = _lib.ViewerArgs(O=_ptr(O), v=_ptr(v), bitmap=_ptr(self._vec(bitmap, "bitmap", R, 3)), n_rays=R,
                            T_threshold=float(T_threshold), n_spheres=int(self._spheres.shape[0]),
                            n_lights=int(lts.shape[0]), epsilon=float(epsilon),
                            shadow_multiplier=float(shadow_multiplier), max_recursion_depth=self.max_recursion_depth)
        a.bg[0], a.bg[1], a.bg[2] = float(bg_color_R), float(bg_color_G), float(bg_color_B)
        a.ambient[0], a.ambient[1], a.ambient[2] = float(Ia_R), float(Ia_G), float(Ia_B)
        a.spheres = ctypes.c_void_p(self._spheres.data_ptr()) if self._spheres.numel() else None
        a.materials = ctypes.c_void_p(mats.data_ptr()) if mats.numel() else None
        a.lights = ctypes.c_void_p(lts.data_ptr()) if lts.numel() else None
        _lib.check(self._lib.flare_viewer_forward(self._h, ctypes.byref(sc), ctypes.byref(a), self._stream()),
                   "Forward")
