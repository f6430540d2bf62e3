"""Drop-in host layer for the reference renderer extension `PYOPTIXFLARERENDERER`.

`CPyOptiXFLARERenderer` keeps the reference class's constructor, its 12 methods and their positional
argument order (source/renderer/PyOptiXFLARERenderer.cpp:12-74, CPyOptiXFLARERenderer.h:14-327), and
`GenerateRays` keeps the module function (GenerateRays.cpp:6-28).  Tensors are passed as raw device
pointers to libflare_b200.so through the C ABI of include/flare_b200.h, on the current CUDA stream of
the renderer's device.  Outputs are filled in place exactly as the reference fills them: accumulated
into caller-zeroed buffers; `Backward` overwrites `I`; weight gradients land in row 0 of the
reference's per-warp fragment-layout buffers (train.py:704-790 sums the rows and un-permutes).

Differences from the reference, by design:
  * arguments are checked (CUDA, contiguous, dtype, shapes); violations raise ValueError instead of
    corrupting memory;
  * failures raise FlareError (a RuntimeError) carrying the library's message instead of `throw 0`;
  * the work runs on torch.cuda.current_stream() of the renderer's device without a host sync per
    pass beyond reading the active-ray count.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

F32, F16, I32 = torch.float32, torch.float16, torch.int32
PASS_SLOTS = 42  # FLARE_PASS_SLOTS: hit slots of an internal traversal pass
PRIM_ROW = 80    # FLARE_PRIM_ROW_FLOATS: floats of a per-primitive gradient row

# decoder kind -> (descriptor width, feature-table floats): 0 = the reference's LUT / sin-cos / 96-wide
# decoder, 1 = the dense-grid / spherical-harmonics / 32-wide variant (include/flare_b200.h)
DECODER_LUT_PE, DECODER_GRID_SH = 0, 1
DECODERS = {DECODER_LUT_PE: (96, 13154), DECODER_GRID_SH: (32, 16502)}


def decoder_kind(cond) -> int:
    """The decoder a descriptor tensor belongs to, from its width (96: LUT/PE, 32: grid/SH)."""
    w = cond.shape[1] if cond.dim() == 2 else -1
    for kind, (cdim, _) in DECODERS.items():
        if w == cdim:
            return kind
    raise ValueError(f"conditioning_variable: shape {tuple(cond.shape)}, expected (N, 96) or (N, 32)")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _need(t, name, dtype, shape=None, device=None):
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name}: expected a torch.Tensor, got {type(t).__name__}")
    if not t.is_cuda:
        raise ValueError(f"{name}: tensor must be on a CUDA device")
    if device is not None and t.device.index != device:
        raise ValueError(f"{name}: tensor on cuda:{t.device.index}, renderer on cuda:{device}")
    if t.dtype != dtype:
        raise ValueError(f"{name}: dtype {t.dtype}, expected {dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: tensor must be contiguous")
    if shape is not None:
        if t.dim() != len(shape) or any(s is not None and s != d for s, d in zip(shape, t.shape)):
            raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {shape}")
    return t


class CPyOptiXFLARERenderer:
    """B200 replacement of the reference `CPyOptiXFLARERenderer` (OptiX is replaced by an LBVH)."""

    def __init__(self, number_of_sides: int, chi_square_squared_radius: float, max_batch_size: int):
        self._lib = _lib.load()
        self.device = torch.cuda.current_device()
        self.number_of_sides = int(number_of_sides)
        self.max_batch_size = int(max_batch_size)
        h = ctypes.c_void_p()
        _lib.check(self._lib.flare_create(int(number_of_sides), float(chi_square_squared_radius), int(max_batch_size),
                                          self.device, ctypes.byref(h)), "CPyOptiXFLARERenderer")
        self._h = h
        self._n = 0

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                self._lib.flare_destroy(h)
            except Exception:
                pass
            self._h = None

    # -------------------------------------------------------------------------------------------
    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _scene(self, m, s, q, RGBA, kappa, dec=None):
        n = m.shape[0] if m.dim() == 2 else -1
        dv = self.device
        _need(m, "m", F32, (n, 3), dv)
        _need(s, "s", F32, (n, 2), dv)
        _need(q, "q", F32, (n, 4), dv)
        _need(RGBA, "RGBA", F32, (n, 4), dv)
        if kappa.numel() != n:
            raise ValueError(f"kappa: {kappa.numel()} elements, expected {n}")
        _need(kappa, "kappa", F32, None, dv)
        if n != self._n:
            raise ValueError(f"scene has {n} primitives but the last SetGeometry had {self._n}")
        sc = _lib.Scene(m=_ptr(m), s=_ptr(s), q=_ptr(q), RGBA=_ptr(RGBA), k=_ptr(kappa), n=n)
        if dec is not None:
            cond, feat, A1, b1, A2, b2, A3, b3 = dec
            kind = decoder_kind(cond)
            cdim, nfeat = DECODERS[kind]
            _need(cond, "conditioning_variable", F16, (n, cdim), dv)
            _need(feat, "features", F32, None, dv)
            if feat.numel() != nfeat:
                raise ValueError(f"features: {feat.numel()} elements, expected {nfeat} for a {cdim}-wide descriptor")
            sc.decoder = kind
            _need(A1, "A1", F16, (64, 128), dv)
            _need(A2, "A2", F16, (64, 64), dv)
            _need(A3, "A3", F16, (16, 64), dv)
            for t, nm, k in ((b1, "b1", 64), (b2, "b2", 64), (b3, "b3", 16)):
                _need(t, nm, F32, None, dv)
                if t.numel() != k:
                    raise ValueError(f"{nm}: {t.numel()} elements, expected {k}")
            sc.cond, sc.features = _ptr(cond), _ptr(feat)
            sc.A1, sc.A2, sc.A3 = _ptr(A1), _ptr(A2), _ptr(A3)
            sc.b1, sc.b2, sc.b3 = _ptr(b1), _ptr(b2), _ptr(b3)
        return sc

    def _rays(self, O, v):
        R = O.shape[0] if O.dim() == 2 else -1
        _need(O, "O", F32, (R, 3), self.device)
        _need(v, "v", F32, (R, 3), self.device)
        if R > self.max_batch_size:
            raise ValueError(f"{R} rays exceed max_batch_size {self.max_batch_size}")
        return R

    def _vec(self, t, name, R, w, dtype=F32):
        if w == 1:
            if t.numel() != R:
                raise ValueError(f"{name}: {t.numel()} elements, expected {R}")
            return _need(t, name, dtype, None, self.device)
        return _need(t, name, dtype, (R, w), self.device)

    def _forward(self, mode, sc, O, v, bitmap, bg, T_threshold, **kw):
        R = self._rays(O, v)
        a = _lib.ForwardArgs(mode=mode, O=_ptr(O), v=_ptr(v), n_rays=R, T_threshold=float(T_threshold))
        a.bg[0], a.bg[1], a.bg[2] = (float(x) for x in bg)
        if bitmap is not None:
            a.bitmap = _ptr(self._vec(bitmap, "bitmap", R, 3))
        for k_, (t, w) in kw.items():
            if t is None:
                continue
            if k_ in ("reg_a", "reg_b"):
                setattr(a, k_, float(t))
                continue
            setattr(a, k_, _ptr(self._vec(t, k_, R, w)) if k_ != "override_colors" else _ptr(t))
        _lib.check(self._lib.flare_forward(self._h, ctypes.byref(sc), ctypes.byref(a), self._stream()),
                   "forward")

    # ------------------------------------------------------------------------------ reference API
    def SetGeometry(self, m, s, q, opacity, kappa):
        """Sets the proxies from ACTIVATED parameters: m, exp(s), q, sigmoid(A), 1 + softplus(k)."""
        n = m.shape[0]
        dv = self.device
        _need(m, "m", F32, (n, 3), dv)
        _need(s, "scale", F32, (n, 2), dv)
        _need(q, "q", F32, (n, 4), dv)
        for t, nm in ((opacity, "opacity"), (kappa, "kappa")):
            _need(t, nm, F32, None, dv)
            if t.numel() != n:
                raise ValueError(f"{nm}: {t.numel()} elements, expected {n}")
        _lib.check(self._lib.flare_set_geometry(self._h, _ptr(m), _ptr(s), _ptr(q), _ptr(opacity), _ptr(kappa), n,
                                                self._stream()), "SetGeometry")
        self._n = n

    def Render(self, O, v, t_min, size):
        """16 nearest hits beyond t_min per ray: (t (16,size) f32, indices (16,size) i32)."""
        size = int(size)
        _need(O, "O", F32, None, self.device)
        _need(v, "v", F32, None, self.device)
        _need(t_min, "t_min", F32, None, self.device)
        if O.numel() < 3 * size or v.numel() < 3 * size or t_min.numel() < size:
            raise ValueError("Render: tensors smaller than size")
        t = torch.empty((16, size), dtype=F32, device=O.device)
        idx = torch.empty((16, size), dtype=I32, device=O.device)
        _lib.check(self._lib.flare_render_hits(self._h, _ptr(O), _ptr(v), _ptr(t_min), size, _ptr(t), _ptr(idx),
                                               self._stream()), "Render")
        return t, idx

    def GetMedianDepth_base(self, O, v, m, s, q, RGBA, kappa, T_threshold, depth_and_index):
        sc = self._scene(m, s, q, RGBA, kappa)
        self._forward(_lib.FWD_MEDIAN, sc, O, v, None, (0, 0, 0), T_threshold,
                      depth_and_index=(depth_and_index, 2))

    def Forward_training_base(self, O, v, bitmap, bg_color_R, bg_color_G, bg_color_B, m, s, q, RGBA, kappa,
                              T_threshold, depth_reg_accums, reg_a, reg_b, depth_and_index, surface_normal,
                              normal_reg_accums):
        sc = self._scene(m, s, q, RGBA, kappa)
        self._forward(_lib.FWD_TRAINING, sc, O, v, bitmap, (bg_color_R, bg_color_G, bg_color_B), T_threshold,
                      depth_reg_accums=(depth_reg_accums, 4), reg_a=(reg_a, 0), reg_b=(reg_b, 0),
                      surface_normal=(surface_normal, 3), normal_reg_accums=(normal_reg_accums, 4))

    def Forward_inference_base(self, O, v, bitmap, bg_color_R, bg_color_G, bg_color_B, m, s, q, RGBA, kappa,
                               T_threshold):
        sc = self._scene(m, s, q, RGBA, kappa)
        self._forward(_lib.FWD_INFERENCE, sc, O, v, bitmap, (bg_color_R, bg_color_G, bg_color_B), T_threshold)

    def Forward_inference_base_with_geometry(self, O, v, bitmap, normal, alpha, expected_depth_numerator, bg_color_R,
                                             bg_color_G, bg_color_B, m, s, q, RGBA, kappa, T_threshold):
        sc = self._scene(m, s, q, RGBA, kappa)
        self._forward(_lib.FWD_INFERENCE_GEOMETRY, sc, O, v, bitmap, (bg_color_R, bg_color_G, bg_color_B), T_threshold,
                      normal=(normal, 3), alpha=(alpha, 1), expected_depth_numerator=(expected_depth_numerator, 1))

    def Backward_base(self, O, v, bg_color_R, bg_color_G, bg_color_B, m, s, q, RGBA, kappa, I, dL_dI, dL_dRGB, dL_dA,
                      dL_d_kappa, dL_dm, dL_ds, dL_dq, T_threshold, depth_reg_accums, depth_normal_reg_prefix_sums,
                      lambda_depth, reg_a, reg_b, depth_and_index, surface_normal, normal_reg_accums, lambda_normal):
        sc = self._scene(m, s, q, RGBA, kappa)
        self._backward(sc, O, v, (bg_color_R, bg_color_G, bg_color_B), I, dL_dI, dL_dRGB, dL_dA, dL_d_kappa, dL_dm,
                       dL_ds, dL_dq, None, T_threshold, depth_reg_accums, depth_normal_reg_prefix_sums, lambda_depth,
                       reg_a, reg_b, surface_normal, lambda_normal)

    def GetMedianDepth(self, conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3, O, v, m, s, q, RGBA,
                       kappa, T_threshold, depth_and_index):
        sc = self._scene(m, s, q, RGBA, kappa, (conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3))
        self._forward(_lib.FWD_MEDIAN, sc, O, v, None, (0, 0, 0), T_threshold, depth_and_index=(depth_and_index, 2))

    def Forward_training(self, conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3, O, v, bitmap,
                         bg_color_R, bg_color_G, bg_color_B, m, s, q, RGBA, kappa, T_threshold, depth_reg_accums,
                         reg_a, reg_b, depth_and_index, surface_normal, normal_reg_accums):
        sc = self._scene(m, s, q, RGBA, kappa, (conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3))
        self._forward(_lib.FWD_TRAINING, sc, O, v, bitmap, (bg_color_R, bg_color_G, bg_color_B), T_threshold,
                      depth_reg_accums=(depth_reg_accums, 4), reg_a=(reg_a, 0), reg_b=(reg_b, 0),
                      surface_normal=(surface_normal, 3), normal_reg_accums=(normal_reg_accums, 4))

    def Forward_inference(self, conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3, O, v, bitmap,
                          bg_color_R, bg_color_G, bg_color_B, m, s, q, RGBA, kappa, T_threshold):
        sc = self._scene(m, s, q, RGBA, kappa, (conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3))
        self._forward(_lib.FWD_INFERENCE, sc, O, v, bitmap, (bg_color_R, bg_color_G, bg_color_B), T_threshold)

    def Forward_pca(self, conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3, override_colors, O, v,
                    bitmap, bg_color_R, bg_color_G, bg_color_B, m, s, q, RGBA, kappa, T_threshold):
        sc = self._scene(m, s, q, RGBA, kappa, (conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3))
        _need(override_colors, "override_colors", F32, (self._n, 3), self.device)
        self._forward(_lib.FWD_PCA, sc, O, v, bitmap, (bg_color_R, bg_color_G, bg_color_B), T_threshold,
                      override_colors=(override_colors, 3))

    def Forward_inference_with_geometry(self, conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3, O,
                                        v, bitmap, normal, alpha, expected_depth_numerator, bg_color_R, bg_color_G,
                                        bg_color_B, m, s, q, RGBA, kappa, T_threshold):
        sc = self._scene(m, s, q, RGBA, kappa, (conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3))
        self._forward(_lib.FWD_INFERENCE_GEOMETRY, sc, O, v, bitmap, (bg_color_R, bg_color_G, bg_color_B), T_threshold,
                      normal=(normal, 3), alpha=(alpha, 1), expected_depth_numerator=(expected_depth_numerator, 1))

    def Backward(self, conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3, O, v, bg_color_R,
                 bg_color_G, bg_color_B, m, s, q, RGBA, kappa, I, dL_dI, dL_dRGB, dL_dA, dL_d_kappa, dL_dw3, dL_db3,
                 dL_dw2, dL_db2, dL_dw1, dL_db1, dL_d_conditioning, dL_d_deatures, dL_dm, dL_ds, dL_dq, T_threshold,
                 depth_reg_accums, depth_normal_reg_prefix_sums, lambda_depth, reg_a, reg_b, depth_and_index,
                 surface_normal, normal_reg_accums, lambda_normal, prim_rows=None):
        """prim_rows (extension, keyword only): a caller-zeroed (N, 80) f32 tensor that receives the
        per-primitive gradient rows instead of dL_dRGB .. dL_dq and dL_d_conditioning (see
        scatter_prim_rows), for data-parallel callers that sum the rows over ranks."""
        sc = self._scene(m, s, q, RGBA, kappa, (conditioning_variable, features_P_hit_object, A1, b1, A2, b2, A3, b3))
        dec = (dL_dw3, dL_db3, dL_dw2, dL_db2, dL_dw1, dL_db1, dL_d_conditioning, dL_d_deatures)
        self._backward(sc, O, v, (bg_color_R, bg_color_G, bg_color_B), I, dL_dI, dL_dRGB, dL_dA, dL_d_kappa, dL_dm,
                       dL_ds, dL_dq, dec, T_threshold, depth_reg_accums, depth_normal_reg_prefix_sums, lambda_depth,
                       reg_a, reg_b, surface_normal, lambda_normal, prim_rows)

    def _backward(self, sc, O, v, bg, I, dL_dI, dL_dRGB, dL_dA, dL_dk, dL_dm, dL_ds, dL_dq, dec, T_threshold,
                  depth_reg_accums, prefix, lambda_depth, reg_a, reg_b, surface_normal, lambda_normal, prim_rows=None):
        R = self._rays(O, v)
        n, dv = self._n, self.device
        a = _lib.BackwardArgs(O=_ptr(O), v=_ptr(v), n_rays=R, T_threshold=float(T_threshold),
                              I=_ptr(self._vec(I, "I", R, 3)), dL_dI=_ptr(self._vec(dL_dI, "dL_dI", R, 3)),
                              lambda_depth=float(lambda_depth), reg_a=float(reg_a), reg_b=float(reg_b),
                              lambda_normal=float(lambda_normal))
        a.bg[0], a.bg[1], a.bg[2] = (float(x) for x in bg)
        for t, nm, w in ((dL_dRGB, "dL_dRGB", 3), (dL_dA, "dL_dA", 1), (dL_dk, "dL_d_kappa", 1), (dL_dm, "dL_dm", 3),
                         (dL_ds, "dL_ds", 2), (dL_dq, "dL_dq", 4)):
            _need(t, nm, F32, None, dv)
            if t.numel() != n * w:
                raise ValueError(f"{nm}: {t.numel()} elements, expected {n * w}")
        a.dL_dRGB, a.dL_dA, a.dL_dk = _ptr(dL_dRGB), _ptr(dL_dA), _ptr(dL_dk)
        a.dL_dm, a.dL_ds, a.dL_dq = _ptr(dL_dm), _ptr(dL_ds), _ptr(dL_dq)
        a.depth_reg_accums = _ptr(self._vec(depth_reg_accums, "depth_reg_accums", R, 4))
        a.depth_normal_reg_prefix_sums = _ptr(self._vec(prefix, "depth_normal_reg_prefix_sums", R, 4))
        a.surface_normal = _ptr(self._vec(surface_normal, "surface_normal", R, 3))
        if dec is not None:
            dw3, db3, dw2, db2, dw1, db1, dcond, dfeat = dec
            for t, nm, w in ((dw3, "dL_dw3", 512), (db3, "dL_db3", 64), (dw2, "dL_dw2", 4096), (db2, "dL_db2", 512),
                             (dw1, "dL_dw1", 8192), (db1, "dL_db1", 512)):
                _need(t, nm, F32, None, dv)
                if t.dim() != 2 or t.shape[1] != w or t.shape[0] < 1:
                    raise ValueError(f"{nm}: shape {tuple(t.shape)}, expected (rows, {w})")
            cdim, nfeat = DECODERS[sc.decoder]
            _need(dcond, "dL_d_conditioning", F32, (n, cdim), dv)
            _need(dfeat, "dL_d_features", F32, None, dv)
            if dfeat.numel() != nfeat:
                raise ValueError(f"dL_d_features: expected {nfeat} elements")
            a.dL_dw1, a.dL_db1, a.dL_dw2, a.dL_db2 = _ptr(dw1), _ptr(db1), _ptr(dw2), _ptr(db2)
            a.dL_dw3, a.dL_db3, a.dL_dcond, a.dL_dfeatures = _ptr(dw3), _ptr(db3), _ptr(dcond), _ptr(dfeat)
            if prim_rows is not None:
                _need(prim_rows, "prim_rows", F32, (n, PRIM_ROW), dv)
                a.prim_rows = _ptr(prim_rows)
        _lib.check(self._lib.flare_backward(self._h, ctypes.byref(sc), ctypes.byref(a), self._stream()), "Backward")

    # ------------------------------------------------------------------------------ extras
    def stats(self):
        st = _lib.Stats()
        _lib.check(self._lib.flare_get_stats(self._h, ctypes.byref(st)), "stats")
        return {k: getattr(st, k) for k, _ in _lib.Stats._fields_}

    def profile(self, enable: bool = True):
        """Enables (and zeroes) or disables per-kernel CUDA-event timing."""
        _lib.check(self._lib.flare_profile(self._h, 1 if enable else 0), "profile")

    def kernel_times(self):
        """{kernel: (total ms, launches)} accumulated since profile(True)."""
        kt = _lib.KernelTimes()
        _lib.check(self._lib.flare_get_kernel_times(self._h, ctypes.byref(kt)), "kernel_times")
        return {n: (kt.ms[i], kt.launches[i]) for i, n in enumerate(_lib.KERNEL_NAMES)}

    def pass_hits(self):
        """The traversal passes of the last Forward_training (valid from the second call on this
        renderer): a list of (ray_ids (count,), t (42, count), idx (42, count)) device tensors."""
        cnt = ctypes.c_int(0)
        _lib.check(self._lib.flare_get_pass_hits(self._h, -1, ctypes.byref(cnt), None, None, None, self._stream()),
                   "pass_hits")
        out = []
        dev = f"cuda:{self.device}"
        for p in range(cnt.value):
            c = ctypes.c_int(0)
            _lib.check(self._lib.flare_get_pass_hits(self._h, p, ctypes.byref(c), None, None, None, self._stream()),
                       "pass_hits")
            ids = torch.empty(c.value, dtype=torch.int32, device=dev)
            t = torch.empty((PASS_SLOTS, c.value), dtype=F32, device=dev)
            idx = torch.empty((PASS_SLOTS, c.value), dtype=torch.int32, device=dev)
            _lib.check(self._lib.flare_get_pass_hits(self._h, p, ctypes.byref(c), _ptr(ids), _ptr(t), _ptr(idx),
                                                     self._stream()), "pass_hits")
            out.append((ids, t, idx))
        return out

    def frames(self):
        """Per-primitive proxy frames (N,12) of the last SetGeometry (used by the hit-list parity test)."""
        out = torch.empty((self._n, 12), dtype=F32, device=f"cuda:{self.device}")
        _lib.check(self._lib.flare_get_frames(self._h, _ptr(out), self._stream()), "frames")
        return out


def scatter_prim_rows(rows, A1, decoder, dL_dRGB, dL_dA, dL_dk, dL_dm, dL_ds, dL_dq, dL_d_conditioning):
    """Adds per-primitive gradient rows (N, 80) -- from Backward(..., prim_rows=...), possibly summed over
    data-parallel ranks -- into the per-primitive gradients (flare_scatter_prim_rows)."""
    lib = _lib.load()
    n = rows.shape[0]
    dv = rows.device.index
    _need(rows, "rows", F32, (n, PRIM_ROW), dv)
    _need(A1, "A1", F16, (64, 128), dv)
    cdim, _ = DECODERS[int(decoder)]
    for t, nm, w in ((dL_dRGB, "dL_dRGB", 3), (dL_dA, "dL_dA", 1), (dL_dk, "dL_d_kappa", 1), (dL_dm, "dL_dm", 3),
                     (dL_ds, "dL_ds", 2), (dL_dq, "dL_dq", 4), (dL_d_conditioning, "dL_d_conditioning", cdim)):
        _need(t, nm, F32, None, dv)
        if t.numel() != n * w:
            raise ValueError(f"{nm}: {t.numel()} elements, expected {n * w}")
    stream = ctypes.c_void_p(torch.cuda.current_stream(rows.device).cuda_stream)
    _lib.check(lib.flare_scatter_prim_rows(_ptr(rows), n, _ptr(A1), int(decoder), _ptr(dL_dRGB), _ptr(dL_dA),
                                           _ptr(dL_dk), _ptr(dL_dm), _ptr(dL_ds), _ptr(dL_dq),
                                           _ptr(dL_d_conditioning), stream), "scatter_prim_rows")


def GenerateRays(R, D, F, width, height, fov_X, fov_Y):
    """Pinhole ray directions (height, width, 3), not normalised (reference GenerateRays.cpp:6-28)."""
    lib = _lib.load()
    dev = R.device
    for t, nm in ((R, "R"), (D, "D"), (F, "F")):
        _need(t, nm, F32, None, dev.index)
        if t.numel() < 3:
            raise ValueError(f"{nm}: needs 3 elements")
    out = torch.empty((int(height), int(width), 3), dtype=F32, device=dev)
    _lib.check(lib.flare_generate_rays(_ptr(R), _ptr(D), _ptr(F), int(width), int(height), float(fov_X), float(fov_Y),
                                       _ptr(out), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)),
               "GenerateRays")
    return out


def selftest_mlp(X, A1, b1, A2, b2, A3, b3):
    """Runs the tensor-core decoder tile on rows X (rows,128) f16 -> (rows,16) f32 (outputs 0..3 set)."""
    lib = _lib.load()
    Y = torch.empty((X.shape[0], 16), dtype=F32, device=X.device)
    _lib.check(lib.flare_selftest_mlp(_ptr(X), X.shape[0], _ptr(A1), _ptr(b1), _ptr(A2), _ptr(b2), _ptr(A3), _ptr(b3),
                                      _ptr(Y), ctypes.c_void_p(torch.cuda.current_stream(X.device).cuda_stream)),
               "selftest_mlp")
    return Y
