"""The reference renderer's own CUDA kernels, driven pass by pass (test infrastructure only).

oracle/Makefile.ref compiles the reference's decode / composite / backward kernels from its sources
(source/renderer/CPyOptiXFLARERenderer_CUDA_{Forward_training,Forward_inference,GetMedianDepth,Backward}
.cu and their _base twins) into oracle/_ref/libref_*.so; oracle/ref_kernels.cu exports one launcher per
library.  This module restates the reference's host pass loop around them
(CPyOptiXFLARERenderer_CUDA_Forward_training.cu:1004-1131 and the same loop in every method):

    t_min <- 0, T <- 1, ray_indices <- 0..R-1
    while R_active > 0:
        hits of the active rays            (the reference: optixLaunch of shaders.cu:81-189)
        kernel(..., ray_indices, t_hit, indices_hit, t_min, T, is_active, ...)
        ray_indices <- ray_indices[is_active]   (thrust exclusive_scan + scatter_if + reduce)

The OptiX traversal is the one piece that cannot run here (closed SDK, RT cores).  Its per-pass
16-nearest hit lists come from the CPU oracle's CSR hit lists (oracle.hit_lists), whose pass p of ray r
is entries [16p, 16p+16) of that ray's list -- the reference's restart semantics (t_min =
nextafter(t_16)).  Everything after the traversal -- frames, LUT, positional encoding, the mma.sync MLP,
compositing, regularisers, the backward and its per-warp weight-gradient layout -- is the reference's
own compiled code.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
KINDS = ("fwd_training", "fwd_inference", "median", "backward", "fwd_training_base", "fwd_inference_base",
         "median_base", "backward_base")
REF_DIR = "/root/reference/source/renderer"
K = 16


def build():
    """Compiles the libraries when the reference sources are present (this container only)."""
    if not os.path.isdir(REF_DIR):
        return False
    import subprocess
    subprocess.run(["make", "-s", "-j8", "-f", os.path.join(HERE, "Makefile.ref")], check=True)
    return True


def available():
    return all(os.path.exists(os.path.join(OUT, f"libref_{k}.so")) for k in KINDS)


class _F3(ctypes.Structure):
    _fields_ = [("x", ctypes.c_float), ("y", ctypes.c_float), ("z", ctypes.c_float)]


_LIBS = {}


def _lib(kind):
    if kind not in _LIBS:
        lib = ctypes.CDLL(os.path.join(OUT, f"libref_{kind}.so"))
        lib.ref_launch.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        lib.ref_launch.restype = ctypes.c_int
        _LIBS[kind] = lib
    return _LIBS[kind]


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _launch(kind, vals, n):
    """vals: the kernel's parameters in order (tensors -> device pointers, python float -> f32, int -> i32,
    3-tuples -> float3)."""
    keep = []
    for v in vals:
        if v is None or torch.is_tensor(v):
            keep.append(_ptr(v))
        elif isinstance(v, tuple):
            keep.append(_F3(*[float(x) for x in v]))
        elif isinstance(v, int):
            keep.append(ctypes.c_int(v))
        else:
            keep.append(ctypes.c_float(float(v)))
    arr = (ctypes.c_void_p * len(keep))(*[ctypes.cast(ctypes.pointer(x), ctypes.c_void_p) for x in keep])
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    rc = _lib(kind).ref_launch(arr, n, sms, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc != 0:
        raise RuntimeError(f"reference kernel {kind}: CUDA error {rc}")


class RefRenderer:
    """Runs the reference kernels over a scene (device tensors in the reference layouts) and the oracle's
    CSR hit lists of its rays."""

    def __init__(self, scene, O, v, csr):
        self.g = scene
        self.O = O.contiguous()
        self.v = v.contiguous()
        self.R = O.shape[0]
        off, tt, ii = csr
        self.off = np.asarray(off, np.int64)
        self.tt = np.asarray(tt, np.float32)
        self.ii = np.asarray(ii, np.int32)
        self.passes = 0

    def _pass_hits(self, rays, p):
        """(16, n) slot-major t / index of pass p of the given rays, padded with (inf, -1)."""
        n = len(rays)
        t = np.full((K, n), np.inf, np.float32)
        idx = np.full((K, n), -1, np.int32)
        start = self.off[rays] + K * p
        cnt = np.clip(self.off[rays + 1] - start, 0, K)
        for k in range(K):
            has = cnt > k
            t[k, has] = self.tt[start[has] + k]
            idx[k, has] = self.ii[start[has] + k]
        return torch.from_numpy(t).cuda(), torch.from_numpy(idx).cuda()

    def _loop(self, kind, make_args):
        dev = self.O.device
        R = self.R
        t_min = torch.zeros(R, device=dev)
        T = torch.ones(R, device=dev)
        rays = torch.arange(R, dtype=torch.int32, device=dev)
        p = 0
        while rays.numel() > 0:
            n = rays.numel()
            t_hit, idx_hit = self._pass_hits(rays.cpu().numpy().astype(np.int64), p)
            is_active = torch.zeros(n, dtype=torch.int32, device=dev)
            _launch(kind, make_args(rays, t_hit, idx_hit, t_min, T, is_active, n, p), n)
            torch.cuda.synchronize()
            rays = rays[is_active.bool()].contiguous()
            p += 1
        self.passes = p

    def _dec(self):
        g = self.g
        return [g.cond, g.features, g.A1, g.b1, g.A2, g.b2, g.A3, g.b3]

    def _geo(self):
        g = self.g
        return [g.m, g.s, g.q, g.RGBA, g.k]

    def forward_training(self, base, bitmap, bg, T_thr, dacc, reg_a, reg_b, dai, sn, nacc):
        """Forward_training(_base): bitmap, depth_reg_accums, normal_reg_accums accumulated in place."""
        kind = "fwd_training_base" if base else "fwd_training"
        dec = [] if base else self._dec()

        def args(rays, th, ih, tmin, T, act, n, p):
            return dec + [self.O, self.v, rays, th, ih, tmin, T, act, bitmap, n, tuple(bg)] + self._geo() + \
                [T_thr, dacc, reg_a, reg_b, dai, sn, nacc]
        self._loop(kind, args)

    def forward_inference(self, base, bitmap, normal, alpha, edn, bg, T_thr, override_colors=None):
        """Forward_inference(_base)(_with_geometry) / Forward_pca: normal, alpha, expected-depth numerator
        may be None (the reference's plain inference passes null pointers)."""
        kind = "fwd_inference_base" if base else "fwd_inference"
        dec = [] if base else self._dec()

        def args(rays, th, ih, tmin, T, act, n, p):
            a = dec + [self.O, self.v, rays, th, ih, tmin, T, act, bitmap, normal, alpha, edn, n, tuple(bg)] + \
                self._geo() + [T_thr]
            return a if base else a + [override_colors]
        self._loop(kind, args)

    def median_depth(self, base, T_thr, dai):
        kind = "median_base" if base else "median"
        dec = [] if base else self._dec()

        def args(rays, th, ih, tmin, T, act, n, p):
            return dec + [self.O, self.v, rays, th, ih, tmin, T, act, n] + self._geo() + [T_thr, p, dai]
        self._loop(kind, args)

    def backward(self, base, bg, I, dL_dI, G, W, T_thr, dacc, prefix, lam_d, reg_a, reg_b, dai, sn, nacc, lam_n):
        """Backward(_base).  G: dict of caller-zeroed gradients RGB A k m s q (+ cond features); W: the
        per-warp weight-gradient buffers w3 b3 w2 b2 w1 b1, (4 * SM_count, .) each."""
        kind = "backward_base" if base else "backward"
        dec = [] if base else self._dec()

        def args(rays, th, ih, tmin, T, act, n, p):
            grads = [G["RGB"], G["A"], G["k"]]
            if not base:
                grads += [W["w3"], W["b3"], W["w2"], W["b2"], W["w1"], W["b1"], G["cond"], G["features"]]
            grads += [G["m"], G["s"], G["q"]]
            return dec + [self.O, self.v, rays, th, ih, tmin, T, act, n, tuple(bg)] + self._geo() + \
                [I, dL_dI] + grads + [T_thr, dacc, prefix, lam_d, reg_a, reg_b, dai, sn, nacc, lam_n]
        self._loop(kind, args)
