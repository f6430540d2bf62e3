"""CPU oracle for the FlaRe render path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs import this module,
and only as the checker or the timed CPU baseline.  The product package (flare_b200/) never imports it.

Pieces (see the headers of trace_oracle.c and decode_oracle.c for the reference lines restated):
  prep_frames      proxy frames from SetGeometry inputs          (Core.cu:553-622)
  hits             16-nearest hits beyond t_min, brute force     (shaders.cu:145-189)
  hit_lists        the multi-pass restart loop -> per-ray CSR    (Forward_training.cu:1004-1131)
  forward          decode + composite over CSR hit lists         (Forward_*.cu, GetMedianDepth*.cu)
Gradients are in grad_oracle.py (torch autograd in float64).

Parity status: the reference needs the closed OptiX SDK and a GPU, so it cannot be run here; the hit
test (octagon proxy) is pinned by analytic known-answer scenes and the LUT by the reference's own
Python LUT level (scripts/encoding_2d_benchmark.py:107-163), see tests/golden/make_golden.py.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

K = 16
MODES = {"training": 0, "inference": 1, "geometry": 2, "pca": 3, "median": 4}


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB):
            build()
        _lib = ctypes.CDLL(_LIB)
        _lib.oracle_shade_csr.restype = ctypes.c_long
        _lib.oracle_next_tmin.restype = ctypes.c_float
        _lib.oracle_next_tmin.argtypes = [ctypes.c_float]
        _lib.oracle_bvh_build.restype = ctypes.c_void_p
        _lib.oracle_bvh_build.argtypes = [ctypes.c_void_p, ctypes.c_int]
        _lib.oracle_bvh_free.argtypes = [ctypes.c_void_p]
        _lib.oracle_bvh_hits.argtypes = [ctypes.c_void_p] + [ctypes.c_void_p] * 3 + [ctypes.c_int] * 2 + \
            [ctypes.c_void_p] * 2
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _np(t, dtype=None):
    """torch tensor or array -> contiguous numpy (float32 unless dtype given)."""
    if hasattr(t, "detach"):
        t = t.detach().cpu().numpy()
    return np.ascontiguousarray(t if dtype is None else np.asarray(t, dtype=dtype))


def polygon_constants(nsides=8):
    c = np.zeros(nsides, np.float32)
    s = np.zeros(nsides, np.float32)
    lib().oracle_polygon_constants(ctypes.c_int(nsides), _p(c), _p(s))
    return c, s


def prep_frames(m, scale, q, opacity, kappa):
    m, scale, q, opacity, kappa = (_f32(_np(x)) for x in (m, scale, q, opacity, kappa))
    n = m.shape[0]
    out = np.zeros((n, 12), np.float32)
    lib().oracle_prep_frames(_p(m), _p(scale), _p(q), _p(opacity), _p(kappa), ctypes.c_int(n), _p(out))
    return out


def hits(frames, O, v, t_min, nsides=8):
    frames, O, v, t_min = (_f32(_np(x)) for x in (frames, O, v, t_min))
    R = O.shape[0]
    t = np.zeros((K, R), np.float32)
    idx = np.zeros((K, R), np.int32)
    lib().oracle_hits(_p(frames), ctypes.c_int(frames.shape[0]), _p(O), _p(v), _p(t_min), ctypes.c_int(R),
                      ctypes.c_int(nsides), _p(t), _p(idx))
    return t, idx


def next_tmin(t16):
    return np.nextafter(np.float32(t16), np.float32(np.inf), dtype=np.float32)


def hit_lists(frames, O, v, nsides=8, max_passes=100000, stop=None):
    """Runs the multi-pass restart loop to exhaustion: every hit of every ray in ascending (t, idx)
    order, with the reference's restart t_min = nextafter(t_16) (ties at t_16 with a larger index are
    dropped, as the reference's k-buffer drops them).  Returns CSR (off (R+1) int64, t, idx).
    `stop`, if given, ends rays early (the renderer stops a ray once its transmittance falls below the
    threshold)."""
    O, v = _f32(_np(O)), _f32(_np(v))
    R = O.shape[0]
    t_min = np.zeros(R, np.float32)
    per_ray_t = [[] for _ in range(R)]
    per_ray_i = [[] for _ in range(R)]
    active = np.arange(R)
    passes = 0
    while active.size and passes < max_passes:
        t, idx = hits(frames, O[active], v[active], t_min[active], nsides)
        for j, r in enumerate(active):
            valid = idx[:, j] >= 0
            per_ray_t[r].extend(t[valid, j].tolist())
            per_ray_i[r].extend(idx[valid, j].tolist())
        full = idx[K - 1] >= 0
        if stop is not None:  # stop(ray ids, CSR so far) -> rays whose compositing has terminated
            full &= ~stop(active, per_ray_t, per_ray_i)
        t_min[active[full]] = np.nextafter(t[K - 1, full], np.float32(np.inf), dtype=np.float32)
        active = active[full]
        passes += 1
    off = np.zeros(R + 1, np.int64)
    off[1:] = np.cumsum([len(x) for x in per_ray_i])
    tt = np.array([x for r in per_ray_t for x in r], np.float32)
    ii = np.array([x for r in per_ray_i for x in r], np.int32)
    return off, tt, ii


def scene_arrays(scene):
    """numpy views of a flare_b200.scene.Scene (or dict) in the oracle's dtypes."""
    g = scene if isinstance(scene, dict) else scene.__dict__
    out = {}
    for k_, x in g.items():
        if k_ in ("cond", "A1", "A2", "A3"):
            out[k_] = _np(x, np.float16)
        else:
            out[k_] = _f32(_np(x))
    return out


def decoder_of(S) -> int:
    """Decoder kind of a scene's arrays: 1 (grid/SH) for a 32-wide descriptor, else 0 (LUT/PE)."""
    c = S.get("cond")
    return 1 if c is not None and c.ndim == 2 and c.shape[1] == 32 else 0


def forward(scene, O, v, csr, mode="training", base=False, bg=(0.0, 0.0, 0.0), T_thr=1e-4, reg_a=0.0,
            reg_b=0.0, surface_normal=None, override_colors=None):
    """Forward over CSR hit lists.  Returns a dict of numpy outputs (rgb, dacc, nacc, normal, alpha,
    edn, med (R,2) with the index as float bits, T, nhits) and the composited-hit total."""
    S = scene_arrays(scene)
    O, v = _f32(_np(O)), _f32(_np(v))
    R = O.shape[0]
    off, tt, ii = csr
    off = np.ascontiguousarray(off, np.int64)
    tt = _f32(tt)
    ii = np.ascontiguousarray(ii, np.int32)
    out = {
        "rgb": np.zeros((R, 3), np.float32), "dacc": np.zeros((R, 4), np.float32),
        "nacc": np.zeros((R, 4), np.float32), "normal": np.zeros((R, 3), np.float32),
        "alpha": np.zeros(R, np.float32), "edn": np.zeros(R, np.float32), "med": np.zeros((R, 2), np.float32),
        "T": np.zeros(R, np.float32), "nhits": np.zeros(R, np.int32),
    }
    sn = None if surface_normal is None else _f32(_np(surface_normal))
    oc = None if override_colors is None else _f32(_np(override_colors))
    bgv = _f32(bg)
    G = lambda k_: _p(S.get(k_)) if not base else None  # noqa: E731
    total = lib().oracle_shade_csr(
        _p(S["m"]), _p(S["s"]), _p(S["q"]), _p(S["RGBA"]), _p(S["k"]),
        G("cond"), G("features"), G("A1"), G("b1"), G("A2"), G("b2"), G("A3"), G("b3"), _p(oc), ctypes.c_int(MODES[mode]), _p(bgv),
        ctypes.c_float(T_thr), ctypes.c_float(reg_a), ctypes.c_float(reg_b), _p(O), _p(v), _p(sn),
        ctypes.c_int(R), _p(off), _p(tt), _p(ii), _p(out["rgb"]), _p(out["dacc"]), _p(out["nacc"]),
        _p(out["normal"]), _p(out["alpha"]), _p(out["edn"]), _p(out["med"]), _p(out["T"]), _p(out["nhits"]),
        ctypes.c_int(decoder_of(S)))
    out["total_hits"] = int(total)
    return out


def lut(features, cu, cw):
    """The 4-level LUT encoding of coordinates (cu, cw) (already scaled by 1/sqrt(11.3449)) -> (n, 8)."""
    features, cu, cw = _f32(_np(features)), _f32(_np(cu)), _f32(_np(cw))
    out = np.zeros((cu.shape[0], 8), np.float32)
    lib().oracle_lut(_p(features), _p(cu), _p(cw), ctypes.c_int(cu.shape[0]), _p(out))
    return out


def grid(features, cu, cw):
    """The 8-level dense-grid encoding of the grid/SH decoder variant -> (n, 16)."""
    features, cu, cw = _f32(_np(features)), _f32(_np(cu)), _f32(_np(cw))
    out = np.zeros((cu.shape[0], 16), np.float32)
    lib().oracle_grid(_p(features), _p(cu), _p(cw), ctypes.c_int(cu.shape[0]), _p(out))
    return out


def sh(v):
    """Degree-3 real spherical harmonics of unit directions (n, 3) -> (n, 16)."""
    v = _f32(_np(v))
    out = np.zeros((v.shape[0], 16), np.float32)
    lib().oracle_sh(_p(v), ctypes.c_int(v.shape[0]), _p(out))
    return out


def all_hits(frames, O, v, t_min=None, nsides=8, cap=4096):
    """Every hit of each ray (t >= t_min, default 0) ascending by (t, index), from one brute-force sweep
    per ray: a list of (t, idx) numpy arrays.  For full-size parity on a few hundred sampled rays."""
    frames, O, v = _f32(_np(frames)), _f32(_np(O)), _f32(_np(v))
    R = O.shape[0]
    t_min = np.zeros(R, np.float32) if t_min is None else _f32(_np(t_min))
    counts = np.zeros(R, np.int32)
    t = np.zeros((R, cap), np.float32)
    idx = np.zeros((R, cap), np.int32)
    worst = lib().oracle_all_hits(_p(frames), ctypes.c_int(frames.shape[0]), _p(O), _p(v), _p(t_min),
                                  ctypes.c_int(R), ctypes.c_int(nsides), ctypes.c_int(cap), _p(counts), _p(t), _p(idx))
    if worst > cap:
        return all_hits(frames, O, v, t_min, nsides, cap=int(worst) + 64)
    return [(t[r, :counts[r]].copy(), idx[r, :counts[r]].copy()) for r in range(R)]


def restart_passes(t, idx, k):
    """Splits one ray's sorted hit sequence into the passes of a k-slot buffer that restarts at
    nextafter(t_k) (Forward_training.cu:929): a pass holds the next k hits at or beyond t_min; hits tied
    with t_k but later in (t, index) order are skipped by the restart, as the reference's k-buffer skips
    them.  Returns a list of (t, idx) arrays, the last one shorter than k (possibly empty)."""
    out = []
    pos = 0
    n = len(t)
    while True:
        chunk_t, chunk_i = t[pos:pos + k], idx[pos:pos + k]
        out.append((chunk_t, chunk_i))
        if len(chunk_t) < k:
            return out
        t_next = np.nextafter(chunk_t[-1], np.float32(np.inf), dtype=np.float32)
        pos += k
        while pos < n and t[pos] < t_next:
            pos += 1


def csr_from_passes(per_ray_passes):
    """CSR (off, t, idx) of the concatenated pass lists of every ray (the form forward() and
    grad_oracle.gradients() read)."""
    lists_t = [np.concatenate([p[0] for p in ps]) if ps else np.zeros(0, np.float32) for ps in per_ray_passes]
    lists_i = [np.concatenate([p[1] for p in ps]) if ps else np.zeros(0, np.int32) for ps in per_ray_passes]
    off = np.zeros(len(lists_t) + 1, np.int64)
    off[1:] = np.cumsum([len(x) for x in lists_t])
    tt = np.concatenate(lists_t).astype(np.float32) if lists_t else np.zeros(0, np.float32)
    ii = np.concatenate(lists_i).astype(np.int32) if lists_i else np.zeros(0, np.int32)
    return off, tt, ii


class CpuBvh:
    """The oracle's CPU hierarchy over a scene's frames (oracle_bvh_build): hits(O, v, t_min) gives the same
    16-nearest lists as hits() without scanning every primitive.  Keeps `frames` alive."""

    def __init__(self, frames, nsides=8):
        self.frames = _f32(_np(frames))
        self.nsides = nsides
        self.h = lib().oracle_bvh_build(_p(self.frames), ctypes.c_int(self.frames.shape[0]))

    def hits(self, O, v, t_min):
        O, v, t_min = (_f32(_np(x)) for x in (O, v, t_min))
        R = O.shape[0]
        t = np.zeros((K, R), np.float32)
        idx = np.zeros((K, R), np.int32)
        lib().oracle_bvh_hits(ctypes.c_void_p(self.h), _p(O), _p(v), _p(t_min), ctypes.c_int(R),
                              ctypes.c_int(self.nsides), _p(t), _p(idx))
        return t, idx

    def render(self, scene, O, v, mode="training", base=False, bg=(0.0, 0.0, 0.0), T_thr=1e-4, reg_a=0.0, reg_b=0.0,
               cap=512):
        """The reference's forward on the CPU end to end (oracle_render_bvh): multi-pass 16-nearest queries on
        this hierarchy, each pass decoded and composited until the ray terminates.  Returns (rgb, CSR of the
        composited hits, nhits, traversal thread-seconds, shading thread-seconds)."""
        S = scene_arrays(scene)
        O, v = _f32(_np(O)), _f32(_np(v))
        R = O.shape[0]
        rgb = np.zeros((R, 3), np.float32)
        T = np.zeros(R, np.float32)
        nh = np.zeros(R, np.int32)
        ht = np.zeros((R, cap), np.float32)
        hi = np.zeros((R, cap), np.int32)
        times = np.zeros(2, np.float64)
        bgv = _f32(bg)
        G = lambda k_: _p(S.get(k_)) if not base else None  # noqa: E731
        lib().oracle_render_bvh(
            ctypes.c_void_p(self.h), ctypes.c_int(self.nsides), _p(S["m"]), _p(S["s"]), _p(S["q"]), _p(S["RGBA"]),
            _p(S["k"]), G("cond"), G("features"), G("A1"), G("b1"), G("A2"), G("b2"), G("A3"), G("b3"),
            ctypes.c_int(MODES[mode]), _p(bgv), ctypes.c_float(T_thr), ctypes.c_float(reg_a), ctypes.c_float(reg_b),
            _p(O), _p(v), ctypes.c_int(R), ctypes.c_int(cap), _p(ht), _p(hi), _p(rgb), _p(T), _p(nh), _p(times),
            ctypes.c_int(decoder_of(S)))
        off = np.zeros(R + 1, np.int64)
        off[1:] = np.cumsum(nh)
        tt = np.concatenate([ht[r, :nh[r]] for r in range(R)]) if R else np.zeros(0, np.float32)
        ii = np.concatenate([hi[r, :nh[r]] for r in range(R)]) if R else np.zeros(0, np.int32)
        return rgb, (off, tt, ii), nh, float(times[0]), float(times[1])

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib().oracle_bvh_free(ctypes.c_void_p(self.h))
                self.h = None
        except Exception:  # interpreter shutdown
            pass

