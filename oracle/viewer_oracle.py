"""CPU oracle of the secondary-ray (viewer) path -- TEST INFRASTRUCTURE ONLY.

Drives the C restatement (viewer_oracle.c, decode_oracle.c, trace_oracle.c) through the reference
viewer's ray-generation loop (source/viewer_renderer/CPyOptiXFLAREVIEWERRenderer_CUDA_Forward.cu:
995-1276): a generation's rays run their k-nearest passes up to the nearest sphere, get shadow flags and
are composited; at the end of the generation each ray that reached a sphere is shaded and split, the
child with more transmittance continuing in place and the other pushed on a stack of ray sets; a set
pushed when the stack is max_recursion_depth deep is dropped together with the in-place children.
Only tests/ and bench.py's CPU legs import it.
"""
from __future__ import annotations

import ctypes

import numpy as np

from .oracle import K, _f32, _np, _p, decoder_of, lib, scene_arrays


def _lib():
    L = lib()
    if not getattr(L, "_viewer_sig", False):
        L.oracle_viewer_composite.restype = ctypes.c_long
        L._viewer_sig = True
    return L


def sphere_nearest(spheres, O, v, tmin):
    R = O.shape[0]
    t = np.zeros(R, np.float32)
    sid = np.zeros(R, np.int32)
    _lib().oracle_sphere_nearest(_p(spheres), ctypes.c_int(spheres.shape[0]), _p(O), _p(v), _p(tmin),
                                 ctypes.c_int(R), _p(t), _p(sid))
    return t, sid


def hits_tmax(frames, O, v, tmin, tmax, nsides=8):
    R = O.shape[0]
    t = np.zeros((K, R), np.float32)
    idx = np.zeros((K, R), np.int32)
    _lib().oracle_hits_tmax(_p(frames), ctypes.c_int(frames.shape[0]), _p(O), _p(v), _p(tmin), _p(tmax),
                            ctypes.c_int(R), ctypes.c_int(nsides), _p(t), _p(idx))
    return t, idx


def hit_lists_tmax(frames, O, v, tmin, tmax, nsides=8):
    """All hits in [tmin, tmax) of each ray in ascending (t, idx) order, with the product's restart rule
    (t_min = nextafter of the last buffered hit)."""
    R = O.shape[0]
    tmin = tmin.copy()
    per_t = [[] for _ in range(R)]
    per_i = [[] for _ in range(R)]
    active = np.arange(R)
    while active.size:
        t, idx = hits_tmax(frames, O[active], v[active], tmin[active], tmax[active], nsides)
        for j, r in enumerate(active):
            ok = idx[:, j] >= 0
            per_t[r].extend(t[ok, j].tolist())
            per_i[r].extend(idx[ok, j].tolist())
        full = idx[K - 1] >= 0
        tmin[active[full]] = np.nextafter(t[K - 1, full], np.float32(np.inf), dtype=np.float32)
        active = active[full]
    off = np.zeros(R + 1, np.int64)
    off[1:] = np.cumsum([len(x) for x in per_i])
    tt = np.array([x for r in per_t for x in r], np.float32)
    ii = np.array([x for r in per_i for x in r], np.int32)
    return off, tt, ii


def viewer_forward(frames, scene, spheres, materials, lights, O, v, bg=(0.0, 0.0, 0.0), T_thr=0.01, eps=1e-4,
                   shadow_mult=0.55, Ia=(0.06, 0.06, 0.07), max_depth=3, nsides=8):
    """Returns (bitmap (R,3), stats dict).  `scene` holds the decoder tensors and RGBA = [RGB | A]."""
    L_ = _lib()
    S = scene_arrays(scene)
    frames = _f32(frames)
    sph, mat, lts = _f32(spheres).reshape(-1, 4), _f32(materials).reshape(-1, 6), _f32(lights).reshape(-1, 6)
    R = O.shape[0]
    bitmap = np.zeros((R, 3), np.float32)
    Iav, bgv = _f32(Ia), _f32(bg)

    def new_set():
        return dict(O=np.zeros((R, 3), np.float32), v=np.zeros((R, 3), np.float32), T=np.zeros(R, np.float32),
                    tmin=np.zeros(R, np.float32), list=np.zeros(0, np.int32), processed=False)

    cur = new_set()
    cur["O"][:] = _f32(_np(O))
    cur["v"][:] = _f32(_np(v))
    cur["T"][:] = 1.0
    cur["list"] = np.arange(R, dtype=np.int32)
    stack = [new_set() for _ in range(max_depth + 1)]
    ss = 0
    gens = 0
    hits_total = 0
    G = lambda k_: _p(S.get(k_))  # noqa: E731
    while True:
        gens += 1
        lst = cur["list"]
        n0 = lst.size
        act_in = np.zeros(n0, np.uint8)
        act_push = np.zeros(n0, np.uint8)
        push = stack[ss]
        if n0:
            Og = np.ascontiguousarray(cur["O"][lst])
            vg = np.ascontiguousarray(cur["v"][lst])
            t_sph, sid = sphere_nearest(sph, Og, vg, np.ascontiguousarray(cur["tmin"][lst]))
            off, tt, ii = hit_lists_tmax(frames, Og, vg, np.ascontiguousarray(cur["tmin"][lst]), t_sph, nsides)
            ray_of_hit = np.repeat(lst, np.diff(off)).astype(np.int32)
            flags = np.zeros(tt.size, np.uint8)
            L_.oracle_shadow_flags(_p(sph), ctypes.c_int(sph.shape[0]), _p(lts), ctypes.c_int(lts.shape[0]),
                                   ctypes.c_float(eps), _p(cur["O"]), _p(cur["v"]), _p(ray_of_hit), _p(tt),
                                   ctypes.c_long(tt.size), _p(flags))
            hits_total += L_.oracle_viewer_composite(
                _p(S["m"]), _p(S["s"]), _p(S["q"]), _p(S["RGBA"]), _p(S["k"]), G("cond"), G("features"), G("A1"),
                G("b1"), G("A2"), G("b2"), G("A3"), G("b3"), ctypes.c_float(T_thr), ctypes.c_float(shadow_mult),
                _p(cur["O"]), _p(cur["v"]), _p(lst), ctypes.c_int(n0), _p(off), _p(tt), _p(ii), _p(flags),
                _p(cur["T"]), _p(bitmap), ctypes.c_int(decoder_of(S)))
            tsf = np.full(R, np.inf, np.float32)
            sidf = np.full(R, -1, np.int32)
            tsf[lst] = t_sph
            sidf[lst] = sid
            L_.oracle_sphere_shade(_p(sph), _p(mat), ctypes.c_int(sph.shape[0]), _p(lts), ctypes.c_int(lts.shape[0]),
                                   ctypes.c_float(eps), ctypes.c_float(shadow_mult), ctypes.c_float(T_thr), _p(Iav),
                                   _p(bgv), _p(lst), ctypes.c_int(n0), _p(cur["O"]), _p(cur["v"]), _p(cur["T"]),
                                   _p(cur["tmin"]), _p(tsf), _p(sidf), _p(bitmap), _p(push["O"]), _p(push["v"]),
                                   _p(push["T"]), _p(push["tmin"]), _p(act_in), _p(act_push))
        in_list = lst[act_in.astype(bool)]
        push_list = lst[act_push.astype(bool)]
        pop = False
        if push_list.size:
            if ss < max_depth:
                push["list"] = push_list
                push["processed"] = False
                ss += 1
                cur["list"] = in_list
            else:
                pop = True
        else:
            cur["list"] = in_list
            pop = in_list.size == 0
        if pop:
            ss -= 1
            while ss >= 0 and stack[ss]["processed"]:
                ss -= 1
            if ss < 0:
                break
            cur = stack[ss]
            cur["processed"] = True
            ss += 1
    return bitmap, {"generations": gens, "hits": int(hits_total)}


def default_spheres():
    """The config-4 spheres and materials of flare_b200.scene.viewer_spheres, as numpy."""
    from flare_b200.scene import viewer_spheres
    sph, mat = viewer_spheres()
    return sph.numpy(), mat.numpy()


def default_lights():
    from flare_b200.scene import viewer_lights
    return viewer_lights().numpy()


__all__ = ["viewer_forward", "sphere_nearest", "hit_lists_tmax", "default_spheres", "default_lights"]
