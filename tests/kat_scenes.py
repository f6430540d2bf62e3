"""Known-answer scenes of the reference's planned test strategy: coplanar primitives with equal t, grazing
rays, and transmittance termination inside a pass.  Shared by the CPU oracle tests and the GPU parity
tests; every scene is (m, s, q, RGBA, k) raw parameters plus rays (O, v), all float32 CPU tensors."""
import math

import torch

IDENT = (1.0, 0.0, 0.0, 0.0)


def _scene(m, log_s, q, rgb, opacity, kappa=2.0):
    n = len(m)
    A = math.log(opacity / (1.0 - opacity))
    k = math.log(math.expm1(kappa - 1.0))  # kappa = 1 + softplus(k)
    return dict(m=torch.tensor(m, dtype=torch.float32), s=torch.full((n, 2), log_s),
                q=torch.tensor([q] * n, dtype=torch.float32),
                RGBA=torch.cat([torch.tensor(rgb, dtype=torch.float32), torch.full((n, 1), A)], 1).contiguous(),
                k=torch.full((n, 1), k))


def coplanar(n=20):
    """n identical-plane primitives at z = 2 whose supports all cover the z axis: rays along +z from the
    origin meet every one at exactly t = 2, so the hit order is by primitive index alone and a 16-entry
    buffer keeps indices 0..15."""
    m = [[0.001 * ((i % 5) - 2), 0.001 * ((i // 5) - 2), 2.0] for i in range(n)]
    rgb = [[(i % 3) / 2.0, 0.5, 1.0 - (i % 3) / 2.0] for i in range(n)]
    sc = _scene(m, math.log(0.2), IDENT, rgb, 0.3)
    O = torch.zeros(64, 3)
    v = torch.zeros(64, 3)
    v[:, 2] = 1.0
    return sc, O, v


def grazing():
    """One primitive in the plane z = 2 and rays that lie in that plane (N.v = 0: no intersection) or
    graze it at shallow angles (the hit moves far along the ray and in and out of the polygon)."""
    sc = _scene([[0.0, 0.0, 2.0]], math.log(0.3), IDENT, [[1.0, 0.0, 0.0]], 0.8)
    rows = []
    for i in range(64):
        ang = 0.0 if i < 8 else 10.0 ** (-7.0 + 6.0 * (i - 8) / 55.0)  # 8 exactly in-plane, then 1e-7 .. 1e-1 rad
        rows.append((math.cos(ang), 0.0, math.sin(ang)))
    v = torch.tensor(rows, dtype=torch.float32)
    O = torch.tensor([[-1.0, 0.0, 2.0]] * 64, dtype=torch.float32)
    O[8:, 2] = 2.0 - 0.5 * v[8:, 2] / v[8:, 0]  # cross z = 2 half a unit along x from the origin
    return sc, O, v


def stack(n=30, opacity=0.8):
    """n large opaque primitives stacked along +z (z = 1, 1.1, ...), rays along the axis through every
    centre: alpha = opacity exactly (G(0) = 1), T after j hits = (1 - opacity)^j, so with T_thr = 1e-4 a
    ray composites the first j with (1 - opacity)^j < 1e-4 hits (6 for opacity 0.8) and then stops, in
    the middle of the first pass."""
    m = [[0.0, 0.0, 1.0 + 0.1 * i] for i in range(n)]
    rgb = [[0.9, 0.1 + 0.02 * i, 0.3] for i in range(n)]
    sc = _scene(m, math.log(0.5), IDENT, rgb, opacity)
    O = torch.zeros(64, 3)
    v = torch.zeros(64, 3)
    v[:, 2] = 1.0
    return sc, O, v


def activated(sc):
    return (sc["m"], torch.exp(sc["s"]), sc["q"], torch.sigmoid(sc["RGBA"][:, 3]).contiguous(),
            (1.0 + torch.nn.functional.softplus(sc["k"][:, 0])).contiguous())


def expected_stack_image(sc, T_thr=1e-4, bg=(0.0, 0.0, 0.0)):
    """Analytic front-to-back composite of the stack scene along its axis: (rgb, composited hits)."""
    a = float(torch.sigmoid(sc["RGBA"][0, 3]))
    T, rgb, j = 1.0, [0.0, 0.0, 0.0], 0
    for i in range(sc["m"].shape[0]):
        if not T >= T_thr:
            break
        for c in range(3):
            rgb[c] += float(sc["RGBA"][i, c]) * a * T
        T -= T * a
        j += 1
    if T >= T_thr:
        rgb = [rgb[c] + bg[c] * T for c in range(3)]
    return rgb, j
