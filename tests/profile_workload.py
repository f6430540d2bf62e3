"""Small fixed workload for kernel profiling (ncu) of the render path.

    python tests/profile_workload.py [n_primitives=1000000] [width=400]

Renders a seeded scene (BASELINE config-0 distributions) with Forward_training + Backward twice through
CPyOptiXFLARERenderer, so each kernel launches several times; pick launches with ncu -k / -s / -c.
"""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from flare_b200.renderer import CPyOptiXFLARERenderer
from flare_b200.scene import camera_rays, make_scene


def main(n=1_000_000, w=400):
    sc = make_scene(n, 0).to("cuda")
    O, v = camera_rays(w, w, 60.0, eye=(0.0, 0.0, 3.0))
    O, v = O.cuda(), v.cuda()
    R = w * w
    r = CPyOptiXFLARERenderer(8, 11.3449, R)
    r.SetGeometry(*[t.contiguous() for t in sc.activated()])
    z = lambda *s: torch.zeros(*s, device="cuda")  # noqa: E731
    dec = (sc.cond, sc.features, sc.A1, sc.b1, sc.A2, sc.b2, sc.A3, sc.b3)
    geo = (sc.m, sc.s, sc.q, sc.RGBA, sc.k)
    for _ in range(2):
        bm, da, na, dai, sn = z(R, 3), z(R, 4), z(R, 4), z(R, 2), z(R, 3)
        r.Forward_training(*dec, O, v, bm, 0.0, 0.0, 0.0, *geo, 1e-4, da, -0.1, 1.0, dai, sn, na)
        st = r.stats()
        G = [z(n, 3), z(n, 1), z(n, 1)]
        W = [z(1, 512), z(1, 64), z(1, 4096), z(1, 512), z(1, 8192), z(1, 512)]
        r.Backward(*dec, O, v, 0.0, 0.0, 0.0, *geo, bm.clone(), torch.randn(R, 3, device="cuda") / R, *G, *W,
                   z(n, 96), z(13154), z(n, 3), z(n, 2), z(n, 4), 1e-4, da, z(R, 4), 0.0, -0.1, 1.0, dai, sn, na, 0.0)
    torch.cuda.synchronize()
    print("forward stats", st)


if __name__ == "__main__":
    main(*(int(a) for a in sys.argv[1:3]))
