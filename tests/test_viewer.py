"""Secondary-ray (viewer) path: the CPU oracle's pieces on known answers, and the CUDA path against the
oracle (GPU).  Spheres stand in for the reference viewer's meshes."""
import numpy as np
import pytest
import torch

from flare_b200.scene import camera_rays, make_scene
from oracle import oracle, viewer_oracle


def test_sphere_nearest_known_answers():
    sph = np.array([[0.0, 0.0, -5.0, 1.0]], np.float32)
    O = np.array([[0, 0, 0], [0, 0, -5], [0, 3, 0], [0, 0, -10]], np.float32)
    v = np.array([[0, 0, -1], [0, 0, -1], [0, 0, -1], [0, 0, -1]], np.float32)
    t, sid = viewer_oracle.sphere_nearest(sph, O, v, np.zeros(4, np.float32))
    assert t[0] == 4.0 and sid[0] == 0          # front face
    assert t[1] == 1.0                          # from the centre: the exit point
    assert np.isinf(t[2]) and sid[2] == -1      # miss
    assert np.isinf(t[3])                       # sphere behind the ray


def _scene_rgba(sc):
    d = dict(sc.__dict__)
    return d


def test_viewer_without_spheres_is_plain_compositing():
    """No spheres, no lights: one generation, every ray composites its whole list with no background,
    which is the inference forward with a black background."""
    sc = make_scene(3000, 4)
    O, v = camera_rays(24, 24, 60.0, eye=(0.0, 0.0, 3.0))
    frames = oracle.prep_frames(*sc.activated())
    bm, st = viewer_oracle.viewer_forward(frames, _scene_rgba(sc), np.zeros((0, 4), np.float32),
                                          np.zeros((0, 6), np.float32), np.zeros((0, 6), np.float32), O, v,
                                          T_thr=1e-4, max_depth=3)
    ref = oracle.forward(sc, O, v, oracle.hit_lists(frames, O, v), mode="inference", T_thr=1e-4)
    assert st["generations"] == 1
    np.testing.assert_allclose(bm, ref["rgb"], rtol=0, atol=1e-6)


def test_viewer_recursion_bounded_and_sane():
    sc = make_scene(3000, 5)
    O, v = camera_rays(24, 24, 60.0, eye=(0.0, 0.0, 3.0))
    frames = oracle.prep_frames(*sc.activated())
    sph, mat = viewer_oracle.default_spheres()
    bm, st = viewer_oracle.viewer_forward(frames, _scene_rgba(sc), sph, mat, viewer_oracle.default_lights(), O, v,
                                          bg=(0.2, 0.3, 0.4), T_thr=0.01, max_depth=3)
    assert st["generations"] > 1
    assert np.isfinite(bm).all() and (bm >= 0).all()
    # depth 0: the pushed sets are dropped at once, fewer generations
    _, st0 = viewer_oracle.viewer_forward(frames, _scene_rgba(sc), sph, mat, viewer_oracle.default_lights(), O, v,
                                          bg=(0.2, 0.3, 0.4), T_thr=0.01, max_depth=0)
    assert st0["generations"] <= st["generations"]


@pytest.mark.gpu
@pytest.mark.parametrize("depth", [0, 3])
def test_viewer_forward_matches_oracle(depth):
    from flare_b200.viewer import CPyFlareViewerRenderer
    sc = make_scene(10000, 6)
    W = 48
    O, v = camera_rays(W, W, 60.0, eye=(0.0, 0.5, 3.0))
    R = W * W
    g = sc.to("cuda")
    r = CPyFlareViewerRenderer(8, 11.3449, R, depth)
    sph, mat = viewer_oracle.default_spheres()
    lts = viewer_oracle.default_lights()
    r.SetGeometry(*[t.contiguous() for t in g.activated()], torch.from_numpy(sph))
    bm = torch.zeros(R, 3, device="cuda")
    args = dict(bg=(0.2, 0.3, 0.4), T_thr=0.01, eps=1e-4, shadow_mult=0.55, Ia=(0.06, 0.06, 0.07))
    r.Forward(g.cond, g.features, g.RGBA[:, :3].contiguous(), g.A1, g.b1, g.A2, g.b2, g.A3, g.b3, O.cuda(), v.cuda(),
              bm, *args["bg"], g.m, g.s, g.q, g.RGBA[:, 3].contiguous(), g.k, args["T_thr"], torch.from_numpy(mat),
              torch.from_numpy(lts), args["eps"], args["shadow_mult"], *args["Ia"])
    frames = r.frames().cpu().numpy()
    ref, st = viewer_oracle.viewer_forward(frames, sc.__dict__, sph, mat, lts, O, v, bg=args["bg"], T_thr=args["T_thr"],
                                           eps=args["eps"], shadow_mult=args["shadow_mult"], Ia=args["Ia"],
                                           max_depth=depth)
    got = bm.cpu().numpy()
    err = np.abs(got - ref).max(axis=1)
    assert st["generations"] > (1 if depth > 0 else 0)
    assert err.max() < 1e-3, ((err > 1e-3).sum(), err.max())
