"""flare_render_hits_noalloc against the renderer path (flare_set_geometry + flare_render_hits).

Some callers cannot allocate device memory at call time: hosts that give this library a fixed device
budget, plugins inside processes whose allocator owns the GPU.  They use flare_render_hits_noalloc, whose scratch is a static device array.  Its hits
must equal the renderer's (indices and t are bit-comparable, the bar of the other hit tests) on calls
in a row that reuse that array.  The file name makes pytest collect it last.
"""
import ctypes

import torch
import pytest

from flare_b200 import _lib
from flare_b200.scene import camera_rays, make_scene

MAX_PRIMS = 32768


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(lib, act, O, v, tmin, sides=8):
    m, scale, q, op, ka = act
    R = O.shape[0]
    t = torch.empty((16, R), dtype=torch.float32, device="cuda")
    idx = torch.empty((16, R), dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.flare_render_hits_noalloc(sides, _p(m), _p(scale), _p(q), _p(op), _p(ka), m.shape[0], _p(O), _p(v),
                                       _p(tmin), R, _p(t), _p(idx), stream)
    _lib.check(rc, "flare_render_hits_noalloc")
    return t, idx


def test_noalloc_rejects_scenes_beyond_its_maximum():
    lib = _lib.load()
    rc = lib.flare_render_hits_noalloc(8, None, None, None, None, None, MAX_PRIMS + 1, None, None, None, 1, None,
                                       None, None)
    assert rc == 1
    assert b"at most 32768" in lib.flare_last_error()


@pytest.mark.gpu
def test_noalloc_matches_renderer_on_consecutive_calls():
    from flare_b200.renderer import CPyOptiXFLARERenderer
    lib = _lib.load()
    # two calls in a row with different scenes, views and t_min: the second reuses the first's scratch
    for n, seed, eye, t0 in [(20000, 0, (0.0, 0.0, 3.0), 0.0), (MAX_PRIMS, 7, (0.5, 1.0, 2.5), 1.5)]:
        sc = make_scene(n, seed).to("cuda")
        act = [t.contiguous() for t in sc.activated()]
        O, v = camera_rays(48, 48, 60.0, eye=eye)
        O, v = O.cuda(), v.cuda()
        tmin = torch.full((O.shape[0],), t0, device="cuda")
        t_na, i_na = _noalloc(lib, act, O, v, tmin)
        r = CPyOptiXFLARERenderer(8, 11.3449, O.shape[0])
        r.SetGeometry(*act)
        t_ref, i_ref = r.Render(O, v, tmin, O.shape[0])
        torch.cuda.synchronize()
        assert (i_ref >= 0).sum().item() > 500
        assert torch.equal(i_na, i_ref)
        assert torch.equal(t_na, t_ref)


@pytest.mark.gpu
def test_noalloc_small_scenes_after_a_large_call():
    """After a full-size call leaves its hierarchy in the shared array, a 0-primitive call reports every
    ray as a miss and a 1-primitive call (the traversal's single-leaf path) equals the renderer: neither
    reads the earlier call's scratch."""
    from flare_b200.renderer import CPyOptiXFLARERenderer
    lib = _lib.load()
    O, v = camera_rays(32, 32, 60.0, eye=(0.0, 0.0, 3.0))
    O, v = O.cuda(), v.cuda()
    R = O.shape[0]
    tmin = torch.zeros(R, device="cuda")
    big = [t.contiguous() for t in make_scene(MAX_PRIMS, 3).to("cuda").activated()]
    _, i_big = _noalloc(lib, big, O, v, tmin)
    assert (i_big >= 0).sum().item() > 100
    empty = [t[:0].contiguous() for t in big]
    t0, i0 = _noalloc(lib, empty, O, v, tmin)
    torch.cuda.synchronize()
    assert torch.all(i0 == -1) and torch.all(torch.isinf(t0))
    # one large primitive facing the camera at the origin: the central rays hit it
    sc1 = make_scene(1, 0)
    sc1.m.zero_()
    sc1.s.fill_(-0.5)
    sc1.q.copy_(torch.tensor([[1.0, 0.0, 0.0, 0.0]]))
    one = [t.contiguous() for t in sc1.to("cuda").activated()]
    t1, i1 = _noalloc(lib, one, O, v, tmin)
    r = CPyOptiXFLARERenderer(8, 11.3449, R)
    r.SetGeometry(*one)
    t_ref, i_ref = r.Render(O, v, tmin, R)
    torch.cuda.synchronize()
    assert (i_ref[0] == 0).sum().item() > 10
    assert torch.equal(i1, i_ref) and torch.equal(t1, t_ref)
