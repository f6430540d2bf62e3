"""The reference's checkpoint tuples: 18- and 17-entry forms map onto the renderer's scene layout, and a
save -> load round trip keeps every tensor (CPU); the optimizer state survives the trip (GPU)."""
import pytest
import torch

from flare_b200 import checkpoint
from flare_b200.scene import make_scene


def _reference_tuple(n=50, legacy=False, seed=0):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    t = [r(n, 3), r(n, 1), r(n, 1), r(64, 8), r(64, 24), r(64, 96), r(64), r(64, 64), r(64), r(16, 64), r(16),
         r(n, 96), r(13154), r(n, 3), r(n, 2), r(n, 4), {"state": {}, "param_groups": []}, 123.5]
    return tuple(t[1:]) if legacy else tuple(t)


def test_tuple_maps_onto_scene_layout():
    t = _reference_tuple()
    sc = checkpoint.scene_from_tensors(checkpoint.tensors_from_tuple(t))
    assert torch.equal(sc.RGBA[:, :3], t[0]) and torch.equal(sc.RGBA[:, 3:], t[1])
    assert torch.equal(sc.A1, torch.cat([t[3], t[4], t[5]], 1).half())    # [uv 8 | view 24 | descriptor 96]
    assert torch.equal(sc.cond, t[11].half()) and torch.equal(sc.m, t[13]) and torch.equal(sc.q, t[15])
    assert sc.A3.shape == (16, 64) and sc.b3.shape == (16,)


def test_legacy_tuple_has_white_base_colour():
    t = _reference_tuple(legacy=True)
    sc = checkpoint.scene_from_tensors(checkpoint.tensors_from_tuple(t))
    assert torch.equal(sc.RGBA[:, :3], torch.ones(50, 3)) and torch.equal(sc.RGBA[:, 3:], t[0])
    with pytest.raises(ValueError):
        checkpoint.tensors_from_tuple(t[:10])


def test_save_load_round_trip(tmp_path):
    sc = make_scene(300, 1)
    p = tmp_path / "best.checkpoint"
    checkpoint.save(p, sc, training_time=7.0)
    sc2, t = checkpoint.load(p)
    for k in ("m", "s", "q", "RGBA", "k", "cond", "features", "A1", "b1", "A2", "b2", "A3", "b3"):
        assert torch.equal(getattr(sc2, k), getattr(sc, k)), k
    assert t["training_time_seconds"] == 7.0 and len(torch.load(p, weights_only=False)) == 18


@pytest.mark.gpu
def test_optimizer_state_round_trip(tmp_path):
    from flare_b200 import optim
    from flare_b200.dp import GradBuffer
    sc = make_scene(400, 2).to("cuda")
    G = GradBuffer(sc.n, True, "cuda")
    opt = optim.ModelOptimizer(sc, G)
    for it in range(1, 4):
        G.flat.normal_()
        opt.step(it)
    p = tmp_path / "c.checkpoint"
    checkpoint.save(p, sc, opt, training_time=1.0)
    sc2, t = checkpoint.load(p, "cuda")
    G2 = GradBuffer(sc2.n, True, "cuda")
    opt2 = optim.ModelOptimizer(sc2, G2)
    checkpoint.restore_optimizer(opt2, t)
    assert opt2.adam.t == 3
    for (m1, v1), (m2, v2) in zip(opt.adam.state, opt2.adam.state):
        assert torch.equal(m1.reshape(-1), m2.reshape(-1)) and torch.equal(v1.reshape(-1), v2.reshape(-1))
    assert torch.equal(opt2.W1, opt.W1) and torch.equal(opt2.cond32, opt.cond32)


def test_legacy_optimizer_state_skips_the_rgb_segment():
    """A 17-entry checkpoint's optimizer has no RGB group: its group 0 holds A's moments."""
    from flare_b200 import optim
    from flare_b200.dp import GradBuffer
    n = 50
    t = list(_reference_tuple(n, legacy=True))
    params = t[:15]
    state = {g: {"step": torch.tensor(5.0), "exp_avg": torch.full_like(p, float(g + 1)),
                 "exp_avg_sq": torch.full_like(p, float(g + 101))} for g, p in enumerate(params)}
    t[15] = {"state": state, "param_groups": []}
    tens = checkpoint.tensors_from_tuple(tuple(t))
    sc = checkpoint.scene_from_tensors(tens)
    opt = optim.ModelOptimizer(sc, GradBuffer(n, True, "cpu"))
    checkpoint.restore_optimizer(opt, tens)
    segs = {s.name: i for i, s in enumerate(opt.adam.segments)}
    assert opt.adam.t == 5
    for g, name in enumerate(checkpoint.GROUP_SEGMENTS[1:]):
        m, v = opt.adam.state[segs[name]]
        assert torch.all(m == g + 1) and torch.all(v == g + 101), name
    m_rgb, _ = opt.adam.state[segs["RGB"]]
    assert torch.all(m_rgb == 0)


def test_optimizer_state_of_the_wrong_size_is_rejected():
    from flare_b200 import optim
    from flare_b200.dp import GradBuffer
    t = list(_reference_tuple(50))
    t[16] = {"state": {0: {"step": torch.tensor(1.0), "exp_avg": torch.zeros(49, 3), "exp_avg_sq": torch.zeros(49, 3)}},
             "param_groups": []}
    tens = checkpoint.tensors_from_tuple(tuple(t))
    opt = optim.ModelOptimizer(checkpoint.scene_from_tensors(tens), GradBuffer(50, True, "cpu"))
    with pytest.raises(ValueError):
        checkpoint.restore_optimizer(opt, tens)
