"""Densification / pruning: the one-launch rebuild against a direct tensor restatement of the reference's
mask / index / cat sequence (train.py:955-1240), and a training loop running through it (GPU)."""
import math

import pytest
import torch

from flare_b200 import densify, optim

pytestmark = pytest.mark.gpu


def _reference(P, S, m_before, mb_state, p, extent):
    """P: name -> tensor (m, s, q, RGB, A, k, cond), S: name -> (exp_avg, exp_avg_sq)."""
    kf = 1.0 + torch.nn.functional.softplus(P["k"])
    Af = torch.sigmoid(P["A"])
    scale = torch.clamp(kf * (11.3449 + 2.0 * torch.log(Af)), min=0.0) ** (1.0 / (2.0 * kf)) / math.sqrt(11.3449)
    s_norm = torch.sqrt((torch.exp(P["s"]) ** 2).sum(1)) * scale.squeeze(1)
    keep = (P["A"] >= math.log(p.opacity_threshold / (1 - p.opacity_threshold))).squeeze(1) & (s_norm >= p.min_s_norm)
    d = P["m"][keep] - m_before[keep]
    dens = (torch.sqrt((d * d).sum(1, keepdim=True)) >= p.mu_threshold).squeeze(1)
    out = {}
    for name, x in list(P.items()) + [(f"{n}.avg", S[n][0]) for n in S] + [(f"{n}.sq", S[n][1]) for n in S]:
        xp = x[keep]
        first = xp[dens]
        if name == "m":
            first = m_before[keep][dens]
        elif name == "m.avg":
            first = mb_state[0][keep][dens]
        elif name == "m.sq":
            first = mb_state[1][keep][dens]
        out[name] = torch.cat([xp[~dens], first, xp[dens]], 0)
    out["s"] = out["s"].clamp(min=math.log(p.min_s_coef), max=math.log(p.max_s_coef * extent / 2))
    out["RGB"] = out["RGB"].clamp(min=0.0)
    return out


def test_densify_matches_reference_restatement():
    from flare_b200.dp import GradBuffer
    from flare_b200.scene import make_scene
    torch.manual_seed(0)
    sc = make_scene(6000, 2).to("cuda")
    n = sc.n
    sc.RGBA[:, 3] = torch.randn(n, device="cuda") * 3.0          # some below the opacity threshold
    sc.s[:200] = -12.0                                           # some below the support threshold
    grads = GradBuffer(n, True, "cuda")
    opt = optim.ModelOptimizer(sc, grads)
    for st in opt.adam.state:
        st[0].normal_()
        st[1].uniform_()
    before = densify.snapshot_before_step(opt)
    sc.m.add_(torch.randn(n, 3, device="cuda") * 0.0015)          # the step moved some centres past 1e-3
    p = densify.DensifyParams()
    names = {s.name: i for i, s in enumerate(opt.adam.segments)}
    P = {"m": sc.m.clone(), "s": sc.s.clone(), "q": sc.q.clone(), "RGB": sc.RGBA[:, :3].clone(),
         "A": sc.RGBA[:, 3:].clone(), "k": sc.k.clone(), "cond": opt.cond32.clone()}
    S = {"m": opt.adam.state[names["m"]], "s": opt.adam.state[names["s"]], "q": opt.adam.state[names["q"]],
         "RGB": opt.adam.state[names["RGB"]], "A": opt.adam.state[names["A"]], "k": opt.adam.state[names["k"]],
         "cond": opt.adam.state[names["conditioning"]]}
    S = {k: (a.clone(), b.clone()) for k, (a, b) in S.items()}
    ref = _reference(P, S, before[0], before[1:], p, extent=3.4)
    n_orig, n_split = densify.densify_and_prune(opt, before, extent=3.4, p=p)
    assert n_split > 0 and n_orig + n_split < n
    assert sc.n == n_orig + 2 * n_split == ref["m"].shape[0]
    got = {"m": sc.m, "s": sc.s, "q": sc.q, "RGB": sc.RGBA[:, :3], "A": sc.RGBA[:, 3:], "k": sc.k,
           "cond": opt.cond32}
    names = {s.name: i for i, s in enumerate(opt.adam.segments)}
    for k_, g in got.items():
        assert torch.equal(g, ref[k_]), k_
    for k_, seg in (("m", "m"), ("s", "s"), ("q", "q"), ("RGB", "RGB"), ("A", "A"), ("k", "k"), ("cond", "conditioning")):
        a, b = opt.adam.state[names[seg]]
        assert torch.equal(a.reshape(ref[k_ + ".avg"].shape), ref[k_ + ".avg"]), k_
        assert torch.equal(b.reshape(ref[k_ + ".sq"].shape), ref[k_ + ".sq"]), k_
    assert torch.equal(sc.cond, opt.cond32.half())
    assert opt.grads["m"].shape[0] == sc.n


def test_training_loop_through_densification():
    from flare_b200.dp import Shard, TrainStep
    from flare_b200.renderer import CPyOptiXFLARERenderer
    from flare_b200.scene import camera_rays, make_scene
    sc = make_scene(20000, 9).to("cuda")
    O, v = camera_rays(48, 48, 60.0, eye=(0.0, 0.0, 3.0))
    tgt = torch.rand(O.shape[0], 3, generator=torch.Generator().manual_seed(1))
    r = CPyOptiXFLARERenderer(8, 11.3449, O.shape[0])
    st = TrainStep(r, sc, [Shard(O.cuda(), v.cuda(), tgt.cuda())], O.shape[0])
    opt = optim.ModelOptimizer(sc, st.grads)
    losses = []
    for it in range(1, 9):
        losses.append(float(st()))
        before = densify.snapshot_before_step(opt) if it == 4 else None
        opt.step(it)
        if before is not None:
            n0 = sc.n
            densify.densify_and_prune(opt, before, extent=3.4, p=densify.DensifyParams(mu_threshold=1e-5))
            assert sc.n != n0
            st.rebind(sc, opt.grads)
    assert all(math.isfinite(x) for x in losses) and losses[-1] < losses[0], losses
