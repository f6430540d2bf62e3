"""Optimizer step: the per-group learning-rate schedule, the fragment-layout un-permutation of the decoder
weight gradients (CPU), and the fused Adam launch against torch.optim.Adam (GPU)."""
import math

import pytest
import torch

from flare_b200 import optim


def test_lr_schedule_decays_to_floor_and_grows_to_ceiling():
    assert optim.lr_at(0.01, -0.001, 0.001, 0) == 0.01
    assert math.isclose(optim.lr_at(0.01, -0.001, 0.001, 1000), 0.01 * math.exp(-1.0))
    assert optim.lr_at(0.01, -0.001, 0.001, 100000) == 0.001            # floor
    assert optim.lr_at(0.001, 0.001, 0.005, 100000) == 0.005            # ceiling when the coefficient grows
    lrs = {k: optim.lr_at(*v, 30000) for k, v in optim.REFERENCE_LR.items()}
    assert len(lrs) == 16 and all(x > 0 for x in lrs.values())


def _pack(W, b, rows, cols, bias_entries):
    """The renderer's fragment layout (pack_dw_kernel, train.py:754-790 inverse): weights at
    ((i*J + j)*64 + c*32 + lane) <- W[8i + lane/4][8j + 2(lane%4) + c]; bias b[8j + lane/4] at c = 0,
    lane%4 = 0."""
    J = cols // 8
    fw = torch.zeros(rows * cols)
    for t in range(rows * cols):
        lane, c, ij = t & 31, (t >> 5) & 1, t >> 6
        fw[t] = W[8 * (ij // J) + (lane >> 2), 8 * (ij % J) + 2 * (lane & 3) + c]
    fb = torch.zeros(bias_entries)
    for t in range(bias_entries):
        lane, c, j = t & 31, (t >> 5) & 1, t >> 6
        if c == 0 and lane % 4 == 0 and 8 * j + lane // 4 < b.numel():
            fb[t] = b[8 * j + lane // 4]
    return fw.reshape(1, -1), fb.reshape(1, -1)


def test_dense_decoder_grads_inverts_the_fragment_layout():
    g = torch.Generator().manual_seed(3)
    W1, W2, W3 = torch.randn(64, 128, generator=g), torch.randn(64, 64, generator=g), torch.randn(8, 64, generator=g)
    b1, b2, b3 = torch.randn(64, generator=g), torch.randn(64, generator=g), torch.randn(8, generator=g)
    G = {}
    G["w1"], G["b1"] = _pack(W1, b1, 64, 128, 512)
    G["w2"], G["b2"] = _pack(W2, b2, 64, 64, 512)
    G["w3"], G["b3"] = _pack(W3, b3, 8, 64, 64)
    d = optim.dense_decoder_grads(G)
    assert torch.equal(d["w1"], W1) and torch.equal(d["w2"], W2) and torch.equal(d["w3"][:8], W3)
    assert torch.equal(d["b1"], b1) and torch.equal(d["b2"], b2) and torch.equal(d["b3"][:8], b3)
    assert not d["w3"][8:].any() and not d["b3"][8:].any()


@pytest.mark.gpu
def test_fused_adam_matches_torch_adam():
    """Strided blocks (RGB / A of one (N,4) tensor, three column blocks of W1), an fp16 mirror and the
    scale regulariser, three steps with changing gradients and learning rates."""
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(7)
    n = 5000
    RGBA = torch.randn(n, 4, device=dev, generator=g)
    W1 = torch.randn(64, 128, device=dev, generator=g) * 0.1
    W1h = W1.half()
    s = torch.randn(n, 2, device=dev, generator=g) - 3.0
    feat = torch.randn(13154, device=dev, generator=g)
    gRGB, gA = torch.zeros(n, 3, device=dev), torch.zeros(n, 1, device=dev)
    gW = {k: torch.zeros(64, w, device=dev) for k, w in (("uv", 8), ("v", 24), ("c", 96))}
    gs, gf = torch.zeros(n, 2, device=dev), torch.zeros(13154, device=dev)
    lam = 0.001 / n
    S = optim.Segment
    ours = optim.FusedAdam([S("RGB", RGBA, gRGB, 3, 0), S("A", RGBA, gA, 1, 3), S("uv", W1, gW["uv"], 8, 0, W1h),
                            S("v", W1, gW["v"], 24, 8, W1h), S("c", W1, gW["c"], 96, 32, W1h),
                            S("s", s, gs, 2, 0, None, lam), S("f", feat, gf, 13154)])
    ref = {"RGB": RGBA[:, :3].clone().requires_grad_(), "A": RGBA[:, 3:].clone().requires_grad_(),
           "uv": W1[:, :8].clone().requires_grad_(), "v": W1[:, 8:32].clone().requires_grad_(),
           "c": W1[:, 32:].clone().requires_grad_(), "s": s.clone().requires_grad_(), "f": feat.clone().requires_grad_()}
    lr0 = {"RGB": 0.005, "A": 0.05, "uv": 0.0125, "v": 0.03, "c": 0.0015, "s": 0.04, "f": 0.005}
    opt = torch.optim.Adam([{"params": [ref[k]], "lr": lr0[k]} for k in ref])
    for it in range(3):
        grads = {"RGB": gRGB, "A": gA, "uv": gW["uv"], "v": gW["v"], "c": gW["c"], "s": gs, "f": gf}
        for k, t in grads.items():
            t.copy_(torch.randn(t.shape, device=dev, generator=g) * (0.1 + it))
        lrs = {k: lr0[k] * (0.9 ** it) for k in lr0}
        for grp, k in zip(opt.param_groups, ref):
            grp["lr"] = lrs[k]
            gr = grads[k].clone()
            if k == "s":
                s2 = torch.exp(ref["s"].detach()) ** 2
                gr = gr + lam * (s2 / torch.sqrt(s2.sum(1, keepdim=True)))
            ref[k].grad = gr
        opt.step()
        ours.step(lrs)
    tol = dict(rtol=2e-5, atol=2e-7)
    torch.testing.assert_close(RGBA[:, :3], ref["RGB"].detach(), **tol)
    torch.testing.assert_close(RGBA[:, 3:], ref["A"].detach(), **tol)
    torch.testing.assert_close(W1, torch.cat([ref["uv"], ref["v"], ref["c"]], 1).detach(), **tol)
    torch.testing.assert_close(s, ref["s"].detach(), **tol)
    torch.testing.assert_close(feat, ref["f"].detach(), **tol)
    assert torch.equal(W1h, W1.half())


@pytest.mark.gpu
def test_training_step_with_optimizer_updates_the_scene():
    """TrainStep + ModelOptimizer: every group moves, the renderer's fp16 tensors follow their fp32
    masters, and the loss drops over a few steps at fixed rays."""
    from flare_b200.dp import Shard, TrainStep
    from flare_b200.renderer import CPyOptiXFLARERenderer
    from flare_b200.scene import camera_rays, make_scene
    sc = make_scene(20000, 9).to("cuda")
    O, v = camera_rays(48, 48, 60.0, eye=(0.0, 0.0, 3.0))
    tgt = torch.rand(O.shape[0], 3, generator=torch.Generator().manual_seed(1))
    r = CPyOptiXFLARERenderer(8, 11.3449, O.shape[0])
    st = TrainStep(r, sc, [Shard(O.cuda(), v.cuda(), tgt.cuda())], O.shape[0])
    before = {k: getattr(sc, k).clone() for k in ("m", "s", "q", "RGBA", "k", "cond", "features", "A1", "b1")}
    opt = optim.ModelOptimizer(sc, st.grads)
    losses = []
    for it in range(1, 6):
        losses.append(float(st()))
        opt.step(it)
    for k, t in before.items():
        assert not torch.equal(getattr(sc, k), t), k
    assert torch.equal(sc.cond, opt.cond32.half()) and torch.equal(sc.A1, opt.W1.half())
    assert losses[-1] < losses[0], losses
