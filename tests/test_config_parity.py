"""Parity at the benchmarked sizes: BASELINE configs 1-3 (1M / 3M / 6M primitives, full cameras) rendered
whole on the GPU, checked against the CPU oracle on a fixed seeded sample of their rays.

For each config the GPU renders the whole image (every ray, so traversal runs under full-size
contention: the persistent heap kernel for large passes, the warp-per-ray kernel for the sparse tail).
Then, for the sampled rays:
  * hit lists: every traversal pass the GPU ran (read back from the renderer's hit cache) is, bit for bit,
    the next run of the oracle's full (t, index)-sorted hit sequence (one brute-force sweep over all
    primitives per sampled ray): a full pass the next 42 hits, then a restart at nextafter(t_42); a bounded
    pass possibly fewer -- no hit skipped or repeated;
  * forward: RGB, depth / normal accumulators (training) and RGB / normal / alpha / expected depth
    (inference with geometry, config 1 at the config's T_threshold 1e-4) within 1e-3 of the oracle's
    compositing over the reference's 16-slot passes;
  * backward (configs 2 and 3): dL/dI is nonzero on the sampled rays only, so the whole-image Backward
    (which replays the cached forward passes) must give the oracle's gradients over those rays: every
    gradient within 1e-3 relative L2, and exactly zero on primitives no sampled ray composited.
The sample: a central 16 x 16 block plus 256 uniformly drawn rays (seed 7).
"""
import numpy as np
import pytest
import torch

from flare_b200.scene import camera_rays, make_scene, sphere_eye
from oracle import grad_oracle, oracle

pytestmark = pytest.mark.gpu
RGB_TOL = 1e-3
GRAD_TOL = 1e-3
T_NEAR, T_FAR = 0.1, 1000.0
REG_A = -(T_NEAR * T_FAR) / (T_FAR - T_NEAR)
REG_B = T_FAR / (T_FAR - T_NEAR)
PASS_SLOTS = 42
CONFIGS = {1: (1_000_000, 800, 800, (0.0, 0.0, 3.0)), 2: (3_000_000, 1600, 1064, (0.0, 0.0, 3.0)),
           3: (6_000_000, 1920, 1080, sphere_eye(0, 8))}


def z(*s):
    return torch.zeros(*s, device="cuda")


def _sample(W, H, seed=7):
    cy, cx = H // 2, W // 2
    block = [(cy - 8 + dy) * W + (cx - 8 + dx) for dy in range(16) for dx in range(16)]
    rnd = np.random.RandomState(seed).choice(W * H, 256, replace=False)
    return np.unique(np.concatenate([np.array(block), rnd])).astype(np.int64)


class Full:
    def __init__(self, cfg):
        from flare_b200.renderer import CPyOptiXFLARERenderer
        n, W, H, eye = CONFIGS[cfg]
        self.cfg = cfg
        self.sc = make_scene(n, 0)
        self.g = self.sc.to("cuda")
        self.O, self.v = camera_rays(W, H, 60.0, eye=eye)
        self.R = W * H
        self.Og, self.vg = self.O.cuda(), self.v.cuda()
        self.r = CPyOptiXFLARERenderer(8, 11.3449, self.R)
        self.r.SetGeometry(*[t.contiguous() for t in self.g.activated()])
        self.S = _sample(W, H)
        frames = self.r.frames().cpu().numpy()
        self.hits = oracle.all_hits(frames, self.O[self.S], self.v[self.S])
        self.csr16 = oracle.csr_from_passes([oracle.restart_passes(t, i, 16) for t, i in self.hits])

    def dec(self):
        g = self.g
        return (g.cond, g.features, g.A1, g.b1, g.A2, g.b2, g.A3, g.b3)

    def geo(self):
        g = self.g
        return (g.m, g.s, g.q, g.RGBA, g.k)

    def forward_training(self, bg, sn):
        R = self.R
        out = None
        for _ in range(2):  # the first forward on a renderer sizes the hit cache, the second fills it
            out = (z(R, 3), z(R, 4), z(R, 4), z(R, 2))
            self.r.Forward_training(*self.dec(), self.Og, self.vg, out[0], *bg, *self.geo(), 1e-4, out[1], REG_A,
                                    REG_B, out[3], sn, out[2])
        return out


@pytest.fixture(scope="module", params=[1, 2, 3])
def full(request):
    f = Full(request.param)
    yield f
    del f.r
    torch.cuda.empty_cache()


def test_pass_hit_lists_bit_exact(full):
    """Every traversal pass the GPU ran, for every sampled ray, is the next run of the oracle's (t, index)-
    sorted hit sequence: a full pass holds exactly the next 42 hits (the K nearest beyond its start), and the
    following pass starts right after them (hits tied with the 42nd at its t are skipped, the restart rule); a
    pass that ran under a bound may hold fewer, and the next one continues where it stopped.  So each pass's
    hits are checked bit for bit and no hit of the sequence is skipped or repeated, whatever bounds the
    renderer chose for its passes."""
    f = full
    bg = (0.0, 0.0, 0.0)
    f.forward_training(bg, z(f.R, 3))
    passes = f.r.pass_hits()
    assert len(passes) >= 2
    where = {int(r): j for j, r in enumerate(f.S)}
    pos = np.zeros(len(f.S), np.int64)
    seen = np.zeros(len(f.S), np.int64)
    multi = short = 0
    for p, (ids, t, idx) in enumerate(passes):
        ids = ids.cpu().numpy()
        sel = np.nonzero(np.isin(ids, f.S))[0]
        t, idx = t[:, sel].cpu().numpy(), idx[:, sel].cpu().numpy()
        for col, rid in zip(range(len(sel)), ids[sel]):
            j = where[int(rid)]
            assert seen[j] == p, f"ray {rid} skipped a pass"
            st, si = f.hits[j]
            n = int((idx[:, col] >= 0).sum())
            assert (idx[n:, col] == -1).all() and np.isinf(t[n:, col]).all()
            a = pos[j]
            assert np.array_equal(idx[:n, col], si[a:a + n]) and np.array_equal(t[:n, col], st[a:a + n]), \
                f"config {f.cfg} pass {p} ray {rid}"
            a += n
            if n == PASS_SLOTS:  # restart at nextafter(t_42): ties with the 42nd hit are skipped
                while a < len(st) and st[a] == t[n - 1, col]:
                    a += 1
            else:
                short += 1
            pos[j] = a
            seen[j] += 1
            multi += p >= 2
    assert seen.min() >= 1
    print(f"config {f.cfg}: {len(passes)} passes, sampled rays over {seen.sum()} ray-passes, {multi} in pass >= 3, "
          f"{short} short passes")


def test_forward_training_on_sample(full):
    f = full
    bg = (0.1, 0.2, 0.3)
    sn = torch.nn.functional.normalize(torch.randn(f.R, 3, generator=torch.Generator().manual_seed(3)), dim=1)
    bitmap, dacc, nacc, _ = f.forward_training(bg, sn.cuda())
    S = f.S
    ref = oracle.forward(f.sc, f.O[S], f.v[S], f.csr16, "training", bg=bg, T_thr=1e-4, reg_a=REG_A, reg_b=REG_B,
                         surface_normal=sn[S].numpy())
    assert np.abs(bitmap[S].cpu().numpy() - ref["rgb"]).max() < RGB_TOL
    d = dacc[S].cpu().numpy()
    assert np.abs(d - ref["dacc"]).max() < RGB_TOL * max(1.0, np.abs(ref["dacc"]).max())
    assert np.abs(nacc[S].cpu().numpy() - ref["nacc"]).max() < RGB_TOL
    assert ref["nhits"].mean() > 10


def test_forward_inference_geometry_on_sample(full):
    """Config 1 is BASELINE's forward-render workload: Forward_inference_with_geometry at T_thr 1e-4."""
    f = full
    R, S = f.R, f.S
    bitmap, normal, alpha, edn = z(R, 3), z(R, 3), z(R), z(R)
    f.r.Forward_inference_with_geometry(*f.dec(), f.Og, f.vg, bitmap, normal, alpha, edn, 0.0, 0.0, 0.0, *f.geo(),
                                        1e-4)
    ref = oracle.forward(f.sc, f.O[S], f.v[S], f.csr16, "geometry", T_thr=1e-4)
    assert np.abs(bitmap[S].cpu().numpy() - ref["rgb"]).max() < RGB_TOL
    assert np.abs(alpha[S].cpu().numpy() - ref["alpha"]).max() < RGB_TOL
    assert np.abs(normal[S].cpu().numpy() - ref["normal"]).max() < RGB_TOL
    e = edn[S].cpu().numpy()
    assert np.abs(e - ref["edn"]).max() < RGB_TOL * max(1.0, np.abs(ref["edn"]).max())


def test_backward_on_sample(full):
    f = full
    if f.cfg == 1:
        pytest.skip("config 1 is the forward-only workload")
    R, S, n = f.R, f.S, f.sc.n
    bg = (0.1, 0.2, 0.3)
    sn = z(R, 3)
    bitmap, dacc, nacc, dai = f.forward_training(bg, sn)
    dLdI = torch.zeros(R, 3)
    dLdI[S] = torch.randn(len(S), 3, generator=torch.Generator().manual_seed(5)) / len(S)
    G = dict(RGB=z(n, 3), A=z(n, 1), k=z(n, 1), m=z(n, 3), s=z(n, 2), q=z(n, 4), cond=z(n, 96), features=z(13154))
    W = dict(w3=z(1, 512), b3=z(1, 64), w2=z(1, 4096), b2=z(1, 512), w1=z(1, 8192), b1=z(1, 512))
    f.r.Backward(*f.dec(), f.Og, f.vg, *bg, *f.geo(), bitmap.clone(), dLdI.cuda(), G["RGB"], G["A"], G["k"], W["w3"],
                 W["b3"], W["w2"], W["b2"], W["w1"], W["b1"], G["cond"], G["features"], G["m"], G["s"], G["q"], 1e-4,
                 dacc, z(R, 4), 0.0, REG_A, REG_B, dai, sn, nacc, 0.0)
    st = f.r.stats()
    assert st["passes"] >= 3, st  # the replayed forward had at least three passes
    ref = oracle.forward(f.sc, f.O[S], f.v[S], f.csr16, "training", bg=bg, T_thr=1e-4, reg_a=REG_A, reg_b=REG_B)
    gr = grad_oracle.gradients(f.sc, f.O[S], f.v[S], f.csr16, ref["nhits"], dLdI[S].numpy(), bg=bg, compact=True)
    off, _, ii = f.csr16
    ray = np.repeat(np.arange(len(S)), ref["nhits"])
    pos = np.concatenate([np.arange(k) for k in ref["nhits"]])
    used = np.unique(ii[off[:-1][ray] + pos])
    from test_gpu_parity import unpack_weight_grads
    w1, b1, w2, b2, w3, b3 = unpack_weight_grads(*(W[k].cpu() for k in ("w1", "b1", "w2", "b2", "w3", "b3")))
    got = {k: G[k].cpu().numpy() for k in G}
    mask = np.ones(n, bool)
    mask[used] = False
    bad = {}
    for k in ("RGB", "A", "k", "m", "s", "q", "cond"):
        e = grad_oracle.rel_l2(got[k][used], gr[k].numpy())
        if not e < GRAD_TOL:
            bad[k] = e
        assert not got[k][mask].any(), f"{k}: gradient on primitives no sampled ray composited"
    for k, x in (("features", got["features"]), ("A1", w1.numpy()), ("b1", b1.numpy()), ("A2", w2.numpy()),
                 ("b2", b2.numpy()), ("A3", w3.numpy()[:4]), ("b3", b3.numpy()[:4])):
        o = gr[k].numpy()
        e = grad_oracle.rel_l2(x, o[:4] if k in ("A3", "b3") else o)
        if not e < GRAD_TOL:
            bad[k] = e
    assert not bad, f"config {f.cfg} relative L2 above {GRAD_TOL}: {bad}"


def test_config4_secondary_rays_on_sample():
    """BASELINE config 4 (1M primitives + mirror / glass spheres, 1024 x 1024, recursion depth 3): the whole
    image on the GPU, 128 sampled primary rays (each with its own tree of reflected / refracted rays)
    through the oracle's viewer restatement."""
    from flare_b200.scene import viewer_lights, viewer_spheres
    from flare_b200.viewer import CPyFlareViewerRenderer
    from oracle import viewer_oracle
    W = 1024
    sc = make_scene(1_000_000, 0)
    g = sc.to("cuda")
    O, v = camera_rays(W, W, 60.0, eye=(0.0, 0.0, 3.0))
    R = W * W
    r = CPyFlareViewerRenderer(8, 11.3449, R, 3)
    sph, mat = viewer_spheres()
    lts = viewer_lights()
    r.SetGeometry(*[t.contiguous() for t in g.activated()], sph)
    bm = z(R, 3)
    r.Forward(g.cond, g.features, g.RGBA[:, :3].contiguous(), g.A1, g.b1, g.A2, g.b2, g.A3, g.b3, O.cuda(), v.cuda(),
              bm, 0.0, 0.0, 0.0, g.m, g.s, g.q, g.RGBA[:, 3].contiguous(), g.k, 0.01, mat, lts, 1e-4, 0.55, 0.06, 0.06,
              0.07)
    frames = r.frames().cpu().numpy()
    # 64 rays through the spheres' screen region (centre-left / centre-right / upper centre) + 64 random
    rs = np.random.RandomState(11)
    ys = np.concatenate([rs.randint(400, 624, 64), rs.randint(0, W, 64)])
    xs = np.concatenate([rs.randint(250, 774, 64), rs.randint(0, W, 64)])
    S = np.unique(ys * W + xs)
    ref, st = viewer_oracle.viewer_forward(frames, sc.__dict__, sph.numpy(), mat.numpy(), lts.numpy(), O[S], v[S],
                                           bg=(0.0, 0.0, 0.0), T_thr=0.01, eps=1e-4, shadow_mult=0.55,
                                           Ia=(0.06, 0.06, 0.07), max_depth=3)
    got = bm[S].cpu().numpy()
    err = np.abs(got - ref).max(axis=1)
    assert st["generations"] > 3
    assert err.max() < RGB_TOL, ((err > RGB_TOL).sum(), err.max())
