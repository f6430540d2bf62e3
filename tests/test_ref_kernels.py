"""Parity against the reference renderer's OWN compiled kernels (oracle/_ref, built by oracle/Makefile.ref
from the reference sources; driven pass by pass by oracle/ref_kernels.py with the oracle's hit lists in
place of the closed OptiX traversal).

What this pins: the reference's decode / composite / regulariser / backward arithmetic (LUT, positional
encoding, mma.sync MLP, compositing, depth / normal accumulators, median depth, every gradient and the
per-warp weight-gradient layout) against both this package's kernels and the CPU oracle.

Bars (from the task): RGB / accumulators within 1e-3 max absolute error; median-depth index bit-exact;
gradients within 1e-3 relative L2.  The reference's backward runs its MLP backward with bf16 tensor-core
operands (Backward.cu:761-1294), which moves the gradients that pass through it (geometry m/s/q, the
descriptor, the LUT and the MLP weights of the decoder path) 1e-3 .. 7e-3 relative L2 away from the exact
gradient; for those, the bar is REF_BF16_TOL against the reference together with being at least as close
to the float64 autograd oracle as the reference is.
"""
import numpy as np
import pytest
import torch

from oracle import grad_oracle, oracle, ref_kernels
from test_gpu_parity import REG_A, REG_B, Case, _surface_normals, unpack_weight_grads

pytestmark = pytest.mark.gpu
RGB_TOL = 1e-3
GRAD_TOL = 1e-3
REF_BF16_TOL = 1e-2
BF16_PATH = ("m", "s", "q", "cond", "features", "A1", "b1", "A2", "b2", "A3")


def z(*s):
    return torch.zeros(*s, device="cuda")


@pytest.fixture(scope="module", params=["case0", "dense"])
def case(request):
    if not ref_kernels.available():
        pytest.skip("oracle/_ref not built (needs the reference sources: make -f oracle/Makefile.ref)")
    if request.param == "case0":
        c = Case(10000, 64, seed=0)
    else:
        c = Case(200000, 32, seed=1, eye=(0.0, 0.0, 1.8), fov=40.0)
    c.ref = ref_kernels.RefRenderer(c.g, c.Og, c.vg, c.csr)
    return c


def _maxabs(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max())


@pytest.mark.parametrize("base", [True, False])
def test_forward_training_matches_reference(case, base):
    c, R = case, case.R
    bg = (0.1, 0.2, 0.3)
    sn = _surface_normals(R).cuda()
    b1, d1, n1, a1 = z(R, 3), z(R, 4), z(R, 4), z(R, 2)
    c.ref.forward_training(base, b1, bg, 1e-4, d1, REG_A, REG_B, a1, sn, n1)
    b2, d2, n2, a2 = z(R, 3), z(R, 4), z(R, 4), z(R, 2)
    args = (c.Og, c.vg, b2, *bg, *c.geo(), 1e-4, d2, REG_A, REG_B, a2, sn, n2)
    c.r.Forward_training_base(*args) if base else c.r.Forward_training(*c.dec(), *args)
    orc = oracle.forward(c.sc, c.O, c.v, c.csr, "training", base=base, bg=bg, T_thr=1e-4, reg_a=REG_A, reg_b=REG_B,
                         surface_normal=sn.cpu().numpy())
    b1, d1, n1 = b1.cpu().numpy(), d1.cpu().numpy(), n1.cpu().numpy()
    assert c.ref.passes >= 2
    assert _maxabs(b2.cpu(), b1) < RGB_TOL, "ours vs reference"
    assert _maxabs(orc["rgb"], b1) < RGB_TOL, "oracle vs reference"
    assert _maxabs(d2.cpu(), d1) < RGB_TOL * max(1.0, np.abs(d1).max())
    assert _maxabs(orc["dacc"], d1) < RGB_TOL * max(1.0, np.abs(d1).max())
    assert _maxabs(n2.cpu(), n1) < RGB_TOL and _maxabs(orc["nacc"], n1) < RGB_TOL


@pytest.mark.parametrize("base", [True, False])
def test_forward_inference_geometry_matches_reference(case, base):
    c, R = case, case.R
    bg = (0.3, 0.1, 0.0)
    outs = []
    for who in ("ref", "ours"):
        b, nrm, al, ed = z(R, 3), z(R, 3), z(R), z(R)
        if who == "ref":
            c.ref.forward_inference(base, b, nrm, al, ed, bg, 1e-4)
        elif base:
            c.r.Forward_inference_base_with_geometry(c.Og, c.vg, b, nrm, al, ed, *bg, *c.geo(), 1e-4)
        else:
            c.r.Forward_inference_with_geometry(*c.dec(), c.Og, c.vg, b, nrm, al, ed, *bg, *c.geo(), 1e-4)
        outs.append([x.cpu().numpy() for x in (b, nrm, al, ed)])
    for k, (x_ref, x_our) in enumerate(zip(*outs)):
        scale = max(1.0, np.abs(x_ref).max()) if k == 3 else 1.0
        assert _maxabs(x_our, x_ref) < RGB_TOL * scale, ("rgb", "normal", "alpha", "edn")[k]


def test_forward_pca_matches_reference(case):
    c, R = case, case.R
    oc = torch.rand(c.sc.n, 3, generator=torch.Generator().manual_seed(9)).cuda()
    b1, b2 = z(R, 3), z(R, 3)
    c.ref.forward_inference(False, b1, None, None, None, (0.1, 0.2, 0.3), 1e-4, override_colors=oc)
    c.r.Forward_pca(*c.dec(), oc, c.Og, c.vg, b2, 0.1, 0.2, 0.3, *c.geo(), 1e-4)
    assert _maxabs(b2.cpu(), b1.cpu()) < RGB_TOL


@pytest.mark.parametrize("base", [True, False])
def test_median_depth_index_bit_exact_vs_reference(case, base):
    c, R = case, case.R
    d1, d2 = z(R, 2), z(R, 2)
    c.ref.median_depth(base, 1e-4, d1)
    c.r.GetMedianDepth_base(c.Og, c.vg, *c.geo(), 1e-4, d2) if base else \
        c.r.GetMedianDepth(*c.dec(), c.Og, c.vg, *c.geo(), 1e-4, d2)
    d1, d2 = d1.cpu().numpy(), d2.cpu().numpy()
    assert np.array_equal(d1[:, 1].view(np.int32), d2[:, 1].view(np.int32))
    assert np.array_equal(d1[:, 0], d2[:, 0])
    assert (d1[:, 1].view(np.int32) > 0).sum() > 10


@pytest.mark.parametrize("base", [True, False])
@pytest.mark.parametrize("lam", [0.0, 1e-3])
def test_backward_matches_reference(case, base, lam):
    c, R, n = case, case.R, case.sc.n
    bg = (0.1, 0.2, 0.3)
    sn = _surface_normals(R, 11).cuda()
    fw = []
    for who in ("ref", "ours"):
        b, d, nn, a = z(R, 3), z(R, 4), z(R, 4), z(R, 2)
        if who == "ref":
            c.ref.forward_training(base, b, bg, 1e-4, d, REG_A, REG_B, a, sn, nn)
        else:
            args = (c.Og, c.vg, b, *bg, *c.geo(), 1e-4, d, REG_A, REG_B, a, sn, nn)
            c.r.Forward_training_base(*args) if base else c.r.Forward_training(*c.dec(), *args)
        fw.append((b, d, nn, a))
    dLdI = (torch.randn(R, 3, generator=torch.Generator().manual_seed(11)) / R).cuda()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    G = [dict(RGB=z(n, 3), A=z(n, 1), k=z(n, 1), m=z(n, 3), s=z(n, 2), q=z(n, 4), cond=z(n, 96),
              features=z(13154)) for _ in range(2)]
    W = [dict(w3=z(4 * sms, 512), b3=z(4 * sms, 64), w2=z(4 * sms, 4096), b2=z(4 * sms, 512),
              w1=z(4 * sms, 8192), b1=z(4 * sms, 512)) for _ in range(2)]
    b, d, nn, a = fw[0]
    c.ref.backward(base, bg, b.clone(), dLdI, G[0], W[0], 1e-4, d, z(R, 4), lam, REG_A, REG_B, a, sn, nn, lam)
    b, d, nn, a = fw[1]
    g, w = G[1], W[1]
    if base:
        c.r.Backward_base(c.Og, c.vg, *bg, *c.geo(), b.clone(), dLdI, g["RGB"], g["A"], g["k"], g["m"], g["s"], g["q"],
                          1e-4, d, z(R, 4), lam, REG_A, REG_B, a, sn, nn, lam)
    else:
        c.r.Backward(*c.dec(), c.Og, c.vg, *bg, *c.geo(), b.clone(), dLdI, g["RGB"], g["A"], g["k"], w["w3"], w["b3"],
                     w["w2"], w["b2"], w["w1"], w["b1"], g["cond"], g["features"], g["m"], g["s"], g["q"], 1e-4, d,
                     z(R, 4), lam, REG_A, REG_B, a, sn, nn, lam)
    orc_f = oracle.forward(c.sc, c.O, c.v, c.csr, "training", base=base, bg=bg, T_thr=1e-4, reg_a=REG_A,
                           reg_b=REG_B, surface_normal=sn.cpu().numpy())
    gr = grad_oracle.gradients(c.sc, c.O, c.v, c.csr, orc_f["nhits"], dLdI.cpu().numpy(), base=base, bg=bg,
                               reg_a=REG_A, reg_b=REG_B, lambda_depth=lam, lambda_normal=lam,
                               surface_normal=sn.cpu().numpy())
    got = [{k: v.cpu().numpy() for k, v in gg.items()} for gg in G]
    keys = ["RGB", "A", "k", "m", "s", "q"]
    if not base:
        keys += ["cond", "features", "A1", "b1", "A2", "b2", "A3", "b3"]
        for gg, ww in zip(got, W):
            u = unpack_weight_grads(*(ww[k].cpu() for k in ("w1", "b1", "w2", "b2", "w3", "b3")))
            gg.update({nm: x.numpy() for nm, x in zip(("A1", "b1", "A2", "b2", "A3", "b3"), u)})
            gg["A3"], gg["b3"] = gg["A3"][:4], gg["b3"][:4]
        gr["A3"], gr["b3"] = gr["A3"][:4], gr["b3"][:4]
    report, bad = {}, {}
    for k in keys:
        ref_, our = got[0][k], got[1][k]
        e_or = grad_oracle.rel_l2(our, ref_)
        e_ro = grad_oracle.rel_l2(ref_, gr[k].numpy())
        e_oo = grad_oracle.rel_l2(our, gr[k].numpy())
        report[k] = (e_or, e_ro, e_oo)
        bf16 = not base and k in BF16_PATH
        if bf16:
            ok = e_or < REF_BF16_TOL and e_oo <= max(e_ro, GRAD_TOL)
        else:
            ok = e_or < GRAD_TOL
        if not ok:
            bad[k] = report[k]
    print({k: tuple(f"{x:.1e}" for x in v) for k, v in report.items()})
    assert not bad, f"(ours-ref, ref-oracle, ours-oracle) relative L2: {bad}"
