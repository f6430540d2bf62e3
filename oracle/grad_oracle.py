"""Gradient oracle for the FlaRe render path -- TEST INFRASTRUCTURE ONLY (torch autograd, float64, CPU).

Rebuilds the forward of decode_oracle.c as a differentiable torch graph over the composited hits (the
set and order of composited hits come from the fp32 C oracle) and differentiates the scalar the
reference's Backward kernel differentiates (source/renderer/CPyOptiXFLARERenderer_CUDA_Backward.cu):

    L = sum_rays dL/dI . C  +  lambda_depth * L_d / 2  +  lambda_normal * L_n

  * C = sum_i w_i c_i + bg T_final, w_i = T_i alpha_i, T_i = prod_{j<i} (1 - alpha_j)    (Backward.cu:1853-1904)
  * L_d = sum_i 4 w_i (t~_i W_<i - (t~ w)_<i), t~ = clamp(a/t + b, 0, 1): the depth accumulator of the
    forward (Forward_training.cu:884-895).  The reference backward (dL_do, dL_dt at Backward.cu:1753-1810)
    is the exact gradient of L_d / 2, which is what this oracle differentiates.
  * L_n = sum_i stopgrad(w_i) (1 - sgn_i N_target . N_i): only the orientation is trained
    (Backward.cu:1814-1817 sets the opacity term to zero).
  * t takes the value of the fp32 traversal hit and the derivative of N.(m - O)/(N.v), so dt/dm and dt/dq
    flow as in Backward.cu:1587-1608,2033-2216 while the LUT cell of every hit is the kernel's.
  * fp16 rounding of the decoder input and hidden activations is kept in the values and passed
    straight through in the gradient (the reference differentiates its rounded activations).
Outputs the gradients in the dense layouts (dW1 (64,128) etc.); the reference fragment layout is a
permutation of these (train.py:754-790).
"""
from __future__ import annotations

import math

import numpy as np
import torch

LUT_SCALE = 0.29689279887990428378374198030042
LUT_RES = (16, 25, 40, 64)
LUT_OFF = (0, 256, 881, 2481)
# grid/SH decoder variant: 8 dense levels of floor(4 * 1.5^l) vertices per side (float2 offsets)
GRID_RES = (4, 6, 9, 13, 20, 30, 45, 68)
GRID_OFF = (0, 16, 52, 133, 302, 702, 1602, 3627)


def _st16(x):
    return x + (x.to(torch.float16).to(x.dtype) - x).detach()


def _hswish(y):
    return y * torch.clamp(y + 3.0, 0.0, 6.0) / 6.0


def _lut(features, cu, cw, res=LUT_RES, offs=LUT_OFF):
    """features (13154,) float64 requiring grad; cu, cw (H,) -> (H, 2 * levels)."""
    F2 = features.view(-1, 2)
    outs = []
    xs = torch.clamp((cu + 1.0) * 0.5, 0.0, 1.0)
    ys = torch.clamp((cw + 1.0) * 0.5, 0.0, 1.0)
    for l in range(len(res)):
        R = res[l]
        px, py = xs * (R - 1), ys * (R - 1)
        ix = torch.clamp(torch.floor(px.detach()), max=R - 2).long()
        iy = torch.clamp(torch.floor(py.detach()), max=R - 2).long()
        fx, fy = px - ix, py - iy
        base = offs[l] + iy * R + ix
        f00, f10 = F2[base], F2[base + 1]
        f01, f11 = F2[base + R], F2[base + R + 1]
        r0 = f00 * (1 - fx)[:, None] + f10 * fx[:, None]
        r1 = f01 * (1 - fx)[:, None] + f11 * fx[:, None]
        outs.append(r0 * (1 - fy)[:, None] + r1 * fy[:, None])
    return torch.cat(outs, 1)


def _pe(v):
    """(H,3) -> (H,24) in the decoder's order: axis a, octave f -> (sin, cos) at 8a + 2f."""
    cols = []
    for a in range(3):
        for f in range(4):
            arg = math.pi * (2 ** f) * v[:, a]
            cols += [torch.sin(arg), torch.cos(arg)]
    return torch.stack(cols, 1)


def _sh(v):
    """(H,3) unit directions -> (H,16) real spherical harmonics of degrees 0..3."""
    x, y, z = v[:, 0], v[:, 1], v[:, 2]
    xx, yy, zz = x * x, y * y, z * z
    cols = [torch.full_like(x, 0.28209479177387814), -0.48860251190291987 * y, 0.48860251190291987 * z,
            -0.48860251190291987 * x, 1.0925484305920792 * x * y, -1.0925484305920792 * y * z,
            0.94617469575755997 * zz - 0.31539156525251999, -1.0925484305920792 * x * z,
            0.54627421529603959 * (xx - yy), 0.59004358992664352 * y * (-3.0 * xx + yy),
            2.8906114426405538 * x * y * z, 0.45704579946446572 * y * (1.0 - 5.0 * zz),
            0.3731763325901154 * z * (5.0 * zz - 3.0), 0.45704579946446572 * x * (1.0 - 5.0 * zz),
            1.4453057213202769 * z * (xx - yy), 0.59004358992664352 * x * (-xx + 3.0 * yy)]
    return torch.stack(cols, 1)


def gradients(scene, O, v, csr, nhits, dL_dI, base=False, bg=(0.0, 0.0, 0.0), reg_a=0.0, reg_b=0.0,
              lambda_depth=0.0, lambda_normal=0.0, surface_normal=None, exact_t=False, compact=False):
    """Returns a dict of float64 gradients (dense layouts) and the composited image C.
    exact_t=True evaluates at the float64 ray-plane t instead of the fp32 traversal t (self-checks).
    compact=True returns per-primitive gradients only for the primitives that were hit (in sorted index
    order) instead of scattering them into full-size tensors."""
    g = scene if isinstance(scene, dict) else scene.__dict__
    dt = torch.float64
    off0, _, ii0 = csr
    nh0 = np.asarray(nhits, np.int64)
    ray0 = np.repeat(np.arange(len(nh0)), nh0)
    pos0 = np.concatenate([np.arange(k) for k in nh0]) if len(nh0) else np.zeros(0, np.int64)
    used = np.unique(np.asarray(ii0, np.int64)[np.asarray(off0[:-1], np.int64)[ray0] + pos0])
    n_all = None
    P = {}
    for k, x in g.items():
        a = x.detach().cpu() if hasattr(x, "detach") else torch.as_tensor(np.asarray(x))
        if k in ("m", "s", "q", "RGBA", "k", "cond"):  # per-primitive: only the rows that are hit
            n_all = a.shape[0]
            a = a[torch.as_tensor(used)]
        P[k] = a.float().to(dt)
    remap = np.full(max(n_all or 0, 1), -1, np.int64)
    remap[used] = np.arange(len(used))
    names = ["m", "s", "q", "RGBA", "k"] + ([] if base else ["cond", "features", "A1", "b1", "A2", "b2", "A3", "b3"])
    for k in names:
        P[k].requires_grad_(True)
    O = torch.as_tensor(np.asarray(O, np.float32), dtype=dt)
    v = torch.as_tensor(np.asarray(v, np.float32), dtype=dt)
    dLdI = torch.as_tensor(np.asarray(dL_dI, np.float32), dtype=dt)
    off, tt_csr, ii = csr
    nhits = np.asarray(nhits, np.int64)
    R = O.shape[0]
    ray = np.repeat(np.arange(R), nhits)
    pos = np.concatenate([np.arange(n) for n in nhits]) if len(nhits) else np.zeros(0, np.int64)
    flat = np.asarray(off[:-1], np.int64)[ray] + pos
    hidx = remap[np.asarray(ii, np.int64)[flat]]
    t_trav = torch.as_tensor(np.asarray(tt_csr, np.float32)[flat], dtype=dt)
    ray_t, idx_t = torch.as_tensor(ray), torch.as_tensor(hidx)
    Oh, vh = O[ray_t], v[ray_t]
    m, s, q = P["m"][idx_t], P["s"][idx_t], P["q"][idx_t]
    S = 2.0 / (q * q).sum(1)
    a, b, c, d = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    U = torch.stack([1 - S * (c * c + d * d), S * (b * c + a * d), S * (b * d - a * c)], 1)
    V = torch.stack([S * (b * c - a * d), 1 - S * (b * b + d * d), S * (c * d + a * b)], 1)
    N = torch.stack([S * (b * d + a * c), S * (c * d - a * b), 1 - S * (b * b + c * c)], 1)
    ndv = (N * vh).sum(1)
    t_rec = (N * (m - Oh)).sum(1) / ndv
    # value: the fp32 traversal t (what the kernels, and the reference, evaluate at); gradient: dt/d(m, q)
    t = t_rec if exact_t else t_trav + (t_rec - t_rec.detach())
    Ph = Oh + t[:, None] * vh
    dlt = Ph - m
    u = torch.exp(-s[:, 0]) * (U * dlt).sum(1)
    w = torch.exp(-s[:, 1]) * (V * dlt).sum(1)
    kappa = 1.0 + torch.nn.functional.softplus(P["k"][idx_t][:, 0])
    r2 = u * u + w * w
    G = torch.exp(-0.5 * torch.pow(r2, kappa) / kappa)
    rgba = P["RGBA"][idx_t]
    if base:
        col = rgba[:, :3]
        alpha = torch.sigmoid(rgba[:, 3]) * G
    else:
        grid = P["cond"].shape[1] == 32  # the grid/SH decoder variant
        if grid:
            # the kernel feeds the grid and spherical-harmonics inputs to layer 1 as f16 hi + lo parts (~22
            # bits), so they are not rounded to f16 here
            x = torch.cat([_lut(P["features"], u * LUT_SCALE, w * LUT_SCALE, GRID_RES, GRID_OFF),
                           _sh(vh), P["cond"][idx_t], torch.zeros(vh.shape[0], 64, dtype=dt)], 1)
            act = torch.relu
        else:
            x = torch.cat([_st16(_lut(P["features"], u * LUT_SCALE, w * LUT_SCALE)),
                           _pe(vh).to(torch.float16).to(dt), P["cond"][idx_t]], 1)
            act = _hswish
        h1 = _st16(act(x @ P["A1"].T + P["b1"]))
        h2 = _st16(act(h1 @ P["A2"].T + P["b2"]))
        y = h2 @ P["A3"].T + P["b3"]
        col = rgba[:, :3] * (torch.sigmoid(y[:, :3]) if grid else torch.relu(y[:, :3]))
        alpha = torch.sigmoid(rgba[:, 3]) * G * torch.sigmoid(y[:, 3])
    Hm = int(nhits.max()) if len(nhits) and nhits.max() > 0 else 1
    pos_t = torch.as_tensor(pos)
    A = torch.zeros(R, Hm, dtype=dt).index_put((ray_t, pos_t), alpha)
    Cc = torch.zeros(R, Hm, 3, dtype=dt).index_put((ray_t, pos_t), col)
    one_minus = 1.0 - A
    Tincl = torch.cumprod(one_minus, 1)
    Texcl = torch.cat([torch.ones(R, 1, dtype=dt), Tincl[:, :-1]], 1)
    W = Texcl * A
    bgv = torch.as_tensor(bg, dtype=dt)
    C = (W[:, :, None] * Cc).sum(1) + Tincl[:, -1:] * bgv[None, :]
    loss = (dLdI * C).sum()
    if lambda_depth != 0.0:
        # The reference's depth-regulariser share of dL/dq uses dt/dq without the factor S = 2/|q|^2
        # (Backward.cu:2096-2110, Backward_base.cu:496-510): the depth term's explicit t is given a
        # q-gradient scaled by 1/S (values and every other gradient unchanged).
        q_d = P["q"][idx_t]
        q_d = q_d.detach() + (q_d - q_d.detach()) / S.detach()[:, None]
        S_d = 2.0 / (q_d * q_d).sum(1)
        a_, b_, c_, d_ = q_d[:, 0], q_d[:, 1], q_d[:, 2], q_d[:, 3]
        N_d = torch.stack([S_d * (b_ * d_ + a_ * c_), S_d * (c_ * d_ - a_ * b_), 1 - S_d * (b_ * b_ + c_ * c_)], 1)
        t_rd = (N_d * (m - Oh)).sum(1) / (N_d * vh).sum(1)
        t_d = t_trav + (t_rd - t_rd.detach()) if not exact_t else t_rd
        tt = torch.zeros(R, Hm, dtype=dt).index_put((ray_t, pos_t), torch.clamp(reg_a / t_d + reg_b, 0.0, 1.0))
        Wb = torch.cumsum(W, 1) - W
        TWb = torch.cumsum(W * tt, 1) - W * tt
        Ld = (4.0 * W * (tt * Wb - TWb)).sum()
        loss = loss + lambda_depth * 0.5 * Ld
    if lambda_normal != 0.0 and surface_normal is not None:
        sn = torch.as_tensor(np.asarray(surface_normal, np.float32), dtype=dt)
        valid = ((sn * sn).sum(1) > 0).to(dt)[ray_t]
        sgn = torch.where(ndv > 0, -1.0, 1.0).detach()
        wd = W.detach()[ray_t, pos_t]
        Ln = (valid * wd * (1.0 - sgn * (sn[ray_t] * N).sum(1))).sum()
        loss = loss + lambda_normal * Ln
    loss.backward()
    out = {}
    for k in names:
        gk = P[k].grad.detach() if P[k].grad is not None else torch.zeros_like(P[k])
        if k in ("m", "s", "q", "RGBA", "k", "cond") and not compact:
            full = torch.zeros((n_all,) + tuple(gk.shape[1:]), dtype=dt)
            full[torch.as_tensor(used)] = gk
            gk = full
        out[k] = gk.clone()
    out["C"] = C.detach()
    out["RGB"] = out["RGBA"][:, :3]
    out["A"] = out["RGBA"][:, 3:4]
    return out


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))
