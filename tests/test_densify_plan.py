"""The densification plan on the CPU: keep / split masks and the row map against a direct restatement of
the reference's rules (source/train.py:955-1240), including the max_primitives cap."""
import math

import torch

from flare_b200 import densify
from flare_b200.scene import make_scene


def _expected_rows(m, m_before, s, A, k, p):
    kf = 1.0 + torch.nn.functional.softplus(k.reshape(-1))
    Af = torch.sigmoid(A.reshape(-1))
    scale = torch.clamp(kf * (11.3449 + 2.0 * torch.log(Af)), min=0.0) ** (1.0 / (2.0 * kf)) / math.sqrt(11.3449)
    s_norm = torch.sqrt((torch.exp(s) ** 2).sum(1)) * scale
    keep = (A.reshape(-1) >= math.log(p.opacity_threshold / (1 - p.opacity_threshold))) & (s_norm >= p.min_s_norm)
    kept = [i for i in range(m.shape[0]) if keep[i]]
    moved = [i for i in kept if float(torch.linalg.norm(m[i] - m_before[i])) >= p.mu_threshold]
    if not (p.max_primitives == -1 or len(kept) <= p.max_primitives):
        moved = []
    orig = [i for i in kept if i not in set(moved)]
    return orig + moved + moved, len(orig), len(moved)


def _case(seed):
    sc = make_scene(400, seed)
    g = torch.Generator().manual_seed(seed + 1)
    A = sc.RGBA[:, 3].clone()
    A[torch.rand(400, generator=g) < 0.2] = -6.0              # opacity below 1/28: pruned
    s = sc.s.clone()
    s[torch.rand(400, generator=g) < 0.1] = math.log(1e-6)     # support below min_s_norm: pruned
    m_before = sc.m - (torch.rand(400, 1, generator=g) < 0.3) * 0.01  # 30 % moved by 0.01 >= mu_threshold
    return sc.m, m_before, s, A, sc.k


def test_plan_matches_reference_rules():
    p = densify.DensifyParams()
    for seed in (0, 1, 2):
        m, mb, s, A, k = _case(seed)
        src, n_orig, n_split = densify.plan(m, mb, s, A, k, p)
        rows, eo, es = _expected_rows(m, mb, s, A, k, p)
        assert (n_orig, n_split) == (eo, es) and n_split > 0 and n_orig > 0
        assert src.dtype == torch.int32 and src.tolist() == rows


def test_plan_stops_splitting_over_max_primitives():
    m, mb, s, A, k = _case(3)
    p = densify.DensifyParams(max_primitives=10)
    src, n_orig, n_split = densify.plan(m, mb, s, A, k, p)
    rows, eo, es = _expected_rows(m, mb, s, A, k, p)
    assert n_split == 0 and es == 0 and src.tolist() == rows
