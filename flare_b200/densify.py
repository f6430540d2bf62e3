"""Densification and pruning of the primitive set on the device (reference source/train.py:816-836 and
955-1240).

Every densification iteration the reference
  * keeps a primitive when its opacity logit A >= logit(opacity_threshold) and its effective support
    ||exp(s)|| * (max(0, kappa (11.3449 + 2 ln sigmoid(A))))^(1/(2 kappa)) / sqrt(11.3449) >= min_s_norm;
  * splits a kept primitive whose centre moved by >= mu_threshold in this iteration's optimizer step
    (unless the set is over max_primitives): one copy stays at the centre from before the step with the
    moments from before the step, the other takes the new centre and moments; every other attribute and
    its Adam moments are duplicated;
  * orders the result [kept, not split | split, first copies | split, second copies], then clamps s to
    [ln min_s_coef, ln(max_s_coef * extent / 2)] and RGB at 0.
Here the plan (masks and the row map) is computed with device tensor ops and all per-primitive tensors --
parameters, fp16 descriptor mirror and Adam moments -- are rebuilt by one flare_gather_rows launch.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib

CHI2 = 11.3449


@dataclass
class DensifyParams:
    """Reference defaults (source/arguments/__init__.py:131-140)."""
    opacity_threshold: float = 1.0 / 28.0
    min_s_norm: float = 0.0001
    mu_threshold: float = 0.001
    max_primitives: int = -1
    min_s_coef: float = 0.0001
    max_s_coef: float = 0.05


def plan(m, m_before, s, A, k, p: DensifyParams):
    """Row map of the new primitive set and its block sizes: (src_row int32 (n_new,), n_orig, n_split)."""
    kf = 1.0 + torch.nn.functional.softplus(k.reshape(-1))
    Af = torch.sigmoid(A.reshape(-1))
    scale = torch.clamp(kf * (CHI2 + 2.0 * torch.log(Af)), min=0.0) ** (1.0 / (2.0 * kf)) / math.sqrt(CHI2)
    s_norm = torch.sqrt((torch.exp(s) ** 2).sum(1)) * scale
    keep = (A.reshape(-1) >= math.log(p.opacity_threshold / (1.0 - p.opacity_threshold))) & (s_norm >= p.min_s_norm)
    kept = keep.nonzero().reshape(-1)
    d = m[kept] - m_before[kept]
    moved = torch.sqrt((d * d).sum(1)) >= p.mu_threshold
    if not (p.max_primitives == -1 or kept.numel() <= p.max_primitives):
        moved = torch.zeros_like(moved)
    orig, split = kept[~moved], kept[moved]
    src = torch.cat([orig, split, split]).to(torch.int32).contiguous()
    return src, int(orig.numel()), int(split.numel())


def gather_rows(items, src_row, n_out, alt_begin, alt_end):
    """items: list of (src tensor, alt tensor or None) -> new tensors of n_out rows (one launch)."""
    lib = _lib.load()
    if len(items) > _lib.GATHER_MAX_TENSORS:
        raise ValueError(f"{len(items)} tensors, at most {_lib.GATHER_MAX_TENSORS}")
    outs = []
    arr = (_lib.GatherTensor * max(len(items), 1))()
    for i, (src, alt) in enumerate(items):
        if not src.is_contiguous() or (alt is not None and (not alt.is_contiguous() or alt.shape != src.shape)):
            raise ValueError("gather_rows: sources must be contiguous, alternatives of the same shape")
        out = torch.empty((n_out,) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
        row_bytes = src[0].numel() * src.element_size() if src.shape[0] else 4
        arr[i].src = ctypes.c_void_p(src.data_ptr())
        arr[i].src_alt = ctypes.c_void_p(alt.data_ptr()) if alt is not None else None
        arr[i].dst = ctypes.c_void_p(out.data_ptr())
        arr[i].row_bytes = int(row_bytes)
        outs.append(out)
    stream = ctypes.c_void_p(torch.cuda.current_stream(src_row.device).cuda_stream)
    _lib.check(lib.flare_gather_rows(arr, len(items), ctypes.c_void_p(src_row.data_ptr()), int(n_out),
                                     int(alt_begin), int(alt_end), stream), "flare_gather_rows")
    return outs


def snapshot_before_step(opt):
    """Centre and centre moments before this iteration's optimizer step (reference train.py:816-831)."""
    seg = {s.name: i for i, s in enumerate(opt.adam.segments)}["m"]
    mm, mv = opt.adam.state[seg]
    return opt.scene.m.clone(), mm.clone(), mv.clone()


def densify_and_prune(opt, before, extent: float, p: DensifyParams = DensifyParams()):
    """Rebuilds the scene's per-primitive tensors, the optimizer's masters / moments and its gradient
    buffer for the new primitive set.  `before` = snapshot_before_step(opt) taken before this iteration's
    optimizer step.  Returns (n_orig, n_split); the new count is n_orig + 2 n_split."""
    from .dp import GradBuffer
    sc = opt.scene
    m_before, m_before_avg, m_before_sq = before
    src, n_orig, n_split = plan(sc.m, m_before, sc.s, sc.RGBA[:, 3], sc.k, p)
    n_new = n_orig + 2 * n_split
    alt = (n_orig, n_orig + n_split)  # first copies of the split primitives: state from before the step
    segs = {s.name: (i, s) for i, s in enumerate(opt.adam.segments)}
    st = opt.adam.state
    items = [(sc.RGBA, None), (sc.k, None), (opt.cond32, None), (sc.cond, None), (sc.m, m_before), (sc.s, None),
             (sc.q, None)]
    per_prim = ["RGB", "A", "k", "conditioning", "m", "s", "q"]
    for name in per_prim:
        i, _ = segs[name]
        a_alt = m_before_avg if name == "m" else None
        v_alt = m_before_sq if name == "m" else None
        items += [(st[i][0], a_alt), (st[i][1], v_alt)]
    outs = gather_rows(items, src, n_new, *alt)
    RGBA, k, cond32, cond16, m, s, q = outs[:7]
    moments = outs[7:]
    s.clamp_(min=math.log(p.min_s_coef), max=math.log(p.max_s_coef * (extent / 2.0)))
    RGBA[:, :3].clamp_(min=0.0)
    sc.RGBA, sc.k, sc.cond, sc.m, sc.s, sc.q = RGBA, k, cond16, m, s, q
    opt.cond32 = cond32
    grads = GradBuffer(n_new, True, m.device)
    opt.rebind(grads, {name: (moments[2 * j], moments[2 * j + 1]) for j, name in enumerate(per_prim)})
    return n_orig, n_split
