"""The optimizer step after the backward: a fused Adam over the reference's 16 parameter groups.

Restates the reference's training step tail (source/train.py:754-790 gradient un-permutation, 833-860
gradients + scale regulariser + optimizer.step(), 860-953 per-group learning-rate schedule) and the
optimizer set-up (source/scene/gaussian_model.py:248-336): torch.optim.Adam with default betas / eps and
one group per parameter tensor, each group's learning rate lr0 * exp(coef * iteration) clamped by its
final value (floor when coef <= 0, ceiling otherwise).  The update runs as one CUDA launch over every
group (flare_adam_step); fp32 masters of the fp16 tensors the renderer reads (descriptor rows, decoder
weights) are kept here and their fp16 copies are refreshed by the same launch.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib

# Reference defaults (source/arguments/__init__.py:148-218): group -> (lr, exp_decay_coef, lr_final), in
# the optimizer's group order (scene/gaussian_model.py:318-335).
REFERENCE_LR = {
    "RGB": (0.005, -0.000086643, 0.001),
    "A": (0.05, -0.000086643, 0.025),
    "k": (0.1, -0.000086643, 0.1),
    "w1_uv": (0.0125, -0.000086643, 0.001),
    "w1_v": (0.03, -0.000086643, 0.001),
    "w1_conditioning": (0.0015, -0.000086643, 0.001),
    "b1": (0.00475, -0.000086643, 0.001),
    "w2": (0.005, -0.000086643, 0.001),
    "b2": (0.005, -0.000086643, 0.001),
    "w3": (0.005, -0.000086643, 0.001),
    "b3": (0.005, -0.000086643, 0.001),
    "conditioning": (0.005, -0.000086643, 0.005),
    "features": (0.005, -0.000086643, 0.005),
    "m": (0.0025, -0.00015, 0.000001189614075),
    "s": (0.0396538025, -0.000086643, 0.0396538025),
    "q": (0.01, -0.000086643, 0.001),
}
REG_SCALE_LAMBDA = 0.001  # arguments/__init__.py:148


def lr_at(lr0: float, coef: float, lr_final: float, iteration: int) -> float:
    """Exponential decay clamped at the final value (a floor when decaying, a ceiling when growing)."""
    x = lr0 * math.exp(coef * iteration)
    return max(x, lr_final) if coef <= 0.0 else min(x, lr_final)


def _fragment_maps(device):
    """Index maps from the reference's per-warp fragment layout (train.py:754-790) to dense matrices:
    entry ((i*J + j)*64 + c*32 + lane) holds W[8i + lane/4][8j + 2(lane%4) + c]; bias entries
    (j*64 + c*32 + lane) sum into b[8j + lane/4]."""
    def wmap(rows, cols):
        J = cols // 8
        out = torch.empty(rows, cols, dtype=torch.long)
        for t in range(rows * cols):
            lane, c, ij = t & 31, (t >> 5) & 1, t >> 6
            i, j = ij // J, ij % J
            out[8 * i + (lane >> 2), 8 * j + 2 * (lane & 3) + c] = t
        return out.to(device)

    def bmap(n_entries):
        return torch.tensor([8 * (t >> 6) + ((t & 31) >> 2) for t in range(n_entries)], dtype=torch.long,
                            device=device)

    return {"w1": wmap(64, 128), "w2": wmap(64, 64), "w3": wmap(8, 64), "b1": bmap(512), "b2": bmap(512),
            "b3": bmap(64)}


_MAPS = {}


def dense_decoder_grads(G) -> dict:
    """Dense gradients (dW1 (64,128), db1 (64), dW2 (64,64), db2 (64), dW3 (16,64), db3 (16)) from the
    fragment-layout buffers the renderer's Backward fills (rows summed, as train.py:754-790 does)."""
    dev = G["w1"].device
    if dev not in _MAPS:
        _MAPS[dev] = _fragment_maps(dev)
    M = _MAPS[dev]
    w1 = G["w1"].reshape(-1, 8192).sum(0)[M["w1"]]
    w2 = G["w2"].reshape(-1, 4096).sum(0)[M["w2"]]
    w3 = torch.zeros(16, 64, device=dev)
    w3[:8] = G["w3"].reshape(-1, 512).sum(0)[M["w3"]]
    b1 = torch.zeros(64, device=dev).index_add_(0, M["b1"], G["b1"].reshape(-1, 512).sum(0))
    b2 = torch.zeros(64, device=dev).index_add_(0, M["b2"], G["b2"].reshape(-1, 512).sum(0))
    b3 = torch.zeros(16, device=dev)
    b3[:8] = torch.zeros(8, device=dev).index_add_(0, M["b3"], G["b3"].reshape(-1, 64).sum(0))
    return {"w1": w1, "b1": b1, "w2": w2, "b2": b2, "w3": w3, "b3": b3}


@dataclass
class Segment:
    name: str
    param: torch.Tensor       # fp32 master (the whole tensor; the segment is a column block of it)
    grad: torch.Tensor        # dense (rows, width), contiguous
    width: int
    offset: int = 0           # first column of the block
    mirror: torch.Tensor = None  # fp16 copy with the same layout (refreshed with the update)
    scale_reg: float = 0.0


class FusedAdam:
    """Adam over segments, all updated by one flare_adam_step launch per step (torch.optim.Adam's
    update with default betas (0.9, 0.999) and eps 1e-8)."""

    def __init__(self, segments, betas=(0.9, 0.999), eps=1e-8):
        self.lib = _lib.load()
        self.segments = list(segments)
        if len(self.segments) > _lib.ADAM_MAX_SEGMENTS:
            raise ValueError(f"{len(self.segments)} segments, at most {_lib.ADAM_MAX_SEGMENTS}")
        self.betas, self.eps = betas, eps
        self.t = 0
        self.state = []
        for s in self.segments:
            stride = s.param.shape[-1] if s.param.dim() > 1 else s.param.numel()
            rows = s.param.numel() // stride
            if s.offset + s.width > stride:
                raise ValueError(f"{s.name}: columns {s.offset}..{s.offset + s.width} outside a row of {stride}")
            if s.grad.numel() != rows * s.width:
                raise ValueError(f"{s.name}: gradient has {s.grad.numel()} elements, expected {rows}x{s.width}")
            self.state.append((torch.zeros_like(s.grad, dtype=torch.float32),
                               torch.zeros_like(s.grad, dtype=torch.float32)))

    def step(self, lrs: dict):
        self.t += 1
        a = _lib.AdamArgs(n_segments=len(self.segments), beta1=self.betas[0], beta2=self.betas[1], eps=self.eps,
                          step=self.t)
        for i, (s, (m, v)) in enumerate(zip(self.segments, self.state)):
            p = s.param
            stride = p.shape[-1] if p.dim() > 1 else p.numel()
            rows = p.numel() // stride
            if not (p.is_contiguous() and s.grad.is_contiguous() and p.dtype == torch.float32):
                raise ValueError(f"{s.name}: parameters and gradients must be contiguous fp32")
            seg = a.seg[i]
            seg.param, seg.grad = ctypes.c_void_p(p.data_ptr()), ctypes.c_void_p(s.grad.data_ptr())
            seg.exp_avg, seg.exp_avg_sq = ctypes.c_void_p(m.data_ptr()), ctypes.c_void_p(v.data_ptr())
            seg.param_f16 = ctypes.c_void_p(s.mirror.data_ptr()) if s.mirror is not None else None
            seg.rows, seg.width, seg.p_stride, seg.p_offset = rows, s.width, stride, s.offset
            seg.lr, seg.scale_reg = float(lrs[s.name]), float(s.scale_reg)
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.segments[0].param.device).cuda_stream)
        _lib.check(self.lib.flare_adam_step(ctypes.byref(a), stream), "flare_adam_step")


class ModelOptimizer:
    """The reference's optimizer over a flare_b200.scene.Scene: the scene's fp32 tensors are the masters
    (RGB and A are the column blocks 0:3 and 3 of RGBA), fp32 masters are created for the fp16
    descriptor rows and decoder weights, whose fp16 tensors in the scene are refreshed every step."""

    def __init__(self, scene, grads, lr_table=REFERENCE_LR, reg_scale_lambda=REG_SCALE_LAMBDA):
        sc = scene
        self.scene, self.grads, self.lr_table = sc, grads, lr_table
        self.reg_scale_lambda = reg_scale_lambda
        self.cond32 = sc.cond.float().contiguous()
        self.W1 = sc.A1.float().contiguous()
        self.W2 = sc.A2.float().contiguous()
        self.W3 = sc.A3.float().contiguous()
        dev = sc.m.device
        self.dense = {"w1_uv": torch.zeros(64, 8, device=dev), "w1_v": torch.zeros(64, 24, device=dev),
                      "w1_conditioning": torch.zeros(64, 96, device=dev)}
        self._dec = {k: torch.zeros_like(v) for k, v in dense_decoder_grads(grads).items()}
        self.adam = FusedAdam(self._segments())

    def _segments(self):
        sc, G, S = self.scene, self.grads, Segment
        n = sc.m.shape[0]
        return [S("RGB", sc.RGBA, G["RGB"], 3, 0), S("A", sc.RGBA, G["A"], 1, 3), S("k", sc.k, G["k"], 1),
                S("w1_uv", self.W1, self.dense["w1_uv"], 8, 0, sc.A1),
                S("w1_v", self.W1, self.dense["w1_v"], 24, 8, sc.A1),
                S("w1_conditioning", self.W1, self.dense["w1_conditioning"], 96, 32, sc.A1),
                S("b1", sc.b1, self._dec["b1"], 64), S("w2", self.W2, self._dec["w2"], 64, 0, sc.A2),
                S("b2", sc.b2, self._dec["b2"], 64), S("w3", self.W3, self._dec["w3"], 64, 0, sc.A3),
                S("b3", sc.b3, self._dec["b3"], 16), S("conditioning", self.cond32, G["cond"], 96, 0, sc.cond),
                S("features", sc.features, G["features"], 13154), S("m", sc.m, G["m"], 3),
                S("s", sc.s, G["s"], 2, 0, None, self.reg_scale_lambda / n), S("q", sc.q, G["q"], 4)]

    def rebind(self, grads, moments: dict):
        """After the primitive set changed (densification): the scene holds the new per-primitive
        tensors, `grads` is the new gradient buffer and `moments` maps the per-primitive groups to their
        rebuilt (exp_avg, exp_avg_sq); the decoder groups keep theirs, the step count is unchanged."""
        old = {s.name: st for s, st in zip(self.adam.segments, self.adam.state)}
        self.grads = grads
        self.adam.segments = self._segments()
        self.adam.state = [moments.get(s.name, old[s.name]) for s in self.adam.segments]
        for s_, (m_, v_) in zip(self.adam.segments, self.adam.state):
            if m_.numel() != s_.grad.numel():
                raise ValueError(f"{s_.name}: {m_.numel()} moments for {s_.grad.numel()} gradients")

    def step(self, iteration: int):
        dg = dense_decoder_grads(self.grads)
        for k, v in dg.items():
            self._dec[k].copy_(v)
        self.dense["w1_uv"].copy_(dg["w1"][:, 0:8])
        self.dense["w1_v"].copy_(dg["w1"][:, 8:32])
        self.dense["w1_conditioning"].copy_(dg["w1"][:, 32:128])
        lrs = {k: lr_at(*v, iteration) for k, v in self.lr_table.items()}
        self.adam.step(lrs)
