"""Data-parallel FlaRe training step over one process per GPU.

The reference trains on one GPU (CPyOptiXFLARERenderer_CUDA_Core.cu:52 fixes device 0); its step is
train.py:449-858: SetGeometry on the activated parameters, Forward_training over a ray batch, an image
loss and its gradient in torch, Backward into zeroed gradient buffers.  Here the same step runs on N
ranks: the scene is replicated, the rays of the step's views are sharded by view (and by row band when
there are more ranks than views), each rank renders and back-propagates its shard into one flat fp32
gradient buffer, and a single all-reduce (NCCL over NVLink) sums that buffer once per step.  With the
decoder, that buffer holds each primitive's 80-float gradient row (flare_backward_args.prim_rows)
rather than its 110 expanded gradient floats; the rows expand after the exchange.  The loss is
normalised by the global ray count, so the summed gradient equals the single-GPU gradient of the whole
batch.

Loss: L1 against a target image, on the image clamped to [0, 1] with the gradient masked where the
clamp is active (the reference clamps before its loss, train.py:688-702).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .scene import Scene

T_NEAR, T_FAR = 0.1, 1000.0
REG_A = -(T_NEAR * T_FAR) / (T_FAR - T_NEAR)
REG_B = T_FAR / (T_FAR - T_NEAR)
T_THRESHOLD_TRAINING = 1e-4  # arguments/__init__.py:129


def shard_rays(n_views: int, rays_per_view: int, world: int, rank: int):
    """This rank's (view, first ray, ray count) pieces.  Views are dealt round-robin; with more ranks
    than views every view is cut into contiguous row bands, one per rank that shares it."""
    if world <= n_views:
        return [(v, 0, rays_per_view) for v in range(rank, n_views, world)]
    per_view = world // n_views
    if world % n_views:
        raise ValueError(f"{world} ranks do not divide evenly over {n_views} views")
    v = rank // per_view
    b = rank % per_view
    lo = rays_per_view * b // per_view
    hi = rays_per_view * (b + 1) // per_view
    return [(v, lo, hi - lo)]


def shard_rays_interleaved(n_views: int, width: int, height: int, world: int, rank: int, block_rows: int = 1):
    """This rank's rays when the image rows of every view are cut into blocks of `block_rows` rows dealt
    round-robin over the ranks (rank r takes blocks r, r + world, ...): (view, first ray, ray count) pieces
    of one block each.  Every rank then sees a mix of dense and sparse parts of every view (one contiguous
    band per rank is not balanced: the middle rows of an image cross the scene's densest part), while a
    block of rows keeps its rays' directions close (a traversal packet stays coherent); a caller passes a
    rank's pieces to the renderer as ONE ray batch."""
    out = []
    nblk = (height + block_rows - 1) // block_rows
    for v in range(n_views):
        for b in range(rank, nblk, world):
            y0, y1 = b * block_rows, min(height, (b + 1) * block_rows)
            out.append((v, y0 * width, (y1 - y0) * width))
    return out


def shard_rays_banded(n_views: int, rays_per_view: int, world: int, rank: int):
    """This rank's (view, first ray, ray count) pieces when every rank takes the same row band of every
    view: band `rank` of `world` contiguous bands per view.  A rank's work then averages over all views
    (views differ in hits per ray, so dealing whole views leaves the rank with the densest view as the
    step's straggler); a caller passes a rank's pieces to the renderer as ONE ray batch."""
    out = []
    for v in range(n_views):
        lo = rays_per_view * rank // world
        hi = rays_per_view * (rank + 1) // world
        if hi > lo:
            out.append((v, lo, hi - lo))
    return out


PRIM_ROW = 80  # FLARE_PRIM_ROW_FLOATS: [dm 3 | ds 2 | dq 4 | dRGB 3 | dA 1 | dk 1 | 0 0 | d1 64]
PER_PRIM = ("RGB", "A", "k", "m", "s", "q", "cond")


def grad_layout(n: int, decoder: bool, cond_dim: int = 96, n_features: int = 13154):
    """(exchanged, local) segments of one step's gradients: name -> shape (N = primitives).  The decoder
    path exchanges each primitive's 80-float row (its geometry / colour gradients and the sum of its
    layer-1 deltas, from which the descriptor gradient is formed after the exchange: it is linear in
    them) instead of the 14 + descriptor-width floats of the expanded gradients; those stay local."""
    per = [("RGB", (n, 3)), ("A", (n, 1)), ("k", (n, 1)), ("m", (n, 3)), ("s", (n, 2)), ("q", (n, 4))]
    if not decoder:
        return [("loss", (1,))] + per, []
    exch = [("loss", (1,)), ("rows", (n, PRIM_ROW)), ("features", (n_features,)), ("w3", (1, 512)), ("b3", (1, 64)),
            ("w2", (1, 4096)), ("b2", (1, 512)), ("w1", (1, 8192)), ("b1", (1, 512))]
    return exch, per + [("cond", (n, cond_dim))]


class GradBuffer:
    """All gradients of a step as views into contiguous fp32 buffers: `flat`, summed over ranks by one
    all-reduce per step, and (decoder path) `local`, the per-primitive gradients that
    expand_rows_() forms from the summed rows."""

    ALIGN = 16  # floats: every segment starts on a 64-byte boundary (the kernels use vector reductions)

    def __init__(self, n: int, decoder: bool, device, cond_dim: int = 96, n_features: int = 13154):
        self.n, self.decoder = n, decoder
        exch, local = grad_layout(n, decoder, cond_dim, n_features)
        self.layout = exch + local
        self.views = {}
        self.flat = self._alloc(exch, device)
        self.local = self._alloc(local, device)

    def _alloc(self, layout, device):
        offs, off = [], 0
        for _, shape in layout:
            offs.append(off)
            cnt = int(torch.tensor(shape).prod())
            off += (cnt + self.ALIGN - 1) // self.ALIGN * self.ALIGN
        buf = torch.zeros(off, dtype=torch.float32, device=device)
        for (name, shape), o in zip(layout, offs):
            cnt = int(torch.tensor(shape).prod())
            self.views[name] = buf[o:o + cnt].view(*shape)
        return buf

    def __getitem__(self, k):
        return self.views[k]

    def zero_(self):
        self.flat.zero_()
        self.local.zero_()

    def allreduce_(self, group=None):
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)

    def expand_rows_(self, A1, decoder_kind: int):
        """Adds the (summed) per-primitive rows into the per-primitive gradients (decoder path)."""
        if self.decoder:
            from .renderer import scatter_prim_rows
            v = self.views
            scatter_prim_rows(v["rows"], A1, decoder_kind, v["RGB"], v["A"], v["k"], v["m"], v["s"], v["q"],
                              v["cond"])

    @property
    def nbytes(self):
        """Bytes summed over ranks per step."""
        return self.flat.numel() * 4


@dataclass
class Shard:
    O: torch.Tensor
    v: torch.Tensor
    target: torch.Tensor


class TrainStep:
    """Runs SetGeometry + per-shard Forward_training / L1 loss / Backward + one all-reduce."""

    def __init__(self, renderer, scene: Scene, shards, total_rays: int, decoder: bool = True, bg=(0.0, 0.0, 0.0),
                 lambda_depth: float = 0.0, lambda_normal: float = 0.0, group=None):
        self.r = renderer
        self.sc = scene
        self.decoder = decoder
        self.shards = shards
        self.total_rays = total_rays
        self.bg = bg
        self.lambda_depth = lambda_depth
        self.lambda_normal = lambda_normal
        self.group = group
        dev = scene.m.device
        self.grads = GradBuffer(scene.n, decoder, dev, scene.cond.shape[1], scene.features.numel())
        self.buf = []
        for sh in shards:
            R = sh.O.shape[0]
            z = lambda *s: torch.zeros(*s, device=dev)  # noqa: E731
            self.buf.append(dict(bitmap=z(R, 3), dacc=z(R, 4), nacc=z(R, 4), dai=z(R, 2), sn=z(R, 3), prefix=z(R, 4),
                                 dLdI=z(R, 3)))
        self.loss = self.grads["loss"]  # summed by the same all-reduce as the gradients
        self.collect_stats = False
        self.hits = 0
        self.fwd_passes = 0

    def rebind(self, scene: Scene, grads: GradBuffer):
        """Uses a new primitive set (after densification) and its gradient buffer."""
        self.sc, self.grads = scene, grads
        self.loss = grads["loss"]

    def geometry(self):
        sc = self.sc
        self.r.SetGeometry(sc.m, torch.exp(sc.s), sc.q, torch.sigmoid(sc.RGBA[:, 3]).contiguous(),
                           (1.0 + torch.nn.functional.softplus(sc.k[:, 0])).contiguous())

    def __call__(self):
        sc, r, G = self.sc, self.r, self.grads
        self.geometry()
        G.zero_()
        inv = 1.0 / (3.0 * self.total_rays)
        for sh, b in zip(self.shards, self.buf):
            for k in ("bitmap", "dacc", "nacc", "prefix"):
                b[k].zero_()
            fargs = (sh.O, sh.v, b["bitmap"], *self.bg, sc.m, sc.s, sc.q, sc.RGBA, sc.k, T_THRESHOLD_TRAINING, b["dacc"],
                     REG_A, REG_B, b["dai"], b["sn"], b["nacc"])
            if self.decoder:
                dec = (sc.cond, sc.features, sc.A1, sc.b1, sc.A2, sc.b2, sc.A3, sc.b3)
                r.Forward_training(*dec, *fargs)
            else:
                r.Forward_training_base(*fargs)
            if self.collect_stats:
                st = r.stats()
                self.hits += st["hits_composited"]
                self.fwd_passes += st["passes"]
            img = b["bitmap"].clamp(0.0, 1.0)
            diff = img - sh.target
            self.loss += diff.abs().sum() * inv
            torch.mul(torch.sign(diff), inv * (img == b["bitmap"]).float(), out=b["dLdI"])
            I = img.contiguous()
            if self.decoder:
                r.Backward(*dec, sh.O, sh.v, *self.bg, sc.m, sc.s, sc.q, sc.RGBA, sc.k, I, b["dLdI"], G["RGB"], G["A"],
                           G["k"], G["w3"], G["b3"], G["w2"], G["b2"], G["w1"], G["b1"], G["cond"], G["features"],
                           G["m"], G["s"], G["q"], T_THRESHOLD_TRAINING, b["dacc"], b["prefix"],
                           self.lambda_depth, REG_A, REG_B, b["dai"], b["sn"], b["nacc"], self.lambda_normal,
                           prim_rows=G["rows"])
            else:
                r.Backward_base(sh.O, sh.v, *self.bg, sc.m, sc.s, sc.q, sc.RGBA, sc.k, I, b["dLdI"], G["RGB"], G["A"],
                                G["k"], G["m"], G["s"], G["q"], T_THRESHOLD_TRAINING, b["dacc"], b["prefix"],
                                self.lambda_depth, REG_A, REG_B, b["dai"], b["sn"], b["nacc"], self.lambda_normal)
        G.allreduce_(self.group)
        if self.decoder:
            G.expand_rows_(sc.A1, 1 if sc.cond.shape[1] == 32 else 0)
        return self.loss
