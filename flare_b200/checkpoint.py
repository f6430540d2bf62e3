"""The reference's checkpoint tuples (source/checkpoint_io.py:12-92, train.py:105-111).

A checkpoint is torch.save of (RGB, A, k, w1_uv, w1_v, w1_conditioning, b1, w2, b2, w3, b3,
conditioning_variable, features, m, s, q, optimizer.state_dict(), training_time) -- 18 entries -- or the
older 17-entry form without RGB.  Loading maps it onto this package's Scene (RGBA = [RGB | A], fp16
descriptor rows and decoder weights as the renderer reads them) and, if wanted, restores the fused
optimizer's moments and step from the Adam state dict; saving writes the same tuple from a Scene and a
ModelOptimizer, so the reference's evaluate / viewer scripts can read it.
"""
from __future__ import annotations

import torch

from .scene import Scene

NAMES = ("RGB", "A", "k", "w1_uv", "w1_v", "w1_conditioning", "b1", "w2", "b2", "w3", "b3",
         "conditioning_variable", "features", "m", "s", "q")
LEGACY_NAMES = NAMES[1:]
# optimizer group index of each reference parameter (scene/gaussian_model.py:318-335) -> fused-Adam segment
GROUP_SEGMENTS = ("RGB", "A", "k", "w1_uv", "w1_v", "w1_conditioning", "b1", "w2", "b2", "w3", "b3",
                  "conditioning", "features", "m", "s", "q")


def tensors_from_tuple(ckpt) -> dict:
    if not isinstance(ckpt, (tuple, list)):
        raise ValueError("unsupported checkpoint object: expected a tuple or list")
    if len(ckpt) == 18:
        names = NAMES
    elif len(ckpt) == 17:
        names = LEGACY_NAMES
    else:
        raise ValueError(f"unsupported checkpoint with {len(ckpt)} entries; expected 17 or 18")
    out = {}
    for i, name in enumerate(names):
        if not isinstance(ckpt[i], torch.Tensor):
            raise ValueError(f"checkpoint entry {i} ({name}) is not a tensor")
        out[name] = ckpt[i].detach()
    out["optimizer"] = ckpt[-2]
    out["training_time_seconds"] = float(ckpt[-1])
    return out


def scene_from_tensors(t: dict, device="cpu") -> Scene:
    n = t["m"].shape[0]
    f32 = lambda x: x.to(device=device, dtype=torch.float32).contiguous()  # noqa: E731
    RGB = t["RGB"] if "RGB" in t else torch.ones(n, 3)
    w1 = torch.cat([t["w1_uv"], t["w1_v"], t["w1_conditioning"]], 1)
    return Scene(m=f32(t["m"]), s=f32(t["s"]), q=f32(t["q"]),
                 RGBA=torch.cat([f32(RGB), f32(t["A"]).reshape(n, 1)], 1).contiguous(),
                 k=f32(t["k"]).reshape(n, 1).contiguous(),
                 cond=t["conditioning_variable"].to(device=device, dtype=torch.float16).contiguous(),
                 features=f32(t["features"]).reshape(-1), A1=w1.to(device=device, dtype=torch.float16).contiguous(),
                 b1=f32(t["b1"]).reshape(-1), A2=t["w2"].to(device=device, dtype=torch.float16).contiguous(),
                 b2=f32(t["b2"]).reshape(-1), A3=t["w3"].to(device=device, dtype=torch.float16).contiguous(),
                 b3=f32(t["b3"]).reshape(-1))


def load(path, device="cpu"):
    """Returns (Scene, tensors dict incl. 'optimizer' state dict and 'training_time_seconds').  The fp32
    descriptor rows and weights stay in the dict (tensors['conditioning_variable'], tensors['w1_uv'], ...)
    for an optimizer that continues training."""
    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    t = tensors_from_tuple(ckpt)
    return scene_from_tensors(t, device), t


def restore_optimizer(opt, tensors: dict):
    """Continues training from a checkpoint: fp32 masters from the checkpoint's fp32 tensors, Adam moments
    and step from its optimizer state dict (groups in the reference order)."""
    w1 = torch.cat([tensors["w1_uv"], tensors["w1_v"], tensors["w1_conditioning"]], 1)
    opt.W1.copy_(w1)
    opt.W2.copy_(tensors["w2"])
    opt.W3.copy_(tensors["w3"])
    opt.cond32.copy_(tensors["conditioning_variable"])
    sd = tensors.get("optimizer")
    if not sd:
        return
    state = sd.get("state", {})
    segs = {s.name: i for i, s in enumerate(opt.adam.segments)}
    # the 17-entry form has no RGB parameter, so its optimizer has no RGB group: group g is segment g + 1
    names = GROUP_SEGMENTS if "RGB" in tensors else GROUP_SEGMENTS[1:]
    step = 0
    for g, name in enumerate(names):
        st = state.get(g)
        if not st:
            continue
        m, v = opt.adam.state[segs[name]]
        for key, dst in (("exp_avg", m), ("exp_avg_sq", v)):
            if st[key].numel() != dst.numel():
                raise ValueError(f"optimizer group {g} ({name}): {key} has {st[key].numel()} values, the "
                                 f"parameter has {dst.numel()}")
        m.copy_(st["exp_avg"].reshape(m.shape))
        v.copy_(st["exp_avg_sq"].reshape(v.shape))
        step = max(step, int(float(st.get("step", 0))))
    opt.adam.t = step


def to_tuple(scene: Scene, opt=None, training_time: float = 0.0):
    """The 18-entry tuple (fp32 tensors on the CPU) with an Adam state dict in torch's format."""
    cpu = lambda x: x.detach().to("cpu", torch.float32).contiguous()  # noqa: E731
    n = scene.m.shape[0]
    W1 = opt.W1 if opt is not None else scene.A1.float()
    W2 = opt.W2 if opt is not None else scene.A2.float()
    W3 = opt.W3 if opt is not None else scene.A3.float()
    cond = opt.cond32 if opt is not None else scene.cond.float()
    params = [cpu(scene.RGBA[:, :3]), cpu(scene.RGBA[:, 3:]), cpu(scene.k.reshape(n, 1)), cpu(W1[:, 0:8]),
              cpu(W1[:, 8:32]), cpu(W1[:, 32:128]), cpu(scene.b1), cpu(W2), cpu(scene.b2), cpu(W3), cpu(scene.b3),
              cpu(cond), cpu(scene.features), cpu(scene.m), cpu(scene.s), cpu(scene.q)]
    state, groups = {}, []
    if opt is not None:
        segs = {s.name: i for i, s in enumerate(opt.adam.segments)}
        for g, name in enumerate(GROUP_SEGMENTS):
            m, v = opt.adam.state[segs[name]]
            state[g] = {"step": torch.tensor(float(opt.adam.t)), "exp_avg": cpu(m).reshape(params[g].shape),
                        "exp_avg_sq": cpu(v).reshape(params[g].shape)}
            groups.append({"lr": 0.0, "betas": opt.adam.betas, "eps": opt.adam.eps, "weight_decay": 0,
                           "amsgrad": False, "params": [g]})
    sd = {"state": state, "param_groups": groups}
    return tuple(params) + (sd, float(training_time))


def save(path, scene: Scene, opt=None, training_time: float = 0.0):
    torch.save(to_tuple(scene, opt, training_time), path)
