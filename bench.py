"""Benchmark of the B200 FlaRe render path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl flare|reference] [--config 2|3]

Workload (seeded synthetic data; no dataset is available offline):
  config 3 (default): data-parallel training step, 6M primitives, 8 views of 1920x1080 on a radius-3
      sphere (strong scaling: the same 16.6M rays at every N); every rank takes the same row band of every
      view and renders its bands as one ray batch (FLARE_BENCH_SHARDING=views: whole views per rank,
      =rows[:B]: row blocks dealt round-robin); one NCCL all-reduce of the flat gradient buffer per step.
  config 2: training step, 3M primitives, one 1600x1064 view (rays split in row bands over ranks).
A step = SetGeometry (LBVH rebuild, as the reference rebuilds its IAS every step) + Forward_training +
L1 loss / dL/dI in torch + Backward (+ all-reduce).  At N=1 the line also carries the config-2
training step (the single-GPU target) and the config-1 forward render.

value: Mrays/s of the whole job, inputs resident on the device; e2e: the same step through the
public renderer API with the step's rays and target copied from pinned host memory and the loss read
back every step.  Timing: CUDA events on the step's stream, barrier + synchronize on both sides, max
over ranks.  Inputs (scene >= 0.75 GB) are larger than the 126 MB L2.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    1: dict(n_prims=1_000_000, width=800, height=800, views=1, mode="forward"),
    2: dict(n_prims=3_000_000, width=1600, height=1064, views=1, mode="train"),
    3: dict(n_prims=6_000_000, width=1920, height=1080, views=8, mode="train"),
    # secondary rays: 1M primitives + a mirror and two glass spheres, recursion depth 3, forward only
    4: dict(n_prims=1_000_000, width=1024, height=1024, views=1, mode="viewer", depth=3),
}
METRIC = "Mrays/s fwd and fwd+bwd at 1/2/4/8 B200; % of traversal/MLP roofline"
# algorithmic bytes per composited hit / per ray and FLOPs per hit (roofline model of the path)
B_HIT_TRACE = 64                 # one 64-B node per composited hit
B_HIT_FWD = 56 + 192             # primitive record + fp16 descriptor row
B_HIT_BWD = 56 + 192 + 440       # re-read + gradient writes (14 geometry + 96 descriptor fp32)
B_RAY_FWD, B_RAY_BWD = 44, 24
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per composited hit of each timed kernel, from a
# one-pass ncu capture of this build over the config-3 bench workload itself (bytes per step / 1.0224e9 hits
# per step); the bench scales it by the hits of its own launches, which reproduces the measured per-launch
# traffic on config 3.
DRAM_BYTES_PER_HIT = {"trace": 16.2, "shade_forward": 17.8, "shade_backward": 20.2}
FLOP_HIT_FWD = 2 * (128 * 64 + 64 * 64 + 64 * 4)
T_THR_FORWARD = 1e-4  # BASELINE config 1's early-termination threshold


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except Exception:
                continue
            for nm, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":  # the CPU arm: rank 0 alone works, no device and no process group needed
        return world, rank, local
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def build_workload(cfg, world, rank, device, seed=0, decoder="lut_pe", sharding=None):
    """Scene + this rank's rays.  sharding "banded" (default): the rank's contiguous row band of every view,
    concatenated into one ray batch (one renderer call per step); "rows[:B]": blocks of B image rows of
    every view dealt round-robin over the ranks, one batch; "views": whole views dealt round-robin, one
    batch per view.  Measured per-rank compute at 8 ranks (config 3, emulated on one GPU): banded 121-139 ms,
    rows:68 122-139, rows:34 125-142, rows:1 158-160 (every 8th row: incoherent packets)."""
    from flare_b200.dp import Shard, shard_rays, shard_rays_banded, shard_rays_interleaved
    from flare_b200.scene import camera_rays, make_scene, sphere_eye
    c = CONFIGS[cfg]
    sharding = sharding or os.environ.get("FLARE_BENCH_SHARDING", "banded")
    scene = make_scene(c["n_prims"], seed, decoder=decoder).to(device)
    W, H, V = c["width"], c["height"], c["views"]
    host = []
    if sharding.startswith("rows"):  # "rows" or "rows:<block rows>"
        blk = int(sharding.split(":")[1]) if ":" in sharding else max(1, -(-H // (4 * world)))
        pieces = shard_rays_interleaved(V, W, H, world, rank, blk)
    elif sharding == "banded":
        pieces = shard_rays_banded(V, W * H, world, rank)
    else:
        pieces = shard_rays(V, W * H, world, rank)
    by_view = {}
    for view, lo, cnt in pieces:
        by_view.setdefault(view, []).append((lo, cnt))
    for view, rng in by_view.items():
        eye = sphere_eye(view, V) if V > 1 else (0.0, 0.0, 3.0)
        O, v = camera_rays(W, H, 60.0, eye=eye)
        g = torch.Generator().manual_seed(1000 + view)
        target = torch.rand(W * H, 3, generator=g)
        sel = torch.cat([torch.arange(lo, lo + cnt) for lo, cnt in rng])
        if sharding == "views":
            host += [tuple(t[lo:lo + cnt].contiguous() for t in (O, v, target)) for lo, cnt in rng]
        else:
            host.append(tuple(t[sel].contiguous() for t in (O, v, target)))
    if sharding != "views" and len(host) > 1:
        host = [tuple(torch.cat([h[k] for h in host]) for k in range(3))]
    host = [tuple(t.pin_memory() for t in h) for h in host]
    shards = [Shard(*(t.to(device) for t in h)) for h in host]
    return scene, shards, host, W * H * V


def time_steps(fn, steps, world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        fn()
    e1.record(st)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def path_roofline(hits, rays, ms, hbm, tflops, backward=True):
    """Roofline of the whole path (north star): the slower of its algorithmic bytes over HBM bandwidth
    and its decoder FLOPs over the tensor peak.  Forward: 312 B + 25088 FLOP per composited hit and 44 B per
    ray; forward + backward: 1064 B + 100352 FLOP per hit and 68 B per ray."""
    if backward:
        nbytes = hits * (2 * B_HIT_TRACE + B_HIT_FWD + B_HIT_BWD) + rays * (B_RAY_FWD + B_RAY_BWD)
        flops = hits * 4 * FLOP_HIT_FWD
    else:
        nbytes = hits * (B_HIT_TRACE + B_HIT_FWD) + rays * B_RAY_FWD
        flops = hits * FLOP_HIT_FWD
    t_mem, t_flop = nbytes / (hbm * 1e9), flops / (tflops * 1e12)
    t_roof = max(t_mem, t_flop)
    return {"roofline_ms": t_roof * 1e3, "frac": t_roof / (ms * 1e-3), "algo_bytes": nbytes, "flops": flops,
            "bound": "hbm" if t_mem >= t_flop else "tensor",
            "note": ("1064 B + 100352 FLOP per composited hit, 68 B per ray" if backward else
                     "312 B + 25088 FLOP per composited hit, 44 B per ray") + "; peaks of MEASURED_PEAKS.json"}


def kernel_roofline(kt, hits, rays, hbm, traversals=1.0):
    """Achieved GB/s of each kernel = algorithmic bytes / kernel time; the dominant one is returned.
    `traversals` = traversals of the hit lists per step (1 when the backward replays the forward's cached
    hits, 2 when it traces again)."""
    algo = {
        "trace": traversals * hits * B_HIT_TRACE,
        "shade_forward": hits * B_HIT_FWD + rays * B_RAY_FWD,
        "shade_backward": hits * B_HIT_BWD + rays * B_RAY_BWD,
    }
    out = {}
    for k, b in algo.items():
        ms, n = kt.get(k, (0.0, 0))
        if ms > 0:
            out[k] = dict(ms=ms, launches=n, algo_bytes=b, achieved_gbs=b / (ms * 1e-3) / 1e9)
    dom = max(out, key=lambda k: out[k]["ms"]) if out else None
    return dom, out


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuPort:
    """The reference's path on the host cores, from the CPU port in oracle/ (the reference itself needs
    OptiX and an RT-core GPU): a C hierarchy over the primitives (built once, the SetGeometry analogue),
    then per step, for a fixed block of rays of the workload's first view: the multi-pass 16-nearest
    traversal with the reference's restarts, decode + composite after every pass until each ray terminates
    (C, OpenMP over all host cores), and -- training workloads -- the backward over the composited hit lists
    (torch autograd, float64)."""

    def __init__(self, cfg, sample_rays=16384, seed=0):
        import numpy as np

        from flare_b200.scene import camera_rays, make_scene, sphere_eye
        from oracle import oracle
        self.cfg = cfg
        c = CONFIGS[cfg]
        self.sc = make_scene(c["n_prims"], seed)
        W, H, V = c["width"], c["height"], c["views"]
        O, v = camera_rays(W, H, 60.0, eye=sphere_eye(0, V) if V > 1 else (0.0, 0.0, 3.0))
        side = int(math.ceil(math.sqrt(sample_rays)))
        cy, cx = H // 2 - side // 2, W // 2 - side // 2  # a centred block: these rays cross the scene
        idx = [(cy + dy) * W + (cx + dx) for dy in range(side) for dx in range(side)][:sample_rays]
        self.O, self.v = O[idx].numpy(), v[idx].numpy()
        self.target = np.random.RandomState(seed).rand(len(idx), 3).astype(np.float32)
        t0 = time.perf_counter()
        self.frames = oracle.prep_frames(*self.sc.activated())
        self.bvh = oracle.CpuBvh(self.frames)
        self.build_s = time.perf_counter() - t0
        self.train = c["mode"] == "train"
        self.T_thr = 1e-4

    def step(self):
        import numpy as np

        from oracle import grad_oracle
        t1 = time.perf_counter()
        rgb, csr, nh, tr_s, sh_s = self.bvh.render(self.sc, self.O, self.v, "training", T_thr=self.T_thr,
                                                    reg_a=-0.1 * 1000 / 999.9, reg_b=1000 / 999.9)
        img = np.clip(rgb, 0, 1)
        dLdI = (np.sign(img - self.target) / (3 * len(self.O))).astype(np.float32)
        t2 = time.perf_counter()
        if self.train:
            grad_oracle.gradients(self.sc, self.O, self.v, csr, nh, dLdI, compact=True)
        t3 = time.perf_counter()
        self.last = (t2 - t1, t3 - t2, int(nh.sum()), tr_s, sh_s)
        return t3 - t1

    def describe(self):
        fwd, bwd, hits, tr_s, sh_s = self.last
        c = CONFIGS[self.cfg]
        return (f"{len(self.O)} central rays of config {self.cfg} view 0 per step ({hits} composited hits), "
                f"{c['n_prims']} primitives, T_threshold {self.T_thr}; host {cpu_model()}, {os.cpu_count()} "
                f"threads. Forward: C hierarchy traversal (16-nearest passes, reference restarts) + C decode / "
                f"composite, OpenMP over rays, {fwd:.2f} s ({tr_s:.1f} thread-s traversal, {sh_s:.1f} thread-s "
                f"shading); backward: torch fp64 autograd over the composited hit lists, {bwd:.2f} s; hierarchy "
                f"build {self.build_s:.2f} s once (not in the step)")


def cpu_baseline(cfg, sample_rays=16384, steps=1):
    port = CpuPort(cfg, sample_rays)
    ts = [port.step() for _ in range(steps)]
    t = statistics.median(ts)
    return dict(value=len(port.O) / t / 1e6, unit="Mrays/s", cores=os.cpu_count(), kind="port",
                sample=port.describe())


def run_reference(args, world, rank):
    if rank != 0:
        return
    port = CpuPort(args.config, args.ref_rays)
    ts = []
    for i in range(args.warmup + args.steps):
        t = port.step()
        if i >= args.warmup:
            ts.append(t)
    v = len(port.O) / statistics.median(ts) / 1e6
    cb = dict(value=v, unit="Mrays/s", cores=os.cpu_count(), kind="port", sample=port.describe())
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "Mrays/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.median(ts) * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, BASELINE.json distributions)",
            "config": {"workload": f"config {args.config} ({CONFIGS[args.config]['n_prims']} primitives), "
                                   f"{args.ref_rays}-ray sample per step", "sample_rays": args.ref_rays},
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "Mrays/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def measure_viewer(cfg, scene, sh, steps, warmup, device, world):
    """Config 4: the secondary-ray forward (reflection, refraction, shadows) of one view."""
    from flare_b200.scene import viewer_lights, viewer_spheres
    from flare_b200.viewer import CPyFlareViewerRenderer
    c = CONFIGS[cfg]
    R = sh.O.shape[0]
    r = CPyFlareViewerRenderer(8, 11.3449, R, c["depth"])
    spheres, materials = viewer_spheres()
    r.SetGeometry(scene.m, torch.exp(scene.s), scene.q, torch.sigmoid(scene.RGBA[:, 3]).contiguous(),
                  (1.0 + torch.nn.functional.softplus(scene.k[:, 0])).contiguous(), spheres)
    RGB, A = scene.RGBA[:, :3].contiguous(), scene.RGBA[:, 3].contiguous()
    dec = (scene.cond, scene.features, RGB, scene.A1, scene.b1, scene.A2, scene.b2, scene.A3, scene.b3)
    bitmap = torch.zeros(R, 3, device=device)
    lights = viewer_lights()

    def fwd():
        bitmap.zero_()
        r.Forward(*dec, sh.O, sh.v, bitmap, 0.0, 0.0, 0.0, scene.m, scene.s, scene.q, A, scene.k, 0.01, materials,
                  lights, 1e-4, 0.55, 0.06, 0.06, 0.07)
    for _ in range(warmup):
        fwd()
    ms = time_steps(fwd, steps, world) / steps
    r.profile(True)
    fwd()
    torch.cuda.synchronize()
    kt = r.kernel_times()
    r.profile(False)
    return dict(workload=f"config {cfg} secondary-ray forward (depth {c['depth']}, 3 spheres)", ms_per_step=ms,
                value=R / (ms * 1e-3) / 1e6, traversal_passes=r.stats()["passes"],
                kernels={k: dict(ms=v[0], launches=v[1]) for k, v in kt.items() if v[1]})


def measure_config(cfg, world, rank, steps, warmup, device, hbm, tflops, profile=True, decoder="lut_pe"):
    from flare_b200.dp import TrainStep
    from flare_b200.renderer import CPyOptiXFLARERenderer
    scene, shards, host, total_rays = build_workload(cfg, world, rank, device, decoder=decoder)
    tag = "" if decoder == "lut_pe" else f", {decoder} decoder"
    if CONFIGS[cfg]["mode"] == "viewer":
        return measure_viewer(cfg, scene, shards[0], steps, warmup, device, world)
    max_rays = max(s.O.shape[0] for s in shards)
    r = CPyOptiXFLARERenderer(8, 11.3449, max_rays)
    out = {}
    if CONFIGS[cfg]["mode"] == "forward":
        sh = shards[0]
        bitmap = torch.zeros(sh.O.shape[0], 3, device=device)
        r.SetGeometry(scene.m, torch.exp(scene.s), scene.q, torch.sigmoid(scene.RGBA[:, 3]).contiguous(),
                      (1.0 + torch.nn.functional.softplus(scene.k[:, 0])).contiguous())
        dec = (scene.cond, scene.features, scene.A1, scene.b1, scene.A2, scene.b2, scene.A3, scene.b3)
        normal = torch.zeros_like(bitmap)
        alpha = torch.zeros(sh.O.shape[0], device=device)
        edn = torch.zeros_like(alpha)

        def fwd():
            bitmap.zero_(); normal.zero_(); edn.zero_()
            r.Forward_inference_with_geometry(*dec, sh.O, sh.v, bitmap, normal, alpha, edn, 0.0, 0.0, 0.0, scene.m,
                                              scene.s, scene.q, scene.RGBA, scene.k, T_THR_FORWARD)
        for _ in range(warmup):
            fwd()
        ms = time_steps(fwd, steps, world) / steps
        hits = r.stats()["hits_composited"]
        r.profile(True)
        fwd()
        torch.cuda.synchronize()
        kt = r.kernel_times()
        r.profile(False)
        R = sh.O.shape[0]
        out = dict(workload=f"config {cfg} forward (Forward_inference_with_geometry, T_threshold {T_THR_FORWARD})",
                   ms_per_step=ms, value=total_rays / (ms * 1e-3) / 1e6, hits_per_ray=hits / R,
                   kernels={k: dict(ms=v[0], launches=v[1]) for k, v in kt.items() if v[1]},
                   roofline=path_roofline(hits, R, ms, hbm, tflops, backward=False))
        return out
    step = TrainStep(r, scene, shards, total_rays)
    for _ in range(warmup):
        step()
    ms = time_steps(step, steps, world) / steps
    # profiled steps (per-kernel CUDA events + hit counts), outside the headline timing
    step.collect_stats = True
    step.hits = 0
    step.fwd_passes = 0
    r.profile(True)
    time_steps(step, 1, world)
    kt = r.kernel_times()
    r.profile(False)
    step.collect_stats = False
    hits = step.hits
    my_rays = sum(s.O.shape[0] for s in shards)
    traversals = kt.get("trace", (0.0, 0))[1] / max(step.fwd_passes, 1)  # 1.0 when the backward replays
    dom, per = kernel_roofline(kt, hits, my_rays, hbm, traversals)
    step_bytes = hits * (2 * B_HIT_TRACE + B_HIT_FWD + B_HIT_BWD) + my_rays * (B_RAY_FWD + B_RAY_BWD)
    out = dict(workload=f"config {cfg} training step{tag}", ms_per_step=ms, value=total_rays / (ms * 1e-3) / 1e6,
               hits_per_ray=hits / max(my_rays, 1), hits=hits, kernels=per, dominant=dom, step_algo_bytes=step_bytes,
               traversals_per_step=traversals,
               kernel_times={k: v for k, v in kt.items()}, grad_allreduce_bytes=step.grads.nbytes,
               step_roofline=path_roofline(hits, my_rays, ms, hbm, tflops))
    # end to end: rays and target from pinned host memory every step, loss read back every step
    def e2e_step():
        for sh, h in zip(shards, host):
            for dst, src in zip((sh.O, sh.v, sh.target), h):
                dst.copy_(src, non_blocking=True)
        return float(step().item())
    for _ in range(1):
        e2e_step()
    ms_e2e = time_steps(e2e_step, steps, world) / steps
    out["e2e"] = dict(value=total_rays / (ms_e2e * 1e-3) / 1e6, unit="Mrays/s",
                      h2d_bytes_per_step=sum(sum(t.numel() * t.element_size() for t in h) for h in host),
                      d2h_bytes_per_step=4)
    out["_r"] = r
    out["shards"] = [(s.O.shape[0]) for s in shards]
    if decoder != "lut_pe":  # the reference's optimizer groups describe its own decoder's W1 blocks
        return out
    # the optimizer step after the backward (reference train.py:833-953): one fused Adam launch over the
    # 16 parameter groups; not part of the headline step (the reference's metric is fwd + bwd)
    from flare_b200.optim import ModelOptimizer
    opt = ModelOptimizer(scene, step.grads)
    it = [0]

    def ostep():
        it[0] += 1
        opt.step(it[0])
    for _ in range(2):
        ostep()
    ms_opt = time_steps(ostep, steps, world) / steps
    elems = sum(sg.grad.numel() for sg in opt.adam.segments)
    half = sum(sg.grad.numel() for sg in opt.adam.segments if sg.mirror is not None)
    obytes = elems * 28 + half * 2  # p, m, v read + write, g read; fp16 mirrors written
    out["optimizer_step"] = dict(ms=ms_opt, elements=elems, algo_bytes=obytes,
                                 achieved_gbs=obytes / (ms_opt * 1e-3) / 1e9)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="flare", choices=["flare", "reference"])
    ap.add_argument("--config", type=int, default=3, choices=[2, 3])
    ap.add_argument("--ref-rays", type=int, default=4096)
    ap.add_argument("--no-extra", action="store_true", help="skip the config-1/2 extras and the CPU baseline")
    args = ap.parse_args()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    device = torch.device(f"cuda:{torch.cuda.current_device()}")
    hbm, tflops, tflops_sus, peak_kind = peaks()
    smi_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else local
    main_cfg = args.config
    # warm-up + timed steps of the headline workload, clocks sampled meanwhile
    with ClockSampler(smi_index) as cs:
        res = measure_config(main_cfg, world, rank, args.steps, args.warmup, device, hbm, tflops_sus)
    clocks = cs.summary()
    extras = {}
    if world == 1 and not args.no_extra:
        runs = [(2, "lut_pe")] if main_cfg == 3 else []
        runs += [(1, "lut_pe"), (4, "lut_pe"), (2, "grid_sh")]
        for c, dk in runs:
            e = measure_config(c, 1, 0, max(2, args.steps), 3, device, hbm, tflops_sus, decoder=dk)
            e.pop("_r", None)
            extras[f"config{c}" + ("" if dk == "lut_pe" else f"_{dk}")] = {
                k: v for k, v in e.items() if k in ("workload", "ms_per_step", "value", "hits_per_ray", "dominant",
                                                    "kernels", "traversal_passes", "optimizer_step", "roofline",
                                                    "step_roofline")}
    if rank != 0:
        dist.destroy_process_group()
        return
    per = res["kernels"]
    dom = res["dominant"]
    d = per[dom]
    roof = {"bound": "hbm", "kernel": dom, "achieved": d["achieved_gbs"], "peak": hbm, "unit": "GB/s",
            "frac": d["achieved_gbs"] / hbm,
            "traffic": (DRAM_BYTES_PER_HIT[dom] * res["hits"] / max(d["launches"], 1)
                        if DRAM_BYTES_PER_HIT.get(dom) else None),
            "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
            if peak_kind == "measured" else "fallback 6.65 TB/s",
            "algo_bytes_per_launch": d["algo_bytes"] / max(d["launches"], 1),
            "avg_launch_ms": d["ms"] / max(d["launches"], 1)}
    # whole-step roofline of the path: the slower of algorithmic bytes / HBM and decoder FLOPs / tensor peak
    step_roof = dict(res["step_roofline"], note=res["step_roofline"]["note"] + "; per rank")
    line = {
        "metric": METRIC, "value": res["value"], "unit": "Mrays/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (decoder f16 tensor-core operands, f32 accumulate)",
        "data": "synthetic (seeded; BASELINE.json configs; random-init decoder)",
        "config": {"workload": res["workload"], "primitives": CONFIGS[main_cfg]["n_prims"],
                   "rays_per_step": CONFIGS[main_cfg]["width"] * CONFIGS[main_cfg]["height"] * CONFIGS[main_cfg]["views"],
                   "views": CONFIGS[main_cfg]["views"], "parallelism": f"dp{world} (rays sharded, scene replicated)",
                   "sharding": os.environ.get("FLARE_BENCH_SHARDING", "banded"),
                   "l2": "inputs larger than L2 (scene >= 0.75 GB); no flush",
                   "hits_per_ray": res["hits_per_ray"], "grad_allreduce_bytes": res["grad_allreduce_bytes"]},
        "roofline": roof,
        "step_roofline": step_roof,
        "kernels": {k: {"ms": v["ms"], "launches": v["launches"], "achieved_gbs": v["achieved_gbs"]}
                    for k, v in per.items()},
        "e2e": res["e2e"],
        "optimizer_step": res.get("optimizer_step"),
        "clocks": clocks,
        # own kernels per step: traversal + shading launches (counted), 6 build kernels per SetGeometry, 1 ray
        # init per call, 3 backward helpers; the CUB radix sort's own launches are not counted
        "gpu_launches": int(args.steps * (res["kernel_times"]["trace"][1] + res["kernel_times"]["shade_forward"][1]
                                          + res["kernel_times"]["shade_backward"][1]
                                          + 6 * res["kernel_times"]["build"][1] + 5 * len(res["shards"]))),
    }
    if extras:
        line["extra_configs"] = extras
    if world == 1 and not args.no_extra:
        try:
            line["cpu_baseline"] = cpu_baseline(main_cfg, sample_rays=16384, steps=1)
        except Exception as ex:  # the baseline is reported, never required
            line["cpu_baseline"] = {"error": str(ex)}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
