"""Data-parallel host logic on CPU with gloo ranks (world size 2): sharding, the flat gradient buffer,
the summed gradient of a sharded step equalling the single-rank gradient, and a failing rank surfacing as
an error on its peer instead of a hang.  The renderer is replaced by a CPU stand-in with the same call
signature (the CUDA renderer itself is covered by the GPU tests)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flare_b200 import dp
from flare_b200.scene import make_scene


def test_shard_rays_covers_every_ray_once():
    for views, rpv in [(8, 100), (1, 97), (2, 10)]:
        for world in (1, 2, 4, 8):
            if world > views and world % views:
                continue
            seen = {}
            for rank in range(world):
                for v, lo, cnt in dp.shard_rays(views, rpv, world, rank):
                    for i in range(lo, lo + cnt):
                        assert (v, i) not in seen
                        seen[(v, i)] = rank
            assert len(seen) == views * rpv


def test_banded_sharding_covers_every_ray_once_and_balances():
    for views, rpv in [(8, 100), (1, 97), (3, 10)]:
        for world in (1, 2, 3, 4, 8):
            seen = {}
            per_rank = []
            for rank in range(world):
                cnt_r = 0
                for v, lo, cnt in dp.shard_rays_banded(views, rpv, world, rank):
                    cnt_r += cnt
                    for i in range(lo, lo + cnt):
                        assert (v, i) not in seen
                        seen[(v, i)] = rank
                per_rank.append(cnt_r)
            assert len(seen) == views * rpv
            assert max(per_rank) - min(per_rank) <= views  # every rank has its share of every view


def test_interleaved_sharding_covers_every_ray_once():
    for views, W, H in [(8, 7, 10), (1, 5, 3), (3, 4, 9)]:
        for world in (1, 2, 3, 4, 8):
            for blk in (1, 3):
                seen = set()
                for rank in range(world):
                    for v, lo, cnt in dp.shard_rays_interleaved(views, W, H, world, rank, blk):
                        assert lo % W == 0 and ((lo // W) // blk) % world == rank and cnt % W == 0
                        for i in range(lo, lo + cnt):
                            assert (v, i) not in seen
                            seen.add((v, i))
                assert len(seen) == views * W * H


def test_grad_buffer_segments_are_aligned_views():
    g = dp.GradBuffer(37, True, "cpu")
    for name, t in g.views.items():
        base = g.flat if name not in dp.PER_PRIM else g.local
        assert (t.data_ptr() - base.data_ptr()) % 64 == 0, name
        t.fill_(1.0)
    assert g.flat.sum().item() + g.local.sum().item() == sum(t.numel() for t in g.views.values())
    # the exchanged buffer holds 80 floats per primitive, not the 110 of the expanded gradients
    assert g.views["rows"].shape == (37, dp.PRIM_ROW) and "cond" not in dict(dp.grad_layout(37, True)[0])


def scatter_rows_cpu(rows, A1, decoder, dRGB, dA, dk, dm, ds, dq, dcond):
    """CPU restatement of flare_scatter_prim_rows (row layout of include/flare_b200.h)."""
    dm += rows[:, 0:3]
    ds += rows[:, 3:5]
    dq += rows[:, 5:9]
    dRGB += rows[:, 9:12]
    dA += rows[:, 12:13]
    dk += rows[:, 13:14]
    c = dcond.shape[1]
    dcond += rows[:, 16:80] @ A1.float()[:, 32:32 + c]


class FakeRenderer:
    """CPU stand-in: renders a deterministic function of the rays and accumulates gradients that depend
    only on each ray and its dL/dI, like the real renderer (sum over rays)."""

    def SetGeometry(self, *a):
        pass

    def stats(self):
        return {"hits_composited": 0}

    def Forward_training(self, *a):
        O, v, bitmap = a[8], a[9], a[10]
        bitmap += torch.sigmoid(v * 3.0 + O)

    def Backward(self, *a, prim_rows=None):
        v, dLdI = a[9], a[19]
        rows = prim_rows
        rows[0, 9:12] += dLdI.sum(0)                 # dRGB of primitive 0
        rows[1, 0:3] += (dLdI * v).sum(0)           # dm of primitive 1
        rows[2, 16:19] += (dLdI * v * v).sum(0)     # layer-1 deltas of primitive 2 -> its descriptor gradient


def _step(world, rank, scene, n_views=4, rpv=64):
    shards = []
    g = torch.Generator().manual_seed(5)
    allv = torch.nn.functional.normalize(torch.randn(n_views * rpv, 3, generator=g), dim=1)
    target = torch.rand(n_views * rpv, 3, generator=g)
    for v, lo, cnt in dp.shard_rays(n_views, rpv, world, rank):
        sl = slice(v * rpv + lo, v * rpv + lo + cnt)
        shards.append(dp.Shard(torch.zeros(cnt, 3), allv[sl].contiguous(), target[sl].contiguous()))
    from flare_b200 import renderer
    renderer.scatter_prim_rows = scatter_rows_cpu  # the CUDA expansion, restated on the CPU
    st = dp.TrainStep(FakeRenderer(), scene, shards, n_views * rpv)
    st()
    G = st.grads
    assert G["cond"][2].abs().sum() > 0 and G["RGB"][0].abs().sum() > 0  # the rows were expanded
    return torch.cat([G.flat, G.local]).clone()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out, mode):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if mode == "fail" and rank == 1:
            raise SystemExit(3)  # this rank dies before the step's all-reduce
        flat = _step(world, rank, make_scene(16, 0))
        out[rank] = flat
    except RuntimeError as e:
        out[rank] = f"error: {type(e).__name__}"
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, mode):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, out, mode)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
        if p.is_alive():
            p.kill()
    return dict(out), [p.exitcode for p in ps]


def test_two_rank_step_equals_single_rank_step():
    ref = _step(1, 0, make_scene(16, 0))
    out, codes = _run(2, "ok")
    assert codes == [0, 0]
    for r in (0, 1):
        assert torch.allclose(out[r], ref, rtol=1e-6, atol=1e-7)


def test_failed_rank_is_reported_by_its_peer():
    out, codes = _run(2, "fail")
    assert codes[1] == 3
    assert isinstance(out.get(0), str) and out[0].startswith("error")
