"""Generates the golden vectors under tests/golden/ (run in a container that has the reference).

    python tests/golden/make_golden.py /path/to/FlaRe

lut_gridlevel.npz -- the reference's own Python LUT level (scripts/encoding_2d_benchmark.py:107-163,
    class GridLevel, use_hash=False, row-major y*R + x indexing, clamp, bilinear) evaluated on seeded
    coordinates with seeded tables, one level per resolution {16, 25, 40, 64}.  The CUDA kernel stores
    these four tables back to back as float2 (Forward_training.cu:114-194), so the oracle's LUT must
    reproduce GridLevel level by level.
grid_multires.npz -- the reference's MultiResolutionEncoding (scripts/encoding_2d_benchmark.py:174-200)
    configured as BASELINE config 0's encoder: 8 levels of floor(4 * 1.5^l) vertices per side, 2 features,
    at most 2^16 entries per level (every level fits, so it addresses row-major, unhashed), evaluated on
    seeded coordinates with a seeded table laid out level after level; the grid/SH decoder variant's
    encoding must reproduce it.
smoke_scene.npz -- the single-primitive scene of scripts/smoke_test_renderer.py:48-88 (inputs only; the
    reference test pins no numbers, the expected image is computed analytically in the tests).
"""
import math
import os
import sys

import numpy as np
import torch

OUT = os.path.dirname(os.path.abspath(__file__))


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "scripts"))
    import encoding_2d_benchmark as eb  # the reference module, imported read-only

    g = torch.Generator().manual_seed(1234)
    n = 512
    # pre-normalisation coordinates slightly beyond [-1, 1] to exercise the clamp
    cu = (torch.rand(n, generator=g) * 2.2 - 1.1).double()
    cw = (torch.rand(n, generator=g) * 2.2 - 1.1).double()
    cu[:4] = torch.tensor([-1.0, 1.0, 0.0, 1.0], dtype=torch.float64)
    cw[:4] = torch.tensor([-1.0, 1.0, 0.0, -1.0], dtype=torch.float64)
    features = (torch.rand(13154, generator=g) * 0.2 - 0.1).float()
    offs = [0, 256, 881, 2481]
    outs = []
    for l, R in enumerate(eb.BASE_RESOLUTIONS):
        lev = eb.GridLevel(R, 2, R * R, use_hash=False).double()
        with torch.no_grad():
            lev.embedding.weight.copy_(features.view(-1, 2)[offs[l]:offs[l] + R * R].double())
        coords = torch.stack([(cu.float().double() + 1.0) * 0.5, (cw.float().double() + 1.0) * 0.5], 1)
        with torch.no_grad():
            outs.append(lev(coords))
    expected = torch.cat(outs, 1).numpy()
    np.savez(os.path.join(OUT, "lut_gridlevel.npz"), cu=cu.float().numpy(), cw=cw.float().numpy(),
             features=features.numpy(), expected=expected, resolutions=np.array(eb.BASE_RESOLUTIONS))
    np.savez(os.path.join(OUT, "smoke_scene.npz"),
             m=np.array([[0.0, 0.0, 3.0]], np.float32), s=np.full((1, 2), math.log(0.75), np.float32),
             q=np.array([[1.0, 0.0, 0.0, 0.0]], np.float32),
             RGBA=np.array([[1.0, 0.0, 0.0, math.log(0.9 / 0.1)]], np.float32),
             k=np.array([[math.log(math.expm1(1.0))]], np.float32), width=8, height=8, fov=1.0,
             bg=np.array([0.01, 0.02, 0.03], np.float32))
    grid_golden(eb)
    print("wrote", OUT)


def grid_golden(eb):
    g = torch.Generator().manual_seed(4321)
    n = 512
    cu = (torch.rand(n, generator=g) * 2.2 - 1.1).float()
    cw = (torch.rand(n, generator=g) * 2.2 - 1.1).float()
    cu[:4] = torch.tensor([-1.0, 1.0, 0.0, 1.0])
    cw[:4] = torch.tensor([-1.0, 1.0, 0.0, -1.0])
    res = tuple(int(4 * 1.5 ** l) for l in range(8))
    cfg = eb.EncodingConfig("grid_sh", res, 2 ** 16, "BASELINE config-0 grid")
    enc = eb.MultiResolutionEncoding(cfg, 2).double()
    assert not any(lev.use_hash for lev in enc.levels)
    features = (torch.rand(2 * sum(r * r for r in res), generator=g) * 0.2 - 0.1).float()
    off = 0
    with torch.no_grad():
        for lev, r in zip(enc.levels, res):
            lev.embedding.weight.copy_(features.view(-1, 2)[off:off + r * r].double())
            off += r * r
        coords = torch.stack([(cu.double() + 1.0) * 0.5, (cw.double() + 1.0) * 0.5], 1)
        expected = enc(coords).numpy()
    np.savez(os.path.join(OUT, "grid_multires.npz"), cu=cu.numpy(), cw=cw.numpy(), features=features.numpy(),
             expected=expected, resolutions=np.array(res))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the FlaRe checkout>")
    main(sys.argv[1])
