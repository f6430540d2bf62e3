"""Seeded synthetic scenes and cameras for the FlaRe render path.

No dataset or checkpoint is available offline, so every workload is generated from a seed with the
distributions of the benchmark configurations (primitive centres U[-1,1]^3, unit quaternions from
normalised N(0,1), log-scales U[ln 0.005, ln 0.05], shape exponent beta U[1,4], descriptor N(0,0.1),
LUT entries U[-0.1,0.1], Xavier-uniform MLP, pinhole cameras on a radius-3 sphere looking at the
origin).  Tensor shapes and dtypes are the ones the reference renderer consumes
(source/scene/gaussian_model.py:62-88,186-204 and source/train.py:449,523,641-644):

    m (N,3) f32, s (N,2) f32 log-scale, q (N,4) f32, RGBA (N,4) f32 = [base RGB, opacity logit],
    k (N,1) f32 raw (kappa = 1 + softplus(k)), cond (N,96) f16, features (13154) f32,
    A1 (64,128) f16, b1 (64) f32, A2 (64,64) f16, b2 (64) f32, A3 (16,64) f16, b3 (16) f32.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

LUT_SIZE = 13154
COND_DIM = 96
# the dense-grid / spherical-harmonics decoder variant (BASELINE config 0's encoder): 8 grid levels of
# floor(4 * 1.5^l) vertices per side, 2 features each; 32-wide descriptor
GRID_RES = tuple(int(4 * 1.5 ** l) for l in range(8))
GRID_SIZE = 2 * sum(r * r for r in GRID_RES)
GRID_COND_DIM = 32


@dataclass
class Scene:
    m: torch.Tensor
    s: torch.Tensor
    q: torch.Tensor
    RGBA: torch.Tensor
    k: torch.Tensor
    cond: torch.Tensor
    features: torch.Tensor
    A1: torch.Tensor
    b1: torch.Tensor
    A2: torch.Tensor
    b2: torch.Tensor
    A3: torch.Tensor
    b3: torch.Tensor

    @property
    def n(self) -> int:
        return self.m.shape[0]

    def to(self, device) -> "Scene":
        return Scene(**{k: v.to(device) for k, v in self.__dict__.items()})

    def activated(self):
        """The activated tensors SetGeometry takes (train.py:449)."""
        return (self.m, torch.exp(self.s), self.q, torch.sigmoid(self.RGBA[:, 3]).contiguous(),
                (1.0 + torch.nn.functional.softplus(self.k[:, 0])).contiguous())


def _xavier(gen, fan_out, fan_in):
    bound = math.sqrt(6.0 / (fan_in + fan_out))
    return (torch.rand(fan_out, fan_in, generator=gen) * 2 - 1) * bound


def make_scene(n: int, seed: int = 0, device="cpu", extent: float = 1.0, decoder: str = "lut_pe") -> Scene:
    """Primitives with the config-0 distributions (BASELINE configs reuse them at larger N).

    decoder "lut_pe": the reference's decoder (96-wide descriptor, 13154-float LUT, W1 over 128 inputs);
    "grid_sh": the variant with a 32-wide descriptor, the 16502-float dense grid and W1 over its 64
    inputs (Xavier over fan-in 64, stored in the left half of a (64, 128) tensor)."""
    if decoder not in ("lut_pe", "grid_sh"):
        raise ValueError(f"unknown decoder {decoder!r}")
    g = torch.Generator().manual_seed(seed)
    m = (torch.rand(n, 3, generator=g) * 2 - 1) * extent
    q = torch.randn(n, 4, generator=g)
    q = q / q.norm(dim=1, keepdim=True)
    s = torch.empty(n, 2).uniform_(math.log(0.005), math.log(0.05), generator=g) + math.log(extent)
    beta = torch.empty(n, 1).uniform_(1.0, 4.0, generator=g).clamp_min(1.0 + 1e-3)
    k = torch.log(torch.expm1(beta - 1.0))                  # kappa = 1 + softplus(k) = beta
    lo, hi = math.log(0.05 / 0.95), math.log(0.95 / 0.05)
    A = torch.empty(n, 1).uniform_(lo, hi, generator=g)     # sigmoid(A) in [0.05, 0.95]
    RGB = torch.rand(n, 3, generator=g)
    grid = decoder == "grid_sh"
    cond = (torch.randn(n, GRID_COND_DIM if grid else COND_DIM, generator=g) * 0.1).to(torch.float16)
    features = torch.empty(GRID_SIZE if grid else LUT_SIZE).uniform_(-0.1, 0.1, generator=g)
    if grid:
        A1 = torch.zeros(64, 128)
        A1[:, :64] = _xavier(g, 64, 64)
        A1 = A1.to(torch.float16)
    else:
        A1 = _xavier(g, 64, 128).to(torch.float16)
    A2 = _xavier(g, 64, 64).to(torch.float16)
    A3 = _xavier(g, 16, 64).to(torch.float16)
    z = lambda c: torch.zeros(c)
    sc = Scene(m=m.contiguous(), s=s.contiguous(), q=q.contiguous(), RGBA=torch.cat([RGB, A], 1).contiguous(),
               k=k.contiguous(), cond=cond.contiguous(), features=features, A1=A1, b1=z(64), A2=A2, b2=z(64),
               A3=A3, b3=z(16))
    return sc.to(device)


def look_at_camera(eye, target=(0.0, 0.0, 0.0), up=(0.0, 1.0, 0.0)):
    """(O, R, D, F): origin, right, down, forward unit vectors (train.py:266-283 convention)."""
    eye = torch.tensor(eye, dtype=torch.float64)
    F = torch.tensor(target, dtype=torch.float64) - eye
    F = F / F.norm()
    upv = torch.tensor(up, dtype=torch.float64)
    Rv = torch.linalg.cross(F, upv)
    if Rv.norm() < 1e-9:
        Rv = torch.linalg.cross(F, torch.tensor([1.0, 0.0, 0.0], dtype=torch.float64))
    Rv = Rv / Rv.norm()
    D = torch.linalg.cross(F, Rv)
    return eye.float(), Rv.float(), D.float(), F.float()


def sphere_eye(view: int, n_views: int, radius: float = 3.0, seed: int = 0):
    """View `view` of `n_views` spread on a radius-3 sphere (golden-angle spiral, seeded offset)."""
    g = torch.Generator().manual_seed(seed + 7919)
    phase = float(torch.rand(1, generator=g)) * 2 * math.pi
    zc = 1.0 - (2.0 * view + 1.0) / (2.0 * n_views)
    zc = max(-0.9, min(0.9, zc * 0.8))
    r = math.sqrt(1.0 - zc * zc)
    th = phase + view * math.pi * (3.0 - math.sqrt(5.0))
    return (radius * r * math.cos(th), radius * zc, radius * r * math.sin(th))


def camera_rays(width: int, height: int, fov_x_deg: float = 60.0, eye=(0.0, 0.0, 3.0), device="cpu"):
    """Normalised pinhole rays of one full raster, pixel order row-major (train.py:68-89,520).

    fov_x is horizontal; fov_y follows the aspect ratio.  Returns O (R,3), v (R,3) float32."""
    O, Rv, D, F = look_at_camera(eye)
    fx = math.radians(fov_x_deg)
    fy = 2.0 * math.atan(math.tan(0.5 * fx) * height / width)
    tx, ty = 2.0 * math.tan(0.5 * fx), 2.0 * math.tan(0.5 * fy)
    ys, xs = torch.meshgrid(torch.arange(height, dtype=torch.float64), torch.arange(width, dtype=torch.float64),
                            indexing="ij")
    dx = (-0.5 + (xs.reshape(-1, 1) + 0.5) / width) * tx
    dy = (-0.5 + (ys.reshape(-1, 1) + 0.5) / height) * ty
    v = Rv.double() * dx + D.double() * dy + F.double()
    v = v / v.norm(dim=1, keepdim=True)
    O = O.double().expand_as(v)
    return O.float().contiguous().to(device), v.float().contiguous().to(device)


def viewer_spheres():
    """Config-4 stand-in for the reference viewer's meshes: a mirror and two glass spheres (IOR 1.5)
    between the default camera (0, 0, 3) and the primitive cube, so that the refracted and reflected rays
    travel into the primitives.  Returns (spheres (3,4) centre + radius, materials (3,6)); material rows
    are the reference viewer's (Id rgb, kd, eta, n), the mirror an extreme-IOR dielectric (R0 -> 1, the
    refracted child carries no transmittance)."""
    spheres = torch.tensor([[-0.55, 0.0, 1.5, 0.35], [0.5, 0.1, 1.45, 0.32], [0.0, 0.55, 1.3, 0.25]])
    materials = torch.tensor([[0.9, 0.9, 0.9, 0.0, 1.0e6, 64.0],
                              [0.75, 0.88, 1.0, 0.03, 1.5, 64.0],
                              [0.95, 0.8, 0.7, 0.03, 1.5, 64.0]])
    return spheres, materials


def viewer_lights():
    """One white directional light along normalised (1, 1, 1) (the reference viewer's default,
    source/viewer.py:72-76,194-196): rows (Is rgb, direction)."""
    d = torch.tensor([1.0, 1.0, 1.0])
    d = d / d.norm()
    return torch.cat([torch.ones(3), d]).reshape(1, 6)
