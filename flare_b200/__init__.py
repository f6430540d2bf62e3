"""flare_b200: B200-native (sm_100a) implementation of FlaRe's differentiable render path.

Public API: `flare_b200.renderer.CPyOptiXFLARERenderer` / `GenerateRays` (the reference extension's
interface), `flare_b200.scene` (seeded synthetic workloads) and `flare_b200.dp` (data-parallel step).
The native library is built with `python -m flare_b200.build`.
"""
__version__ = "0.1.0"
