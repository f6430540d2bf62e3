"""Drop-in module with the reference viewer extension's import name (source/viewer.py:166-170 imports
PYOPTIXFLAREVIEWER).  The class keeps the reference's constructor and Forward; SetGeometry takes a
(S,4) tensor of analytic spheres (centre, radius) where the reference takes mesh instances and hitgroup
records, and Forward drops the mesh normal matrices (M4N)."""
import os
import sys

try:
    import flare_b200  # noqa: F401
except ImportError:  # repository checkout: make the package importable
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from flare_b200.renderer import GenerateRays  # noqa: E402,F401
from flare_b200.viewer import CPyFlareViewerRenderer as CPyOptiXFLAREVIEWERRenderer  # noqa: E402,F401

__all__ = ["CPyOptiXFLAREVIEWERRenderer", "GenerateRays"]
