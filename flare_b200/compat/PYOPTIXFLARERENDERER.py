"""Drop-in module with the reference extension's import name.

The reference callers (train.py:62-65, evaluate.py, render_style.py, extract_mesh.py) put the
extension's output folder on sys.path and `import PYOPTIXFLARERENDERER`.  Putting this folder there
instead gives them the B200 renderer with the same class and function names.
"""
import os
import sys

try:
    import flare_b200  # noqa: F401
except ImportError:  # repository checkout: make the package importable
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from flare_b200.renderer import CPyOptiXFLARERenderer, GenerateRays  # noqa: E402,F401

__all__ = ["CPyOptiXFLARERenderer", "GenerateRays"]
