"""The ctypes mirrors of the C ABI structs (flare_b200/_lib.py) have the header's layout: same size and the
same offset for every member, checked by compiling a probe against include/flare_b200.h (CPU only)."""
import ctypes
import os
import shutil
import subprocess

import pytest

from flare_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PAIRS = {"Scene": "flare_scene", "ForwardArgs": "flare_forward_args", "BackwardArgs": "flare_backward_args",
         "ViewerArgs": "flare_viewer_args", "AdamSegment": "flare_adam_segment", "AdamArgs": "flare_adam_args",
         "GatherTensor": "flare_gather_tensor", "Stats": "flare_stats", "KernelTimes": "flare_kernel_times"}


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs a C compiler")
def test_ctypes_structs_match_the_header(tmp_path):
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "flare_b200.h"', "int main(void) {"]
    expect = []
    for py, c in PAIRS.items():
        cls = getattr(_lib, py)
        lines.append(f'    printf("%zu\\n", sizeof({c}));')
        expect.append((f"sizeof({c})", ctypes.sizeof(cls)))
        for name, _ in cls._fields_:
            lines.append(f'    printf("%zu\\n", offsetof({c}, {name}));')
            expect.append((f"{c}.{name}", getattr(cls, name).offset))
    lines += ["    return 0;", "}"]
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    bad = [(what, want, g) for (what, want), g in zip(expect, got) if want != g]
    assert len(got) == len(expect) and not bad, bad
