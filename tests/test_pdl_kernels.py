"""Static check of the programmatic-dependent-launch rule: every kernel that
the library launches with programmatic stream serialisation (ec_launch_k)
may start while the previous kernel on the stream is still running, so its
body must wait for that kernel (EC_PDL_ENTER / EC_PDL_WAIT, i.e.
griddepcontrol.wait) before it reads or writes memory the previous kernel
touches.  Read from the CUDA sources; no GPU needed."""
from __future__ import annotations

import re
from pathlib import Path

CSRC = Path(__file__).resolve().parent.parent / "edgecore_b200" / "csrc"


def _kernel_bodies(src: str) -> dict[str, str]:
    out = {}
    for m in re.finditer(r"__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s+)?(\w+)\s*\(", src):
        name = m.group(1)
        start = src.index("{", m.end())
        depth, i = 0, start
        while True:
            if src[i] == "{":
                depth += 1
            elif src[i] == "}":
                depth -= 1
                if depth == 0:
                    break
            i += 1
        out[name] = src[start:i + 1]
    return out


def test_pdl_launched_kernels_wait_for_their_predecessor():
    launched, bodies = set(), {}
    for f in sorted(CSRC.glob("*.cu")):
        src = f.read_text()
        bodies.update(_kernel_bodies(src))
        for m in re.finditer(r"ec_launch_k\(\s*(\w+)", src):
            launched.add(m.group(1))
    launched.discard("kern")   # the helper's own parameter name, if any
    assert launched, "no ec_launch_k call found"
    for name in sorted(launched):
        assert name in bodies, f"{name}: launched with ec_launch_k but no kernel body found"
        assert "EC_PDL_ENTER()" in bodies[name] or "EC_PDL_WAIT()" in bodies[name], \
            f"{name} is launched with programmatic serialisation but never waits for its predecessor"
