"""Source check of the rule the dependent-launch triggers rely on.

The library's kernels fire griddepcontrol.launch_dependents early (the GEMV
at its start, the others right after their own wait), so the next grid on the
stream may run beside them.  That is only safe while every kernel launched
with cudaLaunchAttributeProgrammaticStreamSerialization executes
griddepcontrol.wait (pdl_wait) before it touches memory an earlier kernel
writes.  This test finds every kernel launched through cudaLaunchKernelEx and
checks that its body calls pdl_wait(), or that its launch is a cooperative
one (the persistent decode kernel, which never carries the attribute)."""
from __future__ import annotations

import re

from conftest import PKG_DIR

CSRC = PKG_DIR / "csrc"


def _sources() -> str:
    return "\n".join(p.read_text() for p in sorted(CSRC.glob("*.cu*")) + sorted(CSRC.glob("*.h")))


def _kernel_body(src: str, name: str) -> str:
    m = re.search(r"__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s*)?" + re.escape(name) + r"\s*\(", src)
    assert m, f"kernel {name} not found"
    i = src.index("{", m.end())
    depth = 0
    for j in range(i, len(src)):
        if src[j] == "{":
            depth += 1
        elif src[j] == "}":
            depth -= 1
            if depth == 0:
                return src[i:j + 1]
    raise AssertionError(f"unterminated body of {name}")


def test_every_dependent_launch_waits():
    src = _sources()
    launched = set(re.findall(r"cudaLaunchKernelEx\(&\w+,\s*([A-Za-z_]\w*)", src))
    # `kern` variables hold instantiations of these kernels (see the launch sites)
    launched.discard("kern")
    launched |= {"gemv_kernel", "attn_prefill_kernel"}
    assert {"gemv_kernel", "gemm_tc_kernel", "quantize_x_kernel", "rmsnorm_quant_kernel"} <= launched
    for name in sorted(launched):
        body = _kernel_body(src, name)
        if name == "decode_kernel":
            assert "cudaLaunchAttributeCooperative" in src
            assert "pdl_launch_dependents" not in body
            continue
        assert "pdl_wait()" in body, f"{name} is launched as a dependent but never waits"


def test_small_kernels_trigger_after_their_wait():
    src = _sources()
    for name in re.findall(r"__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s*)?(\w+)\s*\(", src):
        body = _kernel_body(src, name)
        if "pdl_launch_dependents()" not in body or name in ("gemv_kernel",):
            continue
        assert body.index("pdl_wait()") < body.index("pdl_launch_dependents()"), name
