"""The C ABI library without a GPU: it builds for sm_100a, loads, exports
every entry point include/b2q.h declares, and fails cleanly (a status code,
no crash) when no device is present.  Plus host-side logic of the mirror."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "b2q.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(b2q_[a-z0-9_]+)\s*\(", text))


def test_library_builds_and_exports_all_symbols(pkg):
    from hf_llm_b200 import _lib, build
    path = build.build()
    assert path.exists()
    lib = C.CDLL(str(path))
    missing = [s for s in sorted(declared_symbols()) if not hasattr(lib, s)]
    assert not missing, f"declared but not exported: {missing}"
    bound = {name for name, _, _ in _lib.SIGNATURES}
    assert declared_symbols() <= bound, declared_symbols() - bound


def test_checks_build_exports_all_symbols(pkg):
    """The debug-bounds twin (-DB2Q_CHECKS) has the same ABI and says so;
    the regular library has its checks compiled out."""
    from hf_llm_b200 import build
    path = build.build(checks=True)
    assert path.exists() and path != build.lib_path()
    lib = C.CDLL(str(path))
    missing = [s for s in sorted(declared_symbols()) if not hasattr(lib, s)]
    assert not missing, f"declared but not exported: {missing}"
    assert lib.b2q_debug_checks_enabled() == 1
    assert C.CDLL(str(build.build())).b2q_debug_checks_enabled() == 0


def test_kernels_compiled_for_sm100a(pkg):
    from hf_llm_b200 import build
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.NVCC_FLAGS)


def test_init_without_device_returns_status(pkg):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from hf_llm_b200 import _lib
    h = C.c_void_p()
    st = _lib.lib().b2q_init(0, C.byref(h))
    assert st != _lib.OK
    assert _lib.lib().b2q_last_error()


def test_null_arguments_rejected(pkg):
    from hf_llm_b200 import _lib
    L = _lib.lib()
    assert L.b2q_init(0, None) == _lib.EINVAL
    assert L.b2q_matmul(None, None, None, None, 1, 1, 1) == _lib.EINVAL
    assert L.b2q_forward(None, None, 1, 0, None, None) == _lib.EINVAL
    assert L.b2q_model_create(None, None, None, None) == _lib.EINVAL


def test_safe_alloc_policy_mirrors_reference(pkg):
    """can_safely_alloc (gpu.rs:403-437): <= 58 % of VRAM offloaded and
    max(total/5, 1600 MiB) kept free."""
    from hf_llm_b200.engine import CudaEngine
    G = 1024 ** 3
    pol = CudaEngine.safe_alloc_policy
    assert pol(0, 0, 8 * G, 0)
    assert pol(1 * G, 6 * G, 8 * G, 0)
    assert not pol(1 * G, 2 * G, 8 * G, 0)             # would eat the reserve
    assert not pol(1 * G, 100 * G, 180 * G, 104 * G)   # past 58 %
    assert pol(1 * G, 100 * G, 180 * G, 90 * G)


def test_ggml_type_table(pkg):
    from hf_llm_b200 import ggml
    assert ggml.row_bytes(ggml.Q8_0, 4096) == 4352
    assert ggml.row_bytes(ggml.Q4_K, 4096) == 2304 and ggml.row_bytes(ggml.Q4_K, 14336) == 8064
    assert ggml.row_bytes(ggml.Q6_K, 4096) == 3360 and ggml.row_bytes(ggml.Q6_K, 14336) == 11760
    with pytest.raises(ValueError):
        ggml.from_u32(4)
    with pytest.raises(ValueError):
        ggml.row_bytes(ggml.Q4_K, 100)


def test_header_is_plain_c_and_links_from_c(pkg, tmp_path):
    """The boundary is for foreign-function callers (Rust extern "C", cgo,
    ctypes): the header must compile as strict C99, and a C program must link
    against the library and call it (version string; init without a device
    or on a bad device id returns a status and an error message)."""
    import shutil
    import subprocess
    from hf_llm_b200 import build
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    lib = build.build()
    src = tmp_path / "abi.c"
    src.write_text(
        '#include <stdio.h>\n#include "b2q.h"\n'
        "int main(void) {\n"
        "  b2q_engine* e = NULL;\n"
        "  b2q_status s = b2q_init(-1, &e);\n"
        '  printf("%s|%d|%d|%s\\n", b2q_version(), (int)s, e == NULL, b2q_last_error());\n'
        "  return s == B2Q_OK;\n"
        "}\n")
    exe = tmp_path / "abi"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", f"-I{HEADER.parent}",
                    str(src), "-o", str(exe), f"-L{lib.parent}", "-lb2q", f"-Wl,-rpath,{lib.parent}"],
                   check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    version, status, null_out, err = r.stdout.strip().split("|", 3)
    assert version.startswith("b2q") and int(status) != 0 and null_out == "1" and err
