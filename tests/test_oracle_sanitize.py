"""The CPU oracle (oracle/*.c) under AddressSanitizer, UndefinedBehaviorSanitizer
and LeakSanitizer: tests/sanitize/oracle_harness.c drives every block type
through dequantisation and both matvecs, and a 2-layer Llama model with q/k/v
biases through the f32 and fp64 forwards and the sampler, on exact-size heap
buffers with two OpenMP threads.  The oracle checks every GPU result, so its
own memory safety is checked here, on CPU."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from conftest import REPO


def test_oracle_is_clean_under_sanitizers(tmp_path):
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    exe = tmp_path / "oracle_harness"
    cmd = [cc, "-std=c11", "-O1", "-g", "-fno-omit-frame-pointer", "-fsanitize=address,undefined",
           "-fno-sanitize-recover=all", "-mavx2", "-mfma", "-mf16c", "-ffp-contract=off", "-fopenmp",
           str(REPO / "tests" / "sanitize" / "oracle_harness.c"), str(REPO / "oracle" / "gguf_oracle.c"),
           str(REPO / "oracle" / "llama_oracle.c"), "-lm", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1", UBSAN_OPTIONS="print_stacktrace=1")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.stdout[-1000:], r.stderr[-3000:])
