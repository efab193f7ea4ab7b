"""The GGUF parser (csrc/gguf.cuh, host code) under AddressSanitizer and
UndefinedBehaviorSanitizer, on CPU.

GGUF files come from outside, so the parser must reject every malformed one
without reading past the file or letting a size wrap around.  The harness
(tests/sanitize/gguf_parse_harness.cpp) parses each case from an exact-size
heap copy and checks the invariants the loader relies on; here it runs on a
small Llama-shaped file, every prefix of it and every header byte mutated, and
on hand-made files whose tensor dims multiply past 64 bits."""
from __future__ import annotations

import shutil
import subprocess

import numpy as np
import pytest

import gguf_fixtures as gf
from conftest import PKG_DIR, REPO

HARNESS = REPO / "tests" / "sanitize" / "gguf_parse_harness.cpp"


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    exe = tmp_path_factory.mktemp("san") / "gguf_parse_harness"
    cmd = [cxx, "-std=c++17", "-O1", "-g", "-fno-omit-frame-pointer", "-fsanitize=address,undefined",
           "-fno-sanitize-recover=all", "-include", "algorithm", "-x", "c++", "-I", str(PKG_DIR / "csrc"),
           str(HARNESS), "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0 and "sanitize" in r.stderr and "cannot find" in r.stderr:
        pytest.skip("no sanitizer runtime")
    assert r.returncode == 0, r.stderr[-3000:]
    return exe


def _run(exe, mode, path):
    r = subprocess.run([str(exe), mode, str(path)], capture_output=True, text=True, timeout=600,
                       env={"ASAN_OPTIONS": "detect_leaks=1:abort_on_error=0", "UBSAN_OPTIONS": "print_stacktrace=1"})
    assert r.returncode == 0, (r.stdout[-1000:], r.stderr[-3000:])
    return r.stdout.strip()


def _small_llama(version: int):
    rng = np.random.default_rng(5)
    kvs = [("general.architecture", gf.STRING, "llama"), ("llama.block_count", gf.U32, 1),
           ("llama.embedding_length", gf.U32, 256), ("general.alignment", gf.U32, 32),
           ("tokenizer.ggml.tokens", gf.ARRAY, ["a", "bc", "def"], gf.STRING),
           ("llama.rope.freq_base", gf.F32, 500000.0)]
    tensors = [("token_embd.weight", 12, [4, 256], rng.integers(0, 256, 4 * 144, dtype=np.uint8).tobytes()),
               ("output_norm.weight", 0, [256], rng.standard_normal(256).astype(np.float32).tobytes()),
               ("blk.0.attn_norm.weight", 1, [256], rng.standard_normal(256).astype(np.float16).tobytes())]
    return gf.raw_bytes(version, kvs, tensors)[0]


@pytest.mark.parametrize("version", [1, 3])
def test_every_prefix_and_header_mutation(harness, tmp_path, version):
    p = tmp_path / f"v{version}.gguf"
    p.write_bytes(_small_llama(version))
    assert _run(harness, "one", p) == "ok"
    out = _run(harness, "fuzz", p)
    acc, rej = int(out.split()[1]), int(out.split()[3])
    assert rej > len(p.read_bytes()) // 2 and acc >= 0


@pytest.mark.parametrize("dims", [
    [1 << 42, 1 << 43, 1 << 43],           # 2^128 elements: a 128-bit product wraps to zero
    [3, 3074457345618258603, 16],           # outer dims multiply to 2^63 + 1 in 64 bits
    [(1 << 63) - 1, 4, 2],                  # past 2^64
])
def test_dims_that_overflow_are_rejected(harness, tmp_path, dims):
    raw = gf.raw_bytes(3, [("general.architecture", gf.STRING, "llama")],
                       [("blk.0.attn_norm.weight", 1, dims, b"\0" * 64, 0)])[0]
    p = tmp_path / "overflow.gguf"
    p.write_bytes(raw)
    out = _run(harness, "one", p)
    assert out.startswith("rejected:") and "overflow" in out, out
