"""Host-side pieces of bench.py that need no GPU: the reference governor's
thread rule (hardware.rs:157-166) and the per-shape CPU matvec timing that
sits beside the GPU's gemv_shapes in the bench line."""
from __future__ import annotations

import importlib.util

from conftest import REPO


def _bench():
    spec = importlib.util.spec_from_file_location("b2q_bench", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_governor_threads_rule():
    b = _bench()
    # min(3/4 cores, cores - 2), at least one thread
    assert [b.governor_threads(c) for c in (1, 2, 3, 4, 8, 16, 32, 112)] == [1, 1, 1, 2, 6, 12, 24, 84]


def test_cpu_matvec_shape_reports_every_thread_count(pkg, orc):
    from hf_llm_b200 import synth
    b = _bench()
    r = b.cpu_matvec_shape(orc, synth, "q4k_1024x4096", 7, [1, 2], min_s=0.0, max_reps=2)
    t, n, k, _ = b.GEMV_SHAPES["q4k_1024x4096"]
    assert r["bytes"] == n * (k // 256) * 144 + 4 * k + 4 * n
    assert r["copies"] * (r["bytes"] - 4 * k - 4 * n) >= b.CPU_ROTATE_BYTES
    for th in (1, 2):
        e = r[f"threads_{th}"]
        assert e["reps"] == 2 and e["us"] > 0 and e["GBps"] > 0


def test_traffic_figures_from_the_committed_captures():
    b = _bench()
    assert b.profile_traffic("decode_kernel_llama3_8b.md") > 4.9e9
    # the 70B launch's traffic scales the 2-layer capture by its algorithmic bytes
    t = b.scaled_profile_traffic("decode_kernel_llama3_70b_2layers_8192ctx.md", 47_046_119_936)
    assert 1.0 < t / 47_046_119_936 < 1.01
    assert b.scaled_profile_traffic("no_such_capture.md", 1) is None
