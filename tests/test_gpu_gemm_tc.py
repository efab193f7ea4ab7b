"""Multi-token matmul on the tensor cores (gemm_tc.cuh, tcgen05.mma with the
accumulator in TMEM) against the fp64 oracle.

Every call with m >= 16 tokens goes this way (b2q_matmul, b2q_ffn_swiglu and
the prompt passes of the model).  Weights are dequantised bit-exactly and
rounded to f16, activations are f16 scaled per token by a power of two, the
sums are f32: the bar is the decode path's rel-L2 <= 1e-3 against fp64.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _check(engine, orc, dtype, n, k, m, seed, dist="bench"):
    from hf_llm_b200 import synth
    raw = synth.tensor_rows(dtype, n, k, seed + 1, 7, dist=dist)
    x = synth.activation(k, seed + 2, m)
    buf = engine.try_upload_weight(raw, dtype, n, k)
    y = engine.matmul_batched(buf, x, m, n, k)
    y64 = orc.matmul_f64(raw, dtype, n, k, x)
    err = rel_l2(y, y64)
    assert np.all(np.isfinite(y))
    assert err <= TOL, f"type {dtype} [{n},{k}] m={m}: rel-L2 {err:.3g}"
    return err


@pytest.mark.parametrize("dtype", [12, 14, 8, 13, 2])
@pytest.mark.parametrize("m", [16, 17, 48, 100, 256, 300])
def test_tc_matmul_tokens(engine, orc, pkg, dtype, m):
    _check(engine, orc, dtype, 520, 1024, m, seed=m)


@pytest.mark.parametrize("dtype,n,k", [(12, 4096, 4096), (12, 1024, 4096), (14, 4096, 14336), (8, 4096, 4096),
                                       (12, 14336, 4096), (14, 1024, 4096)])
def test_tc_matmul_model_shapes(engine, orc, pkg, dtype, n, k):
    _check(engine, orc, dtype, n, k, 64, seed=3)


@pytest.mark.parametrize("dtype", [12, 14, 8, 13, 2])
def test_tc_matmul_ragged_rows_and_k(engine, orc, pkg, dtype):
    # rows not a multiple of 128 (or of 8); k of an odd number of 64-element
    # stages, with padding units in the tile layout (Q8_0 / Q4_0: 34 units, KC 48)
    k = 1088 if dtype in (8, 2) else 1280
    _check(engine, orc, dtype, 77, k, 33, seed=5)
    _check(engine, orc, dtype, 1, k, 16, seed=6)


def test_tc_matmul_unit_distribution_and_scales(engine, orc, pkg):
    from hf_llm_b200 import ggml, synth
    n, k, m = 300, 2048, 40
    raw = synth.tensor_rows(ggml.Q4_K, n, k, 9, 9, dist="unit")
    buf = engine.try_upload_weight(raw, ggml.Q4_K, n, k)
    x = synth.activation(k, 11, m)
    x[3] *= 1e4       # per-token scaling keeps every token's precision
    x[7] *= 1e-5
    x[9] = 0.0        # an all-zero token
    y = engine.matmul_batched(buf, x, m, n, k)
    y64 = orc.matmul_f64(raw, ggml.Q4_K, n, k, x)
    assert np.array_equal(y[9], np.zeros(n, np.float32))
    for t in range(m):
        if t != 9:
            assert rel_l2(y[t], y64[t]) <= TOL, t


def test_tc_ffn_swiglu(engine, orc, pkg):
    from hf_llm_b200 import ggml, synth
    E, F, m = 1024, 2816, 40
    g = synth.tensor_rows(ggml.Q4_K, F, E, 1, 1, dist="unit")
    u = synth.tensor_rows(ggml.Q4_K, F, E, 1, 2, dist="unit")
    d = synth.tensor_rows(ggml.Q6_K, E, F, 1, 3, dist="unit")
    bg, bu, bd = (engine.try_upload_weight(g, ggml.Q4_K, F, E), engine.try_upload_weight(u, ggml.Q4_K, F, E),
                  engine.try_upload_weight(d, ggml.Q6_K, E, F))
    x = synth.activation(E, 3, m)
    y = engine.ffn_swiglu_fused(bg, bu, bd, x, m, E, F)
    gg = orc.matmul_f64(g, ggml.Q4_K, F, E, x)
    uu = orc.matmul_f64(u, ggml.Q4_K, F, E, x)
    h = gg / (1.0 + np.exp(-gg)) * uu
    wd = orc.dequantize(d.reshape(-1), ggml.Q6_K, E * F).reshape(E, F).astype(np.float64)
    assert rel_l2(y, h @ wd.T) <= TOL


def test_tc_matmul_is_deterministic(engine, pkg):
    from hf_llm_b200 import ggml, synth
    n, k, m = 640, 4096, 64
    raw = synth.tensor_rows(ggml.Q4_K, n, k, 2, 2)
    buf = engine.try_upload_weight(raw, ggml.Q4_K, n, k)
    x = synth.activation(k, 4, m)
    a = engine.matmul_batched(buf, x, m, n, k)
    b = engine.matmul_batched(buf, x, m, n, k)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # a row shard gives the same bits as the whole weight (split-K depends on k only)
    half = engine.try_upload_weight(np.ascontiguousarray(raw[:320]), ggml.Q4_K, 320, k)
    c = engine.matmul_batched(half, x, m, 320, k)
    assert np.array_equal(c.view(np.uint32), a[:, :320].view(np.uint32))
    engine.check_device_error()
