"""The CPU oracle against the golden vectors and its own invariants (no GPU).

Pins the restatement of the reference's block formats (dequantize_slice,
f16_to_f32, decode_q4k_scales, src/inference.rs:867-1000, :1347-1474) to the
committed gguf-py fixtures, and checks the restated CPU matvec
(quantised-x AVX2 path, :589-760 / :897-1256) against fp64 within the
error its 8-bit activation quantisation implies.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from conftest import rel_l2

GOLD = Path(__file__).resolve().parent / "golden" / "dequant_golden.npz"
TYPES = {"Q4_K": 12, "Q6_K": 14, "Q8_0": 8, "Q5_K": 13, "Q4_0": 2}
QK = {"Q4_K": 256, "Q6_K": 256, "Q8_0": 32, "Q5_K": 256, "Q4_0": 32}


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def same_bits_nan_equal(a: np.ndarray, b: np.ndarray) -> bool:
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(nan | (a.view(np.uint32) == b.view(np.uint32))))


def test_f16_to_f32_all_65536(orc, gold):
    bits = gold["f16_bits"]
    ours = orc.dequantize(bits.view(np.uint8), 1, bits.size)  # F16 tensor of every bit pattern
    assert same_bits_nan_equal(ours, gold["f16_as_f32"])
    # the reference keeps NaN payloads: mantissa << 13 (inference.rs:884-886);
    # read through memory, not a C float return (which would quiet the NaN)
    sig = ours.view(np.uint32)[0x7C01]
    assert sig == 0x7F802000


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_matches_golden(orc, gold, name):
    raw = gold[f"{name}_raw"]
    want = gold[f"{name}_f32"]
    got = orc.dequantize(raw.reshape(-1), TYPES[name], raw.shape[0] * QK[name])
    assert same_bits_nan_equal(got, want)


def test_decode_q4k_scales_inverts_packing(orc, pkg):
    from hf_llm_b200 import synth
    rng = np.random.default_rng(3)
    for _ in range(200):
        sc = rng.integers(0, 64, 8).astype(np.uint8)
        mn = rng.integers(0, 64, 8).astype(np.uint8)
        s12 = synth.pack_q4k_scales(sc[None], mn[None])[0]
        dsc, dmn = orc.decode_q4k_scales(s12)
        assert np.array_equal(dsc, sc) and np.array_equal(dmn, mn)


def test_synth_row_ranges_are_slices(pkg):
    from hf_llm_b200 import ggml, synth
    full = synth.tensor_rows(ggml.Q6_K, 2500, 512, 9, 4)
    part = synth.tensor_rows(ggml.Q6_K, 2500, 512, 9, 4, 700, 2100)
    assert np.array_equal(full[700:2100], part)
    assert full.shape == (2500, 2 * 210)


@pytest.mark.parametrize("dtype,name", [(12, "Q4_K"), (14, "Q6_K"), (8, "Q8_0")])
def test_reference_cpu_matvec_error_vs_fp64(orc, pkg, dtype, name):
    """The reference CPU path quantises x to 8 bits; its error against fp64 is
    a few 1e-3 (above the GPU tolerance), never catastrophic."""
    from hf_llm_b200 import synth
    n, k = 256, 1024
    raw = synth.tensor_rows(dtype, n, k, 11, 1)
    x = synth.activation(k, 5, 2)
    y = orc.matmul_batched(raw, dtype, n, k, x)
    y64 = orc.matmul_f64(raw, dtype, n, k, x)
    err = rel_l2(y, y64)
    assert 1e-5 < err < 2e-2, err


def test_reference_matvec_threads_deterministic(orc, pkg):
    from hf_llm_b200 import ggml, synth
    raw = synth.tensor_rows(ggml.Q4_K, 300, 512, 2, 2)
    x = synth.activation(512, 1)
    orc.set_threads(1)
    a = orc.matmul_batched(raw, ggml.Q4_K, 300, 512, x)
    orc.set_threads(0)
    b = orc.matmul_batched(raw, ggml.Q4_K, 300, 512, x)
    assert np.array_equal(a, b)


def test_zero_activation_block_is_skipped(orc, pkg):
    """x blocks with d == 0 are skipped (inference.rs:1040-1042): an Inf
    weight scale meeting an all-zero x block does not poison the result."""
    from hf_llm_b200 import ggml, synth
    raw = synth.tensor_rows(ggml.Q4_K, 4, 512, 1, 1).copy()
    raw[:, 0:2] = np.array([0x7C00], np.uint16).view(np.uint8)  # block 0: d = +inf
    x = synth.activation(512, 2)
    x[0, :256] = 0.0
    y = orc.matmul_batched(raw, ggml.Q4_K, 4, 512, x)
    assert np.all(np.isfinite(y))


def test_oracle_forward_ref_vs_f64_small(orc, pkg):
    """The restated reference forward tracks the fp64 forward on a
    well-conditioned model, to the accuracy its 8-bit activations allow."""
    from hf_llm_b200 import model, synth
    cfg = dict(n_layers=2, n_embd=256, n_heads=4, n_kv_heads=2, head_dim=64, n_ff=512,
               n_vocab=512, rms_eps=1e-5, rope_theta=10000.0)
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), 3, dist="unit")
    m = orc.Model(cfg, t, kv_capacity=64)
    toks = [5, 17, 300, 2, 99]
    a = m.forward_ref(toks, 0)
    b = m.forward_f64(toks, 0, kv_f16=False)
    assert rel_l2(a, b) < 0.1
    # decode continues from the cache
    a2 = m.forward_ref([7], 5)
    b2 = m.forward_f64([7], 5, kv_f16=False)
    assert rel_l2(a2, b2) < 0.1
    # f16 KV rounding moves the fp64 logits only slightly
    m.clear_state()
    c = m.forward_f64(toks, 0, kv_f16=True)
    assert rel_l2(c, b) < 1e-3


def test_bench_distribution_is_chaotic(orc, pkg):
    """Documents why logits gates use the unit distribution: with the
    benchmark distributions even f16 KV rounding moves fp64 logits by >1e-3."""
    from hf_llm_b200 import model, synth
    cfg = dict(n_layers=2, n_embd=256, n_heads=4, n_kv_heads=2, head_dim=64, n_ff=512,
               n_vocab=512, rms_eps=1e-5, rope_theta=10000.0)
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), 3, dist="bench")
    b = orc.Model(cfg, t, 64).forward_f64([5, 17, 300, 2, 99], 0, kv_f16=False)
    c = orc.Model(cfg, t, 64).forward_f64([5, 17, 300, 2, 99], 0, kv_f16=True)
    assert rel_l2(c, b) > 1e-3


def test_fill_kv_sets_the_context(orc, pkg):
    """The CPU-baseline timing set-up: n synthetic positions in the reference
    path's KV cache; the next forward attends over them (its logits depend on
    the filled rows) and n beyond the capacity is rejected."""
    from hf_llm_b200 import model, synth
    cfg = dict(n_layers=1, n_embd=256, n_heads=2, n_kv_heads=1, head_dim=128, n_ff=256, n_vocab=64,
               rms_eps=1e-5, rope_theta=500000.0)
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), 3, dist="unit")
    a, b = orc.Model(cfg, t, kv_capacity=40), orc.Model(cfg, t, kv_capacity=40)
    a.fill_kv(32, seed=1)
    b.fill_kv(32, seed=2)
    la, lb = a.forward_ref([5], 32), b.forward_ref([5], 32)
    assert np.all(np.isfinite(la)) and not np.array_equal(la, lb)
    with pytest.raises(ValueError):
        a.fill_kv(41)
