"""Parity of whole-model forwards with the fp64 oracle at the benchmark's own
geometries and at the edges of the reference's contract.

The oracle is the reference's Llama block loop (inference.rs:2695-2860)
restated in double precision over the bit-exact dequantised weights, with
the KV cache rounded to f16 as the device cache is.  Gate: rel-L2 <= 1e-3
of the logits.  Models use the zero-mean "unit" block distribution (the
benchmark distribution is numerically chaotic, see synth.py).

* full depth: the Llama-3-8B geometry with all 32 layers (prompt pass on
  the tensor cores, then persistent single-token steps);
* Llama-3-70B widths (hidden 8192, 64/8 heads, FFN 28672, full vocabulary)
  at two layers;
* long context: attention over 4096 and 8192 cached keys (the reference's
  max_seq_len, inference.rs:2538; positions clamped at 8191, :2756) in the
  prompt pass and in the persistent and per-kernel single-token steps;
* q/k/v biases added before RoPE (inference.rs:2733-2753).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _models(engine, orc, cfg, tensors, max_seq, modes=("persistent",)):
    from hf_llm_b200 import model
    devs = {md: model.StandardNativeEngine.from_tensors(engine, cfg, tensors, max_seq=max_seq, decode=md)
            for md in modes}
    ref = orc.Model(cfg, tensors, kv_capacity=max_seq)
    return devs, ref


def test_llama3_8b_all_32_layers_vs_fp64(engine, orc, pkg):
    """The benchmark's decoder geometry at full depth: a 20-token prompt
    (tensor-core prompt pass) and four persistent single-token steps."""
    from hf_llm_b200 import model, synth
    cfg = dict(model.LLAMA3_8B)
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), 41, dist="unit")
    devs, ref = _models(engine, orc, cfg, t, 64)
    dev = devs["persistent"]
    assert dev.step_path == "persistent"
    rng = np.random.default_rng(41)
    prompt = rng.integers(0, cfg["n_vocab"], 20).tolist()
    a = dev.forward(prompt, 0)
    b = ref.forward_f64(prompt, 0, kv_f16=True)
    assert rel_l2(a, b) <= TOL, f"prompt: {rel_l2(a, b)}"
    pos = len(prompt)
    for step in range(4):
        tok = int(np.argmax(b))
        a = dev.forward([tok], pos)
        b = ref.forward_f64([tok], pos, kv_f16=True)
        assert rel_l2(a, b) <= TOL, f"step {step}: {rel_l2(a, b)}"
        pos += 1
    engine.check_device_error()
    dev.close()


def test_llama3_70b_widths_two_layers_vs_fp64(engine, orc, pkg):
    """Hidden 8192, 64 query / 8 KV heads (eight per group), FFN 28672 and
    the full 128256-row Q6_K head: prompt pass and persistent steps."""
    from hf_llm_b200 import model, synth
    cfg = dict(model.LLAMA3_70B, n_layers=2)
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), 43, dist="unit")
    devs, ref = _models(engine, orc, cfg, t, 96, modes=("persistent", "eager"))
    rng = np.random.default_rng(43)
    prompt = rng.integers(0, cfg["n_vocab"], 37).tolist()
    out = {md: d.forward(prompt, 0) for md, d in devs.items()}
    b = ref.forward_f64(prompt, 0, kv_f16=True)
    for md, a in out.items():
        assert rel_l2(a, b) <= TOL, f"{md} prompt: {rel_l2(a, b)}"
    pos = len(prompt)
    for step in range(3):
        tok = int(np.argmax(b))
        out = {md: d.forward([tok], pos) for md, d in devs.items()}
        b = ref.forward_f64([tok], pos, kv_f16=True)
        assert np.array_equal(out["persistent"].view(np.uint32), out["eager"].view(np.uint32)), step
        assert rel_l2(out["persistent"], b) <= TOL, f"step {step}: {rel_l2(out['persistent'], b)}"
        pos += 1
    engine.check_device_error()
    for d in devs.values():
        d.close()


LONG = dict(n_layers=1, n_embd=512, n_heads=8, n_kv_heads=2, head_dim=128, n_ff=512, n_vocab=512,
            rms_eps=1e-5, rope_theta=500000.0)


def test_attention_over_4096_and_8192_keys(engine, orc, pkg):
    """Prompt passes (256-token chunks on the tensor cores) up to 4096
    tokens, a single-token step at position 4096 (64 attention splits of 64
    keys), prompt passes up to position 8190 and the last single-token step
    at 8191 (128 splits, the reference's max_seq_len): persistent and
    per-kernel steps bit-identical, all within 1e-3 of fp64."""
    from hf_llm_b200 import model, synth
    cfg = dict(LONG)
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), 47, dist="unit")
    devs, ref = _models(engine, orc, cfg, t, 8192, modes=("persistent", "eager"))
    rng = np.random.default_rng(47)
    seq = rng.integers(0, cfg["n_vocab"], 8192).tolist()

    def prompt(b, e):
        for md, d in devs.items():
            for off in range(b, e, 256):
                la = d.forward(seq[off:min(e, off + 256)], off)
            out[md] = la
        return ref.forward_f64(seq[b:e], b, kv_f16=True)

    def step(pos):
        for md, d in devs.items():
            out[md] = d.forward([seq[pos]], pos)
        want = ref.forward_f64([seq[pos]], pos, kv_f16=True)
        assert np.array_equal(out["persistent"].view(np.uint32), out["eager"].view(np.uint32)), pos
        return want

    out = {}
    b = prompt(0, 4096)
    for md in devs:
        assert rel_l2(out[md], b) <= TOL, f"{md} prompt to 4096: {rel_l2(out[md], b)}"
    b = step(4096)
    assert rel_l2(out["persistent"], b) <= TOL, f"step at 4096: {rel_l2(out['persistent'], b)}"
    b = prompt(4097, 8191)
    for md in devs:
        assert rel_l2(out[md], b) <= TOL, f"{md} prompt to 8191: {rel_l2(out[md], b)}"
    b = step(8191)
    assert rel_l2(out["persistent"], b) <= TOL, f"step at 8191: {rel_l2(out['persistent'], b)}"
    engine.check_device_error()
    for d in devs.values():
        d.close()


TOY = dict(n_layers=2, n_embd=512, n_heads=8, n_kv_heads=2, head_dim=128, n_ff=1536,
           n_vocab=1000, rms_eps=1e-5, rope_theta=500000.0)


@pytest.mark.parametrize("gqa", [4, 8])
def test_qkv_biases_vs_fp64(engine, orc, pkg, gqa):
    """attn_q/k/v biases (the Qwen2 layout, inference.rs:2564-2566) are added
    to q, k and v before RoPE and the KV append (:2733-2753): a 40-token
    prompt (tensor cores), a 9-token prompt (GEMV) and single-token steps on
    all three step paths."""
    from hf_llm_b200 import ggml, model, synth
    cfg = dict(TOY, n_kv_heads=8 // gqa)
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), 50 + gqa, dist="unit")
    rng = np.random.default_rng(50 + gqa)
    hd = cfg["head_dim"]
    for i in range(cfg["n_layers"]):
        for role, n in (("attn_q", cfg["n_heads"] * hd), ("attn_k", cfg["n_kv_heads"] * hd),
                        ("attn_v", cfg["n_kv_heads"] * hd)):
            t[f"blk.{i}.{role}.bias"] = (ggml.F32, [n], (0.5 * rng.standard_normal(n)).astype(np.float32))
    devs, ref = _models(engine, orc, cfg, t, 128, modes=("persistent", "graph", "eager"))
    # without the biases the logits are clearly different (the biases matter)
    plain = {k: v for k, v in t.items() if not k.endswith(".bias")}
    ref0 = orc.Model(cfg, plain, kv_capacity=128)
    p1 = rng.integers(0, cfg["n_vocab"], 40).tolist()
    p2 = rng.integers(0, cfg["n_vocab"], 9).tolist()
    out = {md: d.forward(p1, 0) for md, d in devs.items()}
    b = ref.forward_f64(p1, 0, kv_f16=True)
    assert rel_l2(ref0.forward_f64(p1, 0, kv_f16=True), b) > 1e-2
    for md, a in out.items():
        assert rel_l2(a, b) <= TOL, f"{md} prompt 1: {rel_l2(a, b)}"
    out = {md: d.forward(p2, 40) for md, d in devs.items()}
    b = ref.forward_f64(p2, 40, kv_f16=True)
    for md, a in out.items():
        assert rel_l2(a, b) <= TOL, f"{md} prompt 2: {rel_l2(a, b)}"
    pos = 49
    for step in range(3):
        tok = int(np.argmax(b))
        out = {md: d.forward([tok], pos) for md, d in devs.items()}
        b = ref.forward_f64([tok], pos, kv_f16=True)
        for md in ("persistent", "graph"):
            assert np.array_equal(out[md].view(np.uint32), out["eager"].view(np.uint32)), (md, step)
        assert rel_l2(out["persistent"], b) <= TOL, f"step {step}: {rel_l2(out['persistent'], b)}"
        pos += 1
    engine.check_device_error()
    for d in devs.values():
        d.close()


def test_synthetic_kv_fill_steps_persistent_equals_eager(engine, pkg):
    """b2q_model_fill_kv (the benchmark's long-context set-up): after the same
    seeded fill of 8000 positions, persistent and per-kernel single-token
    steps at positions 8000..8002 give the same logits bit for bit, and a
    different seed gives different logits (the steps read the filled rows)."""
    from hf_llm_b200 import model, synth
    cfg = dict(LONG)
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), 53, dist="unit")
    ms = {md: model.StandardNativeEngine.from_tensors(engine, cfg, t, max_seq=8192, decode=md)
          for md in ("persistent", "eager")}
    other = model.StandardNativeEngine.from_tensors(engine, cfg, t, max_seq=8192, decode="eager")
    for m in ms.values():
        m.fill_kv(0, 8000, seed=9, scale=0.5)
    other.fill_kv(0, 8000, seed=10, scale=0.5)
    for pos, tok in ((8000, 17), (8001, 300), (8002, 5)):
        a, b = ms["persistent"].forward([tok], pos), ms["eager"].forward([tok], pos)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), pos
        assert not np.array_equal(a, other.forward([tok], pos))
    engine.check_device_error()
    for m in list(ms.values()) + [other]:
        m.close()
