"""Whole-model forward on the device against the fp64 oracle forward.

The oracle runs the reference's Llama block loop (inference.rs:2695-2860) in
double precision over the bit-exact dequantised weights, with the KV cache
rounded to f16 as the device cache is.  Logits of every forward must be
within rel-L2 <= 1e-3.  Models use the unit-variance synthetic distribution
(see synth.py: the benchmark distribution is numerically chaotic).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3

TOY = dict(n_layers=2, n_embd=512, n_heads=8, n_kv_heads=2, head_dim=128, n_ff=1536,
           n_vocab=1000, rms_eps=1e-5, rope_theta=500000.0)


def _pair(engine, orc, pkg, cfg, seed=1, max_seq=256):
    from hf_llm_b200 import model, synth
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), seed, dist="unit")
    dev = model.StandardNativeEngine.from_tensors(engine, cfg, t, max_seq=max_seq)
    ref = orc.Model(cfg, t, kv_capacity=max_seq)
    return dev, ref


def test_prefill_then_decode_matches_fp64(engine, orc, pkg):
    dev, ref = _pair(engine, orc, pkg, TOY)
    toks = [1, 5, 900, 33, 2, 7, 400]
    a = dev.forward(toks, 0)
    b = ref.forward_f64(toks, 0, kv_f16=True)
    assert rel_l2(a, b) <= TOL
    pos = len(toks)
    for step in range(4):  # single-token steps replay the captured decode graph
        tok = [int(np.argmax(b))]
        a = dev.forward(tok, pos)
        b = ref.forward_f64(tok, pos, kv_f16=True)
        assert rel_l2(a, b) <= TOL, f"decode step {step}: {rel_l2(a, b)}"
        pos += 1


@pytest.mark.parametrize("gqa", [1, 2, 4, 8])
def test_gqa_ratios(engine, orc, pkg, gqa):
    cfg = dict(TOY, n_heads=8, n_kv_heads=8 // gqa)
    dev, ref = _pair(engine, orc, pkg, cfg, seed=gqa)
    toks = [3, 14, 15, 92, 65]
    assert rel_l2(dev.forward(toks, 0), ref.forward_f64(toks, 0, kv_f16=True)) <= TOL
    assert rel_l2(dev.forward([35], 5), ref.forward_f64([35], 5, kv_f16=True)) <= TOL


@pytest.mark.parametrize("gqa", [1, 2, 4, 8])
def test_prompt_attention_rows_and_chunks(engine, orc, pkg, gqa):
    """The prompt-pass attention (16 or more tokens: 64 query rows per CTA,
    64 / G tokens): prompts that fill no CTA exactly (16, 47 and 130 tokens)
    and a two-chunk prompt whose second chunk starts at position 256, for
    every GQA ratio, against the fp64 forward."""
    cfg = dict(TOY, n_heads=8, n_kv_heads=8 // gqa, n_layers=2)
    dev, ref = _pair(engine, orc, pkg, cfg, seed=40 + gqa, max_seq=512)
    rng = np.random.default_rng(gqa)
    pos = 0
    for n in (16, 47, 130):
        toks = rng.integers(0, cfg["n_vocab"], n).tolist()
        a = dev.forward(toks, pos)
        b = ref.forward_f64(toks, pos, kv_f16=True)
        assert rel_l2(a, b) <= TOL, f"G={gqa} {n} tokens at {pos}: {rel_l2(a, b)}"
        pos += n
    toks = rng.integers(0, cfg["n_vocab"], 300).tolist()
    dev2, ref2 = _pair(engine, orc, pkg, cfg, seed=40 + gqa, max_seq=512)
    a = dev2.forward(toks, 0)
    b = ref2.forward_f64(toks, 0, kv_f16=True)
    assert rel_l2(a, b) <= TOL, f"G={gqa} 300 tokens: {rel_l2(a, b)}"


def test_long_prompt_chunks_and_splits(engine, orc, pkg):
    """A prompt longer than one forward chunk (256 tokens; the second one
    ragged) and than one attention split (64 keys) exercises the chunked
    prefill and the split merge."""
    dev, ref = _pair(engine, orc, pkg, dict(TOY, n_layers=1), seed=7, max_seq=512)
    rng = np.random.default_rng(0)
    toks = rng.integers(0, TOY["n_vocab"], 300).tolist()
    a = dev.forward(toks, 0)
    b = ref.forward_f64(toks, 0, kv_f16=True)
    assert rel_l2(a, b) <= TOL
    assert rel_l2(dev.forward([11], 300), ref.forward_f64([11], 300, kv_f16=True)) <= TOL


def test_llama3_8b_geometry_two_layers(engine, orc, pkg):
    """Full Llama-3-8B widths (hidden 4096, 32/8 heads, FFN 14336, vocab
    128256) with 2 layers."""
    from hf_llm_b200 import model
    cfg = dict(model.LLAMA3_8B, n_layers=2)
    dev, ref = _pair(engine, orc, pkg, cfg, seed=11, max_seq=64)
    toks = [128000, 9906, 1917, 11]
    assert rel_l2(dev.forward(toks, 0), ref.forward_f64(toks, 0, kv_f16=True)) <= TOL
    assert rel_l2(dev.forward([13], 4), ref.forward_f64([13], 4, kv_f16=True)) <= TOL


def test_graph_decode_equals_eager(engine, orc, pkg):
    """The captured single-token graph and the eager path give identical
    logits (same kernels, same order), the eager step on a foreign stream."""
    import torch
    from hf_llm_b200 import model, synth
    t = synth.llama_tensors(TOY, model.q4_k_m_types(), 5, dist="unit")
    a_m = model.StandardNativeEngine(engine, TOY, max_seq=64, decode="graph")
    b_m = model.StandardNativeEngine(engine, TOY, max_seq=64, use_graph=False)
    for mm in (a_m, b_m):
        for name, (dt, dims, arr) in t.items():
            mm.set_tensor(name, dt, dims, arr)
        mm.finalize()
        mm.forward([1, 2, 3], 0)
    la = a_m.forward([4], 3)  # graph replay
    tok = torch.tensor([4], dtype=torch.int32, device="cuda")
    lb = torch.empty(TOY["n_vocab"], dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    b_m.forward_dev(tok.data_ptr(), 1, 3, lb.data_ptr(), 0, s.cuda_stream)  # eager, other stream
    s.synchronize()
    assert np.array_equal(la, lb.cpu().numpy())


@pytest.mark.parametrize("gqa", [1, 2, 4, 8])
def test_persistent_decode_bit_identical(engine, orc, pkg, gqa):
    """The persistent decode kernel computes every value with the operations
    and order of the per-kernel path: logits and argmax agree bit for bit
    with the eager and graph steps, step after step, across the 128-key
    attention split boundary, and stay within the fp64 tolerance."""
    from hf_llm_b200 import model, synth
    cfg = dict(TOY, n_heads=8, n_kv_heads=8 // gqa)
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), 20 + gqa, dist="unit")
    modes = ("persistent", "graph", "eager")
    ms = {md: model.StandardNativeEngine.from_tensors(engine, cfg, t, max_seq=320, decode=md) for md in modes}
    ref = orc.Model(cfg, t, kv_capacity=320)
    rng = np.random.default_rng(gqa)
    prompt = rng.integers(0, cfg["n_vocab"], 125).tolist()
    first = {md: m.forward(prompt, 0) for md, m in ms.items()}
    b = ref.forward_f64(prompt, 0, kv_f16=True)
    tok = int(np.argmax(first["eager"]))
    for step in range(6):  # positions 125..130: the step at 128 opens a second split
        pos = 125 + step
        outs = {md: m.forward([tok], pos) for md, m in ms.items()}
        b = ref.forward_f64([tok], pos, kv_f16=True)
        for md in ("persistent", "graph"):
            assert np.array_equal(outs[md].view(np.uint32), outs["eager"].view(np.uint32)), (md, pos)
        assert rel_l2(outs["persistent"], b) <= TOL, f"pos {pos}: {rel_l2(outs['persistent'], b)}"
        # argmax written by the kernel itself == first index of the maximum
        am = {md: m.forward_argmax([tok], pos) for md, m in ms.items()}
        assert am["persistent"] == am["eager"] == am["graph"] == int(np.argmax(outs["eager"]))
        tok = am["eager"]


def test_persistent_decode_llama3_8b_geometry(engine, orc, pkg):
    """Llama-3-8B widths (4096 / 32:8 heads / 14336 / vocab 128256), the
    benchmark's weight distributions, one layer: the persistent step equals
    the eager step bit for bit, including the 128256-row output head split
    over the grid and the grid-wide argmax, through the device-pointer API
    on a foreign stream."""
    import torch
    from hf_llm_b200 import model, synth
    cfg = dict(model.LLAMA3_8B, n_layers=1)
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), 17, dist="bench")
    pm = model.StandardNativeEngine.from_tensors(engine, cfg, t, max_seq=64, decode="persistent")
    em = model.StandardNativeEngine.from_tensors(engine, cfg, t, max_seq=64, decode="eager")
    assert pm.decode_mode == "persistent"
    toks = [128000, 791, 4062, 14198, 39935]
    for m in (pm, em):
        m.forward(toks, 0)
    s = torch.cuda.Stream()
    tok = torch.tensor([1234], dtype=torch.int32, device="cuda")
    res = {}
    for name, m in (("p", pm), ("e", em)):
        lg = torch.empty(cfg["n_vocab"], dtype=torch.float32, device="cuda")
        am = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        m.forward_dev(tok.data_ptr(), 1, 5, lg.data_ptr(), am.data_ptr(), s.cuda_stream)
        s.synchronize()
        res[name] = (lg.cpu().numpy(), int(am.item()))
    assert np.array_equal(res["p"][0].view(np.uint32), res["e"][0].view(np.uint32))
    assert res["p"][1] == res["e"][1] == int(np.argmax(res["e"][0]))
    engine.check_device_error()


def test_persistent_decode_llama3_70b_geometry(engine, pkg):
    """Llama-3-70B widths (hidden 8192, 64:8 heads, FFN 28672), one layer,
    a reduced vocabulary: the persistent kernel (64 KB of staged FFN input,
    eight query heads per KV head) equals the eager kernels bit for bit."""
    from hf_llm_b200 import model, synth
    cfg = dict(model.LLAMA3_70B, n_layers=1, n_vocab=4000)
    t = synth.llama_tensors(cfg, model.q4_k_m_types(), 23, dist="unit")
    pm = model.StandardNativeEngine.from_tensors(engine, cfg, t, max_seq=96, decode="persistent")
    em = model.StandardNativeEngine.from_tensors(engine, cfg, t, max_seq=96, decode="eager")
    toks = list(range(7, 77))
    assert np.array_equal(pm.forward(toks, 0), em.forward(toks, 0))
    for step, tok in enumerate((11, 3999, 0)):
        a, b = pm.forward([tok], 70 + step), em.forward([tok], 70 + step)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), step
    engine.check_device_error()


def test_greedy_generation_follows_fp64_argmax(engine, orc, pkg):
    dev, ref = _pair(engine, orc, pkg, TOY, seed=3)
    out = dev.generate_greedy([5, 6, 7], 6)
    pos, tok = 3, None
    logits = ref.forward_f64([5, 6, 7], 0, kv_f16=True)
    for t in out:
        srt = np.sort(logits)
        if srt[-1] - srt[-2] > 1e-3 * np.abs(srt[-1]):  # no near-tie
            assert t == int(np.argmax(logits))
        logits = ref.forward_f64([t], pos, kv_f16=True)
        pos += 1


def test_model_error_paths(engine, pkg):
    from hf_llm_b200 import model, synth
    from hf_llm_b200._lib import B2QError, EINVAL
    t = synth.llama_tensors(TOY, model.q4_k_m_types(), 2, dist="unit")
    m = model.StandardNativeEngine.from_tensors(engine, TOY, t, max_seq=16)
    with pytest.raises(B2QError) as e:
        m.forward([TOY["n_vocab"]], 0)  # token id out of range
    assert e.value.status == EINVAL
    with pytest.raises(B2QError) as e:
        m.forward([1, 2], 15)  # beyond the KV capacity
    assert e.value.status == EINVAL
    incomplete = model.StandardNativeEngine(engine, TOY, max_seq=16)
    with pytest.raises(B2QError):
        incomplete.finalize()  # tensors missing
    engine.check_device_error()


@pytest.mark.parametrize("kind", ["q5_k_m", "q4_0"])
def test_model_q5k_and_q40_weights(engine, orc, pkg, kind):
    """Models whose projections are Q5_K (a Q5_K_M-style mix) or Q4_0: the
    prompt pass (tensor cores) and decode steps stay within the fp64
    tolerance; single-token steps run the persistent kernel and equal the
    eager per-kernel steps bit for bit."""
    from hf_llm_b200 import ggml, model, synth
    base = model.q4_k_m_types()
    if kind == "q5_k_m":
        types = {r: (ggml.Q5_K if t == ggml.Q4_K else t) for r, t in base.items()}
    else:
        types = {r: ggml.Q4_0 for r in base}
    t = synth.llama_tensors(TOY, types, 31, dist="unit")
    dev = model.StandardNativeEngine.from_tensors(engine, TOY, t, max_seq=96)
    eag = model.StandardNativeEngine.from_tensors(engine, TOY, t, max_seq=96, decode="eager")
    ref = orc.Model(TOY, t, kv_capacity=96)
    assert dev.step_path == "persistent" and eag.step_path == "eager"
    toks = list(range(2, 42))
    a, e = dev.forward(toks, 0), eag.forward(toks, 0)
    b = ref.forward_f64(toks, 0, kv_f16=True)
    assert rel_l2(a, b) <= TOL, rel_l2(a, b)
    for step, tok in enumerate((5, 77, 999)):
        a, e = dev.forward([tok], 40 + step), eag.forward([tok], 40 + step)
        b = ref.forward_f64([tok], 40 + step, kv_f16=True)
        assert np.array_equal(a.view(np.uint32), e.view(np.uint32)), step
        assert rel_l2(a, b) <= TOL, (step, rel_l2(a, b))
    engine.check_device_error()
