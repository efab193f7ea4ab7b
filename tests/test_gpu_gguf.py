"""A model loaded from a GGUF file (b2q_gguf_open + b2q_model_load_gguf, the
StandardNativeEngine::from_gguf path, src/inference.rs:2513-2620) gives the
same logits, bit for bit, as the same tensors handed over one by one.

Files are written by gguf-py's GGUFWriter, so layout, alignment and dims
order come from an implementation independent of this library.
"""
from __future__ import annotations

import numpy as np
import pytest

import gguf_fixtures as gf

pytestmark = pytest.mark.gpu
pytest.importorskip("gguf")

TOY = dict(n_layers=2, n_embd=512, n_heads=8, n_kv_heads=2, head_dim=128, n_ff=1536,
           n_vocab=1000, rms_eps=1e-5, rope_theta=500000.0)


@pytest.mark.parametrize("variant", ["plain", "tied_output", "f16_norms"])
@pytest.mark.parametrize("decode", ["eager", "persistent"])
def test_from_gguf_equals_from_tensors(engine, pkg, tmp_path, variant, decode):
    from hf_llm_b200 import model, synth
    t = synth.llama_tensors(TOY, model.q4_k_m_types(), 8, dist="unit")
    drop = ("output.weight",) if variant == "tied_output" else ()
    f16 = variant == "f16_norms"
    path = tmp_path / "toy.gguf"
    gf.write_ggufpy(path, "llama", gf.llama_kvs(TOY), gf.llama_tensor_list(t, drop=drop, f16_norms=f16))
    ref_t = {}
    for name, (dt, dims, arr) in t.items():
        if name in drop:
            continue
        if f16 and dt == 0 and len(dims) == 1:
            arr = arr.astype(np.float16).astype(np.float32)
        ref_t[name] = (dt, dims, arr)
    gm = model.StandardNativeEngine.from_gguf(engine, path, max_seq=128, decode=decode)
    assert gm.cfg == pytest.approx(TOY)
    rm = model.StandardNativeEngine.from_tensors(engine, TOY, ref_t, max_seq=128, decode=decode)
    assert gm.weight_bytes == rm.weight_bytes
    toks = list(range(3, 40))
    a, b = gm.forward(toks, 0), rm.forward(toks, 0)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    for step, tok in enumerate((17, 999)):
        a, b = gm.forward([tok], 37 + step), rm.forward([tok], 37 + step)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), step
    gm.close()
    rm.close()
    engine.check_device_error()


def test_from_gguf_missing_tensor_is_an_error(engine, pkg, tmp_path):
    from hf_llm_b200 import _lib, model, synth
    t = synth.llama_tensors(TOY, model.q4_k_m_types(), 8, dist="unit")
    path = tmp_path / "broken.gguf"
    gf.write_ggufpy(path, "llama", gf.llama_kvs(TOY), gf.llama_tensor_list(t, drop=("blk.1.ffn_up.weight",)))
    with pytest.raises(_lib.B2QError) as e:
        model.StandardNativeEngine.from_gguf(engine, path, max_seq=64)
    assert e.value.status == _lib.EINVAL
    assert "blk.1.ffn_up.weight" in str(e.value)
