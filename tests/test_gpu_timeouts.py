"""Failure handling without faulting or hanging a GPU.

Every device-side wait of the library is bounded (b2q_set_wait_limit_cycles);
a wait that runs out sets a device error word and lets its kernel finish.
The failures are planted on the host:

* one GPU: the host's persistent-kernel launch sequence is advanced without a
  launch (b2q_model_debug_desync), which is how a launch skipped by a peer
  looks from this GPU.  The next step's grid barriers cannot complete; with
  a 1 ms wait limit its waits give up, b2q_forward returns B2Q_ETIMEOUT
  (the reference silently fell back to the CPU instead, inference.rs:600-606),
  the error word is cleared and the barrier state re-armed, and the same step
  then repeats with logits bit-identical to the per-kernel path;
* the NCCL set-up of a tensor-parallel model whose second rank never joins
  ends with B2Q_ETIMEOUT after the host-side timeout (ncclCommAbort), in a
  child process so that a regression cannot stall this run.
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent

TOY = dict(n_layers=2, n_embd=512, n_heads=8, n_kv_heads=2, head_dim=128, n_ff=1536,
           n_vocab=1000, rms_eps=1e-5, rope_theta=500000.0)


def test_persistent_step_timeout_is_reported_and_recovers(engine, orc, pkg):
    from hf_llm_b200 import model, synth
    from hf_llm_b200._lib import ETIMEOUT, B2QError, check, lib
    t = synth.llama_tensors(TOY, model.q4_k_m_types(), 61, dist="unit")
    dev = model.StandardNativeEngine.from_tensors(engine, TOY, t, max_seq=64, decode="persistent")
    eag = model.StandardNativeEngine.from_tensors(engine, TOY, t, max_seq=64, decode="eager")
    ref = orc.Model(TOY, t, kv_capacity=64)
    assert dev.step_path == "persistent"
    prompt = [3, 1, 4, 1, 5, 9, 2]
    dev.forward(prompt, 0)
    eag.forward(prompt, 0)
    b = ref.forward_f64(prompt, 0, kv_f16=True)
    check(lib().b2q_set_wait_limit_cycles(engine.handle, 2_000_000))  # ~1 ms
    try:
        tok = int(np.argmax(b))
        check(lib().b2q_model_debug_desync(dev._h))
        with pytest.raises(B2QError) as e:
            dev.forward([tok], 7)
        assert e.value.status == ETIMEOUT
        engine.check_device_error()  # the word was cleared by b2q_forward
        # the step repeats normally, and so does the next one
        for pos in (7, 8):
            a, c = dev.forward([tok], pos), eag.forward([tok], pos)
            b = ref.forward_f64([tok], pos, kv_f16=True)
            assert np.array_equal(a.view(np.uint32), c.view(np.uint32)), pos
            assert rel_l2(a, b) <= 1e-3
            tok = int(np.argmax(b))
    finally:
        check(lib().b2q_set_wait_limit_cycles(engine.handle, 0))
    engine.check_device_error()
    dev.close()
    eag.close()


def test_tp_setup_times_out_when_a_rank_never_joins(pkg):
    r = subprocess.run([sys.executable, str(HERE / "nccl_join_worker.py"), "3000"], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    from hf_llm_b200._lib import ETIMEOUT
    assert out["status"] == ETIMEOUT, out
    assert 2.5 <= out["waited_s"] <= 60, out
    assert out["gemv_rel_l2_after"] <= 1e-3, out
