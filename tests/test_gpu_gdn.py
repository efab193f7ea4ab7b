"""The device Gated DeltaNet step (b2q_gdn_step_dev: gdn_conv_kernel +
gdn_head_kernel) against the oracle restatement of the reference's Qwen3.5
mixer core (src/inference.rs:2296-2374), token after token: outputs and the
updated convolution and state tensors within rel-L2 1e-5 (f32 sums in
another order), the convolution history bit for bit."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from test_gdn import gdn_inputs

pytestmark = pytest.mark.gpu

QWEN35 = dict(n_k_heads=16, n_v_heads=32, d_k=128, d_v=128, conv_kernel=4, eps=1e-6)


def _run(engine, cfg, d, steps):
    import torch
    from hf_llm_b200._lib import GdnConfig, check, lib
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in d.items()}
    n_tok = d["qkv"].shape[0]
    y = torch.zeros((n_tok, cfg["n_v_heads"] * cfg["d_v"]), dtype=torch.float32, device="cuda")
    c = GdnConfig(cfg["n_k_heads"], cfg["n_v_heads"], cfg["d_k"], cfg["d_v"], cfg["conv_kernel"], cfg["eps"])
    # `steps` calls of n_tok / steps tokens each: the state carries over
    per = n_tok // steps
    for s in range(steps):
        o = s * per
        sl = lambda k, w: t[k][o:o + per].data_ptr()
        check(lib().b2q_gdn_step_dev(engine.handle, C.byref(c), per, sl("qkv", 0), sl("z", 0), sl("alpha", 0),
                                     sl("beta", 0), t["conv_w"].data_ptr(), t["ssm_a"].data_ptr(),
                                     t["dt_bias"].data_ptr(), t["ssm_norm"].data_ptr(), t["conv_state"].data_ptr(),
                                     t["ssm_state"].data_ptr(), y[o:o + per].data_ptr(), None))
    torch.cuda.synchronize()
    return y.cpu().numpy(), t["conv_state"].cpu().numpy(), t["ssm_state"].cpu().numpy()


def _rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b.astype(np.float64)), 1e-30))


@pytest.mark.parametrize("cfg,n_tok,steps", [(QWEN35, 1, 1), (QWEN35, 6, 3), (dict(QWEN35, n_v_heads=16, d_v=256), 4, 1),
                                             (dict(QWEN35, n_k_heads=2, n_v_heads=6, d_v=64, conv_kernel=2), 5, 5)])
def test_gdn_step_matches_oracle(engine, orc, pkg, cfg, n_tok, steps):
    d = gdn_inputs(cfg, n_tok, 3)
    y, cs, ss = _run(engine, cfg, d, steps)
    y0, cs0, ss0 = orc.gdn_step(cfg, **d)
    assert np.array_equal(cs, cs0)
    assert _rel(y, y0) <= 1e-5, _rel(y, y0)
    assert _rel(ss, ss0) <= 1e-5, _rel(ss, ss0)
    engine.check_device_error()


def test_gdn_rejects_bad_shapes(engine, pkg):
    from hf_llm_b200._lib import EINVAL, EUNSUP, GdnConfig, lib
    c = GdnConfig(16, 32, 64, 128, 4, 1e-6)  # d_k 64
    dummy = C.c_void_p(256)
    assert lib().b2q_gdn_step_dev(engine.handle, C.byref(c), 1, *([dummy] * 12), None) == EUNSUP
    c = GdnConfig(16, 24, 128, 128, 4, 1e-6)  # value heads not a multiple of key heads
    assert lib().b2q_gdn_step_dev(engine.handle, C.byref(c), 1, *([dummy] * 12), None) == EINVAL
