"""The Gated DeltaNet oracle (oracle_gdn_step, a restatement of the
reference's Qwen3.5 Gated DeltaNet mixer core, src/inference.rs:2296-2374
with ssm_head_step_avx2 :1535-1583) against an independent numpy
restatement of the same steps, in float64."""
from __future__ import annotations

import numpy as np

CFG = dict(n_k_heads=2, n_v_heads=4, d_k=128, d_v=64, conv_kernel=4, eps=1e-6)


def gdn_inputs(cfg, n_tokens, seed):
    rng = np.random.default_rng(seed)
    ch = 2 * cfg["n_k_heads"] * cfg["d_k"] + cfg["n_v_heads"] * cfg["d_v"]
    vd = cfg["n_v_heads"] * cfg["d_v"]
    nv, K = cfg["n_v_heads"], cfg["conv_kernel"]
    f = np.float32
    return dict(qkv=rng.standard_normal((n_tokens, ch)).astype(f), z=rng.standard_normal((n_tokens, vd)).astype(f),
                alpha=rng.standard_normal((n_tokens, nv)).astype(f), beta=rng.standard_normal((n_tokens, nv)).astype(f),
                conv_w=(rng.standard_normal((ch, K)) * 0.5).astype(f), ssm_a=-np.abs(rng.standard_normal(nv)).astype(f),
                dt_bias=rng.standard_normal(nv).astype(f), ssm_norm=(1 + 0.1 * rng.standard_normal(cfg["d_v"])).astype(f),
                conv_state=rng.standard_normal((ch, K - 1)).astype(f),
                ssm_state=(rng.standard_normal((nv, cfg["d_v"], cfg["d_k"])) * 0.1).astype(f))


def np_gdn(cfg, d):
    nk, nv, dk, dv, K, eps = (cfg[k] for k in ("n_k_heads", "n_v_heads", "d_k", "d_v", "conv_kernel", "eps"))
    silu = lambda x: x / (1 + np.exp(-x))
    cs = d["conv_state"].astype(np.float64).copy()
    S = d["ssm_state"].astype(np.float64).copy()
    w = d["conv_w"].astype(np.float64)
    ys = []
    for t in range(d["qkv"].shape[0]):
        x = d["qkv"][t].astype(np.float64)
        c = silu((cs * w[:, :K - 1]).sum(1) + x * w[:, K - 1])
        cs = np.concatenate([cs[:, 1:], x[:, None]], axis=1)
        qk = c[:2 * nk * dk].reshape(2 * nk, dk)
        qk = qk / np.sqrt((qk ** 2).sum(1, keepdims=True) + eps)
        q, k = qk[:nk], qk[nk:]
        v = c[2 * nk * dk:].reshape(nv, dv)
        out = np.zeros((nv, dv))
        for vh in range(nv):
            kh = vh % nk
            b = 1 / (1 + np.exp(-d["beta"][t, vh]))
            a = d["alpha"][t, vh] + d["dt_bias"][vh]
            sp = a if a > 20 else np.exp(a) if a < -20 else np.log1p(np.exp(a))
            g = np.exp(sp * d["ssm_a"][vh])
            sk = S[vh] @ k[kh]
            dd = (v[vh] - g * sk) * b
            S[vh] = g * S[vh] + np.outer(dd, k[kh])
            out[vh] = (S[vh] @ q[kh]) / np.sqrt(dk)
        inv = 1 / np.sqrt((out ** 2).mean(1, keepdims=True) + eps)
        zz = d["z"][t].astype(np.float64).reshape(nv, dv)
        ys.append((out * inv * d["ssm_norm"][None, :] * silu(zz)).reshape(-1))
    return np.array(ys), cs, S


def test_gdn_oracle_matches_numpy(orc):
    d = gdn_inputs(CFG, 5, 1)
    y, cs, ss = orc.gdn_step(CFG, **d)
    y64, cs64, ss64 = np_gdn(CFG, d)
    assert np.allclose(cs, cs64, rtol=0, atol=0)  # the history is moved, not computed
    assert np.linalg.norm(y - y64) / np.linalg.norm(y64) < 1e-5
    assert np.linalg.norm(ss - ss64) / np.linalg.norm(ss64) < 1e-5
