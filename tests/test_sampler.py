"""The sampler oracle (oracle/llama_oracle.c oracle_sample), a restatement
of SelfMadeSampler (src/inference.rs:1600-1681), checked on CPU against an
independent Python restatement of the same steps and against xorshift64
values computed here by hand."""
from __future__ import annotations

import math

import numpy as np
import pytest

DEFAULT_STATE = 0x853C49E6748FEA9B
M64 = (1 << 64) - 1


def xorshift(state: int) -> tuple[int, float]:
    x = state
    x ^= (x << 13) & M64
    x ^= x >> 7
    x ^= (x << 17) & M64
    return x, np.float32((x >> 40) & 0xFFFFFFFF) / np.float32(1 << 24)


def py_sample(logits: np.ndarray, temperature: float, top_p: float, state: int):
    """Step-by-step restatement (f32 arithmetic through numpy scalars)."""
    f = np.float32
    if temperature <= 1e-5:
        best, bv = 0, f(-np.inf)
        for i, v in enumerate(logits):
            if v > bv:
                bv, best = v, i
        return best, state, False
    inv = f(1.0) / f(temperature)
    mx = f(-np.inf)
    for v in logits:
        if v > mx:
            mx = v
    cutoff = f(mx - f(14.0) * f(temperature))
    cands, s = [], f(0.0)
    for i, v in enumerate(logits):
        if v >= cutoff:
            p = f(math.exp(f((v - mx) * inv)))
            cands.append((i, p))
            s = f(s + p)
    if not cands or s <= 0:
        return 0, state, False
    cands.sort(key=lambda c: (-c[1], c[0]))
    target = f(s * f(top_p))
    cum, keep = f(0.0), len(cands)
    for idx, (_, p) in enumerate(cands):
        cum = f(cum + p)
        if cum >= target:
            keep = idx + 1
            break
    state, u = xorshift(state)
    r = f(u * min(cum, s))
    acc = f(0.0)
    for i, p in cands[:keep]:
        acc = f(acc + p)
        if r <= acc:
            return i, state, True
    return cands[0][0], state, True


@pytest.fixture(scope="module")
def orc_s(orc):
    return orc


def test_xorshift_known_values(orc_s):
    import ctypes as C
    st = C.c_uint64(DEFAULT_STATE)
    s = DEFAULT_STATE
    for _ in range(6):
        s, u = xorshift(s)
        v = orc_s.lib().oracle_xorshift_f32(C.byref(st))
        assert st.value == s
        assert np.float32(v) == u
        assert 0.0 <= u < 1.0


@pytest.mark.parametrize("temperature,top_p", [(0.0, 0.9), (0.7, 0.9), (1.0, 1.0), (1.5, 0.5), (0.3, 0.05)])
def test_oracle_matches_python_restatement(orc_s, temperature, top_p):
    rng = np.random.default_rng(7)
    state = DEFAULT_STATE
    for trial in range(25):
        n = int(rng.integers(1, 300))
        logits = (rng.standard_normal(n) * rng.uniform(0.1, 6.0)).astype(np.float32)
        if trial % 5 == 0:
            logits[rng.integers(0, n, size=max(1, n // 4))] = logits.max()  # ties at the top
        want = py_sample(logits, temperature, top_p, state)
        got = orc_s.sample(logits, temperature, top_p, state)
        assert got == want, (trial, got, want)
        state = got[1]


def test_oracle_edge_cases(orc_s):
    # all -inf: every logit passes the (-inf) cutoff, the weights are NaN, the
    # sampler draws and returns its first candidate
    neg = np.full(10, -np.inf, dtype=np.float32)
    assert orc_s.sample(neg, 1.0, 0.9, 5) == (0, xorshift(5)[0], True)
    # all NaN: no candidate (NaN fails every comparison): token 0, no draw
    nan = np.full(10, np.nan, dtype=np.float32)
    assert orc_s.sample(nan, 1.0, 0.9, 5) == (0, 5, False)
    one = np.array([0.5], dtype=np.float32)
    tok, st, drew = orc_s.sample(one, 1.0, 0.9, 5)
    assert (tok, drew) == (0, True) and st == xorshift(5)[0]
