"""The allocation-free matvec entry point, b2q_matmul_noalloc_dev.

It exists for callers that cannot allocate device memory (a fixed memory
pool, a real-time path, a host that owns the allocator).  Its scratch is a
fixed array inside the library; here it is called through the C ABI twice in
a row and checked against the allocating entry point, b2q_matmul_dev, with
the matvec tolerance of the other GPU tests.  The file is named to be
collected last, and it needs no state from other tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3


def test_noalloc_matches_matmul_dev_twice(engine, pkg):
    import torch
    from hf_llm_b200 import ggml, synth
    from hf_llm_b200._lib import check, lib
    n, k = 3072, 4096
    raw = synth.tensor_rows(ggml.Q4_K, n, k, 31, 5)
    w = engine.try_upload_weight(raw, ggml.Q4_K, n, k)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        m = 1 + call  # one token, then two
        x = torch.from_numpy(synth.activation(k, 40 + call, m)).cuda()
        y_ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
        y_na = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        check(lib().b2q_matmul_dev(engine.handle, w.handle, x.data_ptr(), y_ref.data_ptr(), m, n, k, stream))
        check(lib().b2q_matmul_noalloc_dev(w.handle, x.data_ptr(), y_na.data_ptr(), m, n, k, stream))
        torch.cuda.synchronize()
        a, b = y_na.cpu().numpy(), y_ref.cpu().numpy()
        assert np.all(np.isfinite(a))
        assert rel_l2(a, b) <= TOL, f"call {call}: rel-L2 {rel_l2(a, b)}"


def test_noalloc_rejects_oversized_input(engine, pkg):
    from hf_llm_b200 import ggml, synth
    from hf_llm_b200._lib import EINVAL, lib
    n, k = 64, 65536
    raw = synth.tensor_rows(ggml.Q8_0, n, k, 1, 1)
    w = engine.try_upload_weight(raw, ggml.Q8_0, n, k)
    # 8 tokens x 65536 = 524288 activations > the 262144 the scratch holds;
    # rejected before any pointer is touched
    st = lib().b2q_matmul_noalloc_dev(w.handle, C.c_void_p(16), C.c_void_p(16), 8, n, k, None)
    assert st == EINVAL
    assert b"exceeds" in lib().b2q_last_error()
