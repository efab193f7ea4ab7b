"""The allocation-free matvec entry point, b2q_matmul_noalloc_dev.

It exists for callers that cannot allocate device memory: code that runs
inside a memory pool fixed for the life of the process, a real-time path
that cannot take the implicit synchronisation of an allocation, or a host
that owns the device allocator.  Its only scratch, the quantised
activations, is a fixed array inside the library.

Checked here, always through the C ABI and twice in a row on the same
weight (the array keeps the previous call's contents):
  * below 16 tokens both entry points run the same quantiser and GEMV, so
    the outputs must be bit-identical to b2q_matmul_dev, and within rel-L2
    1e-3 of the oracle's fp64 matvec;
  * a call that fills the scratch exactly (m * round_up(k, 256) = 262144),
    with an inner dimension that is not a multiple of 256 (the padding);
  * 16 tokens and more: the no-alloc call stays on the GEMV path while
    b2q_matmul_dev moves to the tensor cores, so the two are compared with
    the fp64 oracle, each within 1e-3;
  * oversized inputs are rejected before any pointer is touched.
The file is named to be collected last; it needs no state from other tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3  # rel-L2 against the fp64 oracle, as every matvec test


def _both(engine, w, x_host, m, n, k):
    """(no-alloc output, b2q_matmul_dev output) for the same inputs."""
    import torch
    from hf_llm_b200._lib import check, lib
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.from_numpy(np.ascontiguousarray(x_host, dtype=np.float32)).cuda()
    y_ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
    y_na = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    check(lib().b2q_matmul_noalloc_dev(w.handle, x.data_ptr(), y_na.data_ptr(), m, n, k, stream))
    check(lib().b2q_matmul_dev(engine.handle, w.handle, x.data_ptr(), y_ref.data_ptr(), m, n, k, stream))
    torch.cuda.synchronize()
    return y_na.cpu().numpy(), y_ref.cpu().numpy()


@pytest.mark.parametrize("dtype_name,n,k,ms", [
    ("Q4_K", 3072, 4096, (1, 2)),       # one token, then two
    ("Q4_K", 512, 65536, (4, 4)),       # m * k = 262144: the whole scratch
    ("Q8_0", 256, 65280, (4, 3)),       # k % 256 != 0: padded to 65536, the whole scratch
    ("Q6_K", 1024, 14336, (15, 2)),     # the largest GEMV-only batch, then a small one
])
def test_noalloc_bit_identical_to_matmul_dev_twice(engine, orc, pkg, dtype_name, n, k, ms):
    from hf_llm_b200 import ggml, synth
    dtype = getattr(ggml, dtype_name)
    raw = synth.tensor_rows(dtype, n, k, 31, 5)
    w = engine.try_upload_weight(raw, dtype, n, k)
    for call, m in enumerate(ms):
        x = synth.activation(k, 40 + call, m)
        a, b = _both(engine, w, x, m, n, k)
        assert np.all(np.isfinite(a)), f"call {call}: unwritten outputs"
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"call {call}: differs from b2q_matmul_dev"
        want = orc.matmul_f64(raw, dtype, n, k, x)
        assert rel_l2(a, want) <= TOL, f"call {call}: rel-L2 {rel_l2(a, want)} against fp64"
    w.free()


def test_noalloc_many_tokens_stays_on_gemv(engine, orc, pkg):
    """m >= 16: the no-alloc call runs GEMV passes of one or two tokens,
    b2q_matmul_dev the tensor-core GEMM; both within 1e-3 of fp64, twice."""
    from hf_llm_b200 import ggml, synth
    n, k = 2048, 4096
    raw = synth.tensor_rows(ggml.Q4_K, n, k, 7, 9)
    w = engine.try_upload_weight(raw, ggml.Q4_K, n, k)
    for call, m in enumerate((16, 48)):
        x = synth.activation(k, 60 + call, m)
        a, b = _both(engine, w, x, m, n, k)
        want = orc.matmul_f64(raw, ggml.Q4_K, n, k, x)
        assert rel_l2(a, want) <= TOL, f"call {call}: no-alloc rel-L2 {rel_l2(a, want)}"
        assert rel_l2(b, want) <= TOL, f"call {call}: matmul_dev rel-L2 {rel_l2(b, want)}"
    w.free()


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
    w.free()
