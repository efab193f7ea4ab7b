"""Parity of the sm_100a kernels with the CPU oracle, through the C ABI.

* Dequantisation is bit-exact (dequantize_slice, inference.rs:1347-1474),
  including f16 subnormal and inf scales.  The F16 conversion keeps NaN
  payloads exactly; a NaN produced by arithmetic (NaN * x, inf - inf) is
  compared as NaN only, since its payload is platform-defined (x86 returns
  the input NaN or its default NaN, the GPU a canonical NaN).
* Matvec results are within rel-L2 <= 1e-3 of an fp64 matvec over the
  bit-exact dequantised weights (the tolerance of the decode path).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3  # rel-L2 against fp64
GOLD = Path(__file__).resolve().parent / "golden" / "dequant_golden.npz"
QK = {12: 256, 14: 256, 8: 32, 13: 256, 2: 32}


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def test_library_is_native(engine):
    from hf_llm_b200 import _lib
    assert engine.device_name, "no device name"
    assert "sm_100a" in _lib.lib().b2q_version().decode()


@pytest.mark.parametrize("name,dtype", [("Q4_K", 12), ("Q6_K", 14), ("Q8_0", 8), ("Q5_K", 13),
                                        ("Q4_0", 2)])
def test_dequant_bit_exact_golden(engine, orc, torch_cuda, name, dtype):
    torch = torch_cuda
    g = np.load(GOLD)
    raw = g[f"{name}_raw"].reshape(-1)
    n_el = g[f"{name}_raw"].shape[0] * QK[dtype]
    want = orc.dequantize(raw, dtype, n_el)
    d_raw = torch.from_numpy(raw.copy()).cuda()
    d_out = torch.empty(n_el, dtype=torch.float32, device="cuda")
    engine.dequantize_dev(d_raw.data_ptr(), dtype, n_el, d_out.data_ptr(),
                          torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = d_out.cpu().numpy()
    nan = np.isnan(got) & np.isnan(want)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got.view(np.uint32)[~nan], want.view(np.uint32)[~nan])
    assert (~nan).sum() > 0.9 * got.size


def test_dequant_f16_all_patterns(engine, orc, torch_cuda):
    torch = torch_cuda
    bits = np.arange(65536, dtype=np.uint16)
    want = orc.dequantize(bits.view(np.uint8), 1, bits.size)
    d_raw = torch.from_numpy(bits.view(np.uint8).copy()).cuda()
    d_out = torch.empty(bits.size, dtype=torch.float32, device="cuda")
    engine.dequantize_dev(d_raw.data_ptr(), 1, bits.size, d_out.data_ptr(),
                          torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(d_out.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("dtype", [12, 14, 8])
def test_dequant_bit_exact_random(engine, orc, torch_cuda, pkg, dtype):
    from hf_llm_b200 import synth
    torch = torch_cuda
    raw = synth.tensor_rows(dtype, 97, 1024, 21, 3).reshape(-1)
    want = orc.dequantize(raw, dtype, 97 * 1024)
    d_raw = torch.from_numpy(raw.copy()).cuda()
    d_out = torch.empty(97 * 1024, dtype=torch.float32, device="cuda")
    engine.dequantize_dev(d_raw.data_ptr(), dtype, 97 * 1024, d_out.data_ptr(), 0)
    torch.cuda.synchronize()
    assert np.array_equal(d_out.cpu().numpy().view(np.uint32), want.view(np.uint32))


SHAPES_SMALL = [(1, 256), (7, 512), (33, 1024), (300, 4096), (129, 2304)]


def _check_matvec(engine, orc, pkg, dtype, n, k, m=1, seed=0, dist="bench"):
    from hf_llm_b200 import synth
    raw = synth.tensor_rows(dtype, n, k, seed + 1, 7, dist=dist)
    x = synth.activation(k, seed + 2, m)
    buf = engine.try_upload_weight(raw, dtype, n, k)
    y = engine.matmul_batched(buf, x, m, n, k)
    y64 = orc.matmul_f64(raw, dtype, n, k, x)
    err = rel_l2(y, y64)
    assert err <= TOL, f"type {dtype} [{n},{k}] m={m}: rel-L2 {err:.3g}"
    return err


@pytest.mark.parametrize("dtype", [12, 14, 8, 13, 2])
@pytest.mark.parametrize("n,k", SHAPES_SMALL)
def test_matvec_small_shapes(engine, orc, pkg, dtype, n, k):
    if k % 256 and dtype not in (8, 2):
        pytest.skip("K-quants need k % 256 == 0")
    _check_matvec(engine, orc, pkg, dtype, n, k)


@pytest.mark.parametrize("dtype,n,k", [
    (8, 4096, 4096),                                   # Q8_0 matvec config
    (12, 4096, 4096), (12, 1024, 4096), (12, 14336, 4096), (12, 4096, 14336),  # Q4_K set
    (14, 1024, 4096), (14, 4096, 14336),               # Q6_K attn_v / ffn_down
])
def test_matvec_config_shapes(engine, orc, pkg, dtype, n, k):
    _check_matvec(engine, orc, pkg, dtype, n, k, seed=5)


def test_matvec_q6k_output_head(engine, orc, pkg):
    _check_matvec(engine, orc, pkg, 14, 128256, 4096, seed=9)


@pytest.mark.parametrize("m", [2, 3, 8, 11, 17])
@pytest.mark.parametrize("dtype", [12, 14, 8, 13, 2])
def test_matvec_multi_token(engine, orc, pkg, dtype, m):
    _check_matvec(engine, orc, pkg, dtype, 520, 1024, m=m, seed=m)


@pytest.mark.parametrize("dtype,n,k", [(13, 4096, 4096), (13, 14336, 4096), (13, 4096, 14336), (2, 4096, 4096),
                                       (2, 1024, 4096)])
def test_matvec_q5k_q40_model_shapes(engine, orc, pkg, dtype, n, k):
    """Q5_K and Q4_0 (the other types the reference's GPU engine loads,
    gpu.rs:316-318) at Llama-3-8B shapes."""
    _check_matvec(engine, orc, pkg, dtype, n, k, seed=11)


def test_matvec_unit_distribution(engine, orc, pkg):
    for dtype in (12, 14, 8, 13, 2):
        _check_matvec(engine, orc, pkg, dtype, 1000, 4096, dist="unit")


def test_matvec_zero_and_ragged_inputs(engine, orc, pkg):
    from hf_llm_b200 import ggml, synth
    n, k = 64, 1024
    raw = synth.tensor_rows(ggml.Q4_K, n, k, 3, 3)
    buf = engine.try_upload_weight(raw, ggml.Q4_K, n, k)
    x = np.zeros((1, k), np.float32)
    assert np.array_equal(engine.matmul_batched(buf, x, 1, n, k), np.zeros((1, n), np.float32))
    # one non-zero block, huge dynamic range between blocks
    x = synth.activation(k, 4)
    x[0, 32:] *= 1e-6
    x[0, :32] *= 1e4
    y = engine.matmul_batched(buf, x, 1, n, k)
    y64 = orc.matmul_f64(raw, ggml.Q4_K, n, k, x)
    assert rel_l2(y, y64) <= TOL


@pytest.mark.parametrize("dtype", [12, 14, 8])
def test_matvec_nan_activation_elements(engine, orc, pkg, dtype):
    """A NaN activation element contributes nothing and leaves the rest of
    its block intact, as in quantize_row_q8_k (inference.rs:933-962: NaN
    never wins the |x| scan, `NaN as i8` is 0): the matvec equals the
    fp64 one over the activations with the NaN elements set to zero, for
    one token, for several (GEMV) and for enough to take the tensor-core
    path."""
    from hf_llm_b200 import ggml, synth
    n, k = 512, 4096
    raw = synth.tensor_rows(dtype, n, k, 3, 21)
    buf = engine.try_upload_weight(raw, dtype, n, k)
    for m in (1, 5, 20):  # 20 tokens: the tensor-core path
        x = np.concatenate([synth.activation(k, 30 + t) for t in range(m)], axis=0)
        x[0, [3, 64, 65, 1000, 4095]] = np.nan  # blocks 0, 1, 15 and 63 keep their other elements
        if m > 1:
            x[m - 1, 128:192] = np.nan             # a whole block
        y = engine.matmul_batched(buf, x, m, n, k)
        assert np.isfinite(y).all()
        y64 = orc.matmul_f64(raw, dtype, n, k, np.nan_to_num(x, nan=0.0))
        assert rel_l2(y, y64) <= TOL, f"type {dtype} m={m}: rel-L2 {rel_l2(y, y64):.3g}"


def test_matmul_group_same_input(engine, orc, pkg):
    """QKV-style group: outputs concatenated in order (gpu.rs:617-646)."""
    from hf_llm_b200 import ggml, synth
    k = 4096
    specs = [(ggml.Q4_K, 4096), (ggml.Q4_K, 1024), (ggml.Q6_K, 1024), (ggml.Q8_0, 256), (ggml.Q4_K, 256)]
    raws = [synth.tensor_rows(t, n, k, 2, i) for i, (t, n) in enumerate(specs)]
    bufs = [engine.try_upload_weight(r, t, n, k) for r, (t, n) in zip(raws, specs)]
    x = synth.activation(k, 8, 2)
    outs = engine.matmul_group_same_input([(b, n) for b, (_, n) in zip(bufs, specs)], x, 2, k)
    for o, r, (t, n) in zip(outs, raws, specs):
        assert o.shape == (2, n)
        assert rel_l2(o, orc.matmul_f64(r, t, n, k, x)) <= TOL


@pytest.mark.parametrize("m", [1, 3])
def test_ffn_swiglu(engine, orc, pkg, m):
    from hf_llm_b200 import ggml, synth
    E, F = 1024, 2816
    g = synth.tensor_rows(ggml.Q4_K, F, E, 1, 1, dist="unit")
    u = synth.tensor_rows(ggml.Q4_K, F, E, 1, 2, dist="unit")
    d = synth.tensor_rows(ggml.Q6_K, E, F, 1, 3, dist="unit")
    bg, bu, bd = (engine.try_upload_weight(g, ggml.Q4_K, F, E), engine.try_upload_weight(u, ggml.Q4_K, F, E),
                  engine.try_upload_weight(d, ggml.Q6_K, E, F))
    x = synth.activation(E, 3, m)
    y = engine.ffn_swiglu_fused(bg, bu, bd, x, m, E, F)
    gg = orc.matmul_f64(g, ggml.Q4_K, F, E, x)
    uu = orc.matmul_f64(u, ggml.Q4_K, F, E, x)
    h = gg / (1.0 + np.exp(-gg)) * uu
    wd = orc.dequantize(d.reshape(-1), ggml.Q6_K, E * F).reshape(E, F).astype(np.float64)
    y64 = h @ wd.T
    assert rel_l2(y, y64) <= TOL


def test_error_paths(engine, pkg):
    from hf_llm_b200 import ggml, synth
    from hf_llm_b200._lib import B2QError, EINVAL, EUNSUP
    raw = synth.tensor_rows(ggml.Q4_K, 8, 256, 1, 1)
    with pytest.raises(B2QError) as e:
        engine.try_upload_weight(raw[:, :100], ggml.Q4_K, 8, 256)  # short buffer
    assert e.value.status == EINVAL
    with pytest.raises(B2QError) as e:
        engine.try_upload_weight(raw, 3, 8, 256)  # Q4_1: no kernel
    assert e.value.status == EUNSUP
    buf = engine.try_upload_weight(raw, ggml.Q4_K, 8, 256)
    with pytest.raises(B2QError) as e:
        engine.matmul_batched(buf, np.zeros(512, np.float32), 1, 8, 512)  # k mismatch
    assert e.value.status == EINVAL
    engine.check_device_error()


def test_dev_pointer_matmul_matches_host(engine, pkg, torch_cuda):
    from hf_llm_b200 import ggml, synth
    torch = torch_cuda
    n, k = 2048, 4096
    raw = synth.tensor_rows(ggml.Q4_K, n, k, 4, 4)
    buf = engine.try_upload_weight(raw, ggml.Q4_K, n, k)
    x = synth.activation(k, 1)
    y_host = engine.matmul_batched(buf, x, 1, n, k)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty((1, n), dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream()
    engine.matmul_dev(buf, dx.data_ptr(), dy.data_ptr(), 1, n, k, s.cuda_stream)
    s.synchronize()
    assert np.array_equal(dy.cpu().numpy(), y_host)
