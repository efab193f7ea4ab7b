"""ctypes binding of libb2q.so (the C ABI declared in include/b2q.h).

The library must be built (build.py) before use; there is no fallback: a
missing library or a failing call raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
# B2Q_CHECKS=1 selects the debug-bounds build (build.py --checks), the same
# kernels with index and layout checks compiled in
LIB_PATH = HERE / ("libb2q_checks.so" if os.environ.get("B2Q_CHECKS") == "1" else "libb2q.so")

OK, EINVAL, ENOMEM, ECUDA, ENCCL, ETIMEOUT, EUNSUP = range(7)
_STATUS_NAMES = {0: "B2Q_OK", 1: "B2Q_EINVAL", 2: "B2Q_ENOMEM", 3: "B2Q_ECUDA",
                 4: "B2Q_ENCCL", 5: "B2Q_ETIMEOUT", 6: "B2Q_EUNSUP"}


class B2QError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{_STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class GdnConfig(C.Structure):
    _fields_ = [("n_k_heads", C.c_int), ("n_v_heads", C.c_int), ("d_k", C.c_int), ("d_v", C.c_int),
                ("conv_kernel", C.c_int), ("eps", C.c_float)]


class ModelConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("n_embd", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("n_ff", C.c_int),
                ("n_vocab", C.c_int), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
                ("max_seq", C.c_int), ("tp_rank", C.c_int), ("tp_size", C.c_int),
                ("no_graph", C.c_int)]


# (name, restype, argtypes) for every symbol of include/b2q.h
_VP, _I, _I64, _SZ, _F = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_float
_FP = C.POINTER(C.c_float)
_U32P = C.POINTER(C.c_uint32)
SIGNATURES = [
    ("b2q_last_error", C.c_char_p, []),
    ("b2q_version", C.c_char_p, []),
    ("b2q_init", _I, [_I, C.POINTER(_VP)]),
    ("b2q_engine_destroy", _I, [_VP]),
    ("b2q_device_info", _I, [_VP, C.c_char_p, _SZ, C.POINTER(_SZ), C.POINTER(_SZ)]),
    ("b2q_can_alloc", _I, [_VP, _SZ, _SZ]),
    ("b2q_upload_weight", _I, [_VP, _VP, _SZ, _I, _I64, _I64, C.POINTER(_VP)]),
    ("b2q_weight_free", _I, [_VP]),
    ("b2q_weight_bytes", _SZ, [_VP]),
    ("b2q_matmul", _I, [_VP, _VP, _FP, _FP, _I, _I, _I]),
    ("b2q_matmul_dev", _I, [_VP, _VP, _VP, _VP, _I, _I, _I, _VP]),
    ("b2q_matmul_noalloc_dev", _I, [_VP, _VP, _VP, _I, _I, _I, _VP]),
    ("b2q_matmul_group", _I, [_VP, C.POINTER(_VP), C.POINTER(_I), _I, _FP, _I, _I, _FP]),
    ("b2q_matmul_group_dev", _I, [_VP, C.POINTER(_VP), C.POINTER(_I), _I, _VP, _I, _I, _VP, _VP]),
    ("b2q_ffn_swiglu", _I, [_VP, _VP, _VP, _VP, _FP, _I, _I, _I, _FP]),
    ("b2q_ffn_swiglu_dev", _I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _VP, _VP]),
    ("b2q_dequantize_dev", _I, [_VP, _VP, _I, _I64, _VP, _VP]),
    ("b2q_tp_unique_id", _I, [C.POINTER(C.c_ubyte)]),
    ("b2q_model_create", _I, [_VP, C.POINTER(ModelConfig), C.POINTER(C.c_ubyte), C.POINTER(_VP)]),
    ("b2q_model_set_tensor", _I, [_VP, C.c_char_p, _I, C.POINTER(_I64), _I, _VP, _SZ]),
    ("b2q_model_set_tensor_rows", _I, [_VP, C.c_char_p, _I, C.POINTER(_I64), _I, _I64, _I64, _VP, _SZ]),
    ("b2q_model_shard_rows", _I, [_VP, C.c_char_p, _I64, C.POINTER(_I64), C.POINTER(_I64)]),
    ("b2q_tp_shard_rows", _I, [C.POINTER(ModelConfig), C.c_char_p, _I64, C.POINTER(_I64), C.POINTER(_I64)]),
    ("b2q_tp_shard_cols", _I, [C.POINTER(ModelConfig), C.c_char_p, _I64, C.POINTER(_I64), C.POINTER(_I64)]),
    ("b2q_model_finalize", _I, [_VP]),
    ("b2q_forward", _I, [_VP, _U32P, _I, _I, _FP, _U32P]),
    ("b2q_forward_dev", _I, [_VP, _VP, _I, _I, _VP, _VP, _VP]),
    ("b2q_clear_state", _I, [_VP]),
    ("b2q_forward_sample", _I, [_VP, _U32P, _I, _I, _F, _F, C.POINTER(C.c_uint64), _U32P]),
    ("b2q_sampler_state", C.c_uint64, [C.c_uint64]),
    ("b2q_sample_dev", _I, [_VP, _VP, _I, _F, _F, C.POINTER(C.c_uint64), _U32P, _VP]),
    ("b2q_gdn_step_dev", _I, [_VP, C.POINTER(GdnConfig), _I] + [_VP] * 12),
    ("b2q_gguf_open", _I, [C.c_char_p, C.POINTER(_VP)]),
    ("b2q_gguf_close", _I, [_VP]),
    ("b2q_gguf_version", _I, [_VP]),
    ("b2q_gguf_n_tensors", _I64, [_VP]),
    ("b2q_gguf_n_kv", _I64, [_VP]),
    ("b2q_gguf_kv_key", _I, [_VP, _I64, C.POINTER(C.c_char_p), C.POINTER(_I)]),
    ("b2q_gguf_tensor_info", _I, [_VP, _I64, C.POINTER(C.c_char_p), C.POINTER(_I), C.POINTER(_I),
                                  C.POINTER(_I64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    ("b2q_gguf_find_tensor", _I, [_VP, C.c_char_p, C.POINTER(_I64)]),
    ("b2q_gguf_tensor_data", _VP, [_VP, _I64]),
    ("b2q_gguf_get_usize", _I, [_VP, C.c_char_p, C.POINTER(C.c_uint64)]),
    ("b2q_gguf_get_f32", _I, [_VP, C.c_char_p, C.POINTER(C.c_float)]),
    ("b2q_gguf_get_str", _I, [_VP, C.c_char_p, C.POINTER(_VP), C.POINTER(_SZ)]),
    ("b2q_gguf_llama_config", _I, [_VP, C.c_char_p, C.POINTER(ModelConfig)]),
    ("b2q_model_load_gguf", _I, [_VP, _VP]),
    ("b2q_model_weight_bytes", _SZ, [_VP]),
    ("b2q_model_step_path", _I, [_VP]),
    ("b2q_model_destroy", _I, [_VP]),
    ("b2q_time_gemv", _I, [_VP, C.POINTER(_VP), _I, _VP, _I, _I, _VP, C.POINTER(C.c_float), _I]),
    ("b2q_kernel_launch_count", C.c_uint64, [_VP]),
    ("b2q_check_device_error", _I, [_VP]),
    ("b2q_debug_checks_enabled", _I, []),
    ("b2q_debug_check_site", _I, [_VP, C.POINTER(_I)]),
    ("b2q_set_wait_limit_cycles", _I, [_VP, C.c_longlong]),
    ("b2q_model_debug_desync", _I, [_VP]),
    ("b2q_model_fill_kv", _I, [_VP, _I, _I, C.c_uint64, _F]),
    ("b2q_set_tp_init_timeout_ms", _I, [_I]),
]

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise B2QError(EUNSUP, f"{LIB_PATH} is not built; run build.py (nvcc, sm_100a)")
        L = C.CDLL(str(LIB_PATH))
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != OK:
        msg = lib().b2q_last_error()
        raise B2QError(status, msg.decode() if msg else "")
