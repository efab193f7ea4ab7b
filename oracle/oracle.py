"""ctypes binding of the CPU oracle (liboracle.so, built by oracle/Makefile).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py's CPU-baseline / reference leg.  The product
library never loads it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
_lib = None


def build(force: bool = False) -> Path:
    srcs = [HERE / "gguf_oracle.c", HERE / "llama_oracle.c", HERE / "Makefile"]
    if force or not LIB_PATH.exists() or any(s.stat().st_mtime > LIB_PATH.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-s", "-C", str(HERE), "-B" if force else "liboracle.so"],
                       check=True)
    return LIB_PATH


class OracleConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("n_embd", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("n_ff", C.c_int),
                ("n_vocab", C.c_int), ("rms_eps", C.c_float), ("rope_theta", C.c_float)]


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        u8p, f32p, f64p = C.POINTER(C.c_uint8), C.POINTER(C.c_float), C.POINTER(C.c_double)
        L.oracle_f16_to_f32.argtypes = [C.c_uint16]
        L.oracle_f16_to_f32.restype = C.c_float
        L.oracle_dequantize.argtypes = [u8p, C.c_int, C.c_int64, f32p]
        L.oracle_matmul_batched.argtypes = [u8p, C.c_int, C.c_int64, C.c_int64, f32p, C.c_int64, f32p]
        L.oracle_matmul_f64.argtypes = [u8p, C.c_int, C.c_int64, C.c_int64, f32p, C.c_int64, f64p]
        L.oracle_decode_q4k_scales.argtypes = [u8p, u8p, u8p]
        L.oracle_quantize_row_q8_k.argtypes = [f32p, C.c_int64, C.c_void_p]
        L.oracle_quantize_row_q8_0.argtypes = [f32p, C.c_int64, C.c_void_p]
        L.oracle_set_threads.argtypes = [C.c_int]
        L.oracle_model_create.argtypes = [C.POINTER(OracleConfig), C.c_int64]
        L.oracle_model_create.restype = C.c_void_p
        L.oracle_model_free.argtypes = [C.c_void_p]
        L.oracle_clear_state.argtypes = [C.c_void_p]
        L.oracle_fill_kv.argtypes = [C.c_void_p, C.c_int64, C.c_uint64]
        L.oracle_model_set.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                       C.c_int64, C.c_int64]
        L.oracle_forward_ref.argtypes = [C.c_void_p, C.POINTER(C.c_uint32), C.c_int64, C.c_int64, f32p]
        L.oracle_forward_f64.argtypes = [C.c_void_p, C.POINTER(C.c_uint32), C.c_int64, C.c_int64,
                                         C.c_int, f64p]
        L.oracle_rope_table.argtypes = [C.c_void_p, C.c_int]
        L.oracle_rope_table.restype = f32p
        L.oracle_xorshift_f32.argtypes = [C.POINTER(C.c_uint64)]
        L.oracle_xorshift_f32.restype = C.c_float
        L.oracle_sample.argtypes = [f32p, C.c_int64, C.c_float, C.c_float, C.POINTER(C.c_uint64),
                                    C.POINTER(C.c_int)]
        L.oracle_sample.restype = C.c_uint32
        L.oracle_gdn_step.argtypes = [C.c_int] * 5 + [C.c_float, C.c_int] + [f32p] * 11
        _lib = L
    return _lib


def sample(logits: np.ndarray, temperature: float, top_p: float, state: int) -> tuple[int, int, bool]:
    """SelfMadeSampler::sample (inference.rs:1619-1681): (token, new rng
    state, whether the random number was drawn)."""
    v = np.ascontiguousarray(logits, dtype=np.float32).reshape(-1)
    st = C.c_uint64(state if state != 0 else 0x853C49E6748FEA9B)
    drew = C.c_int(0)
    tok = lib().oracle_sample(_p(v, C.c_float), v.size, temperature, top_p, C.byref(st), C.byref(drew))
    return int(tok), int(st.value), bool(drew.value)


def gdn_step(cfg: dict, qkv, z, alpha, beta, conv_w, ssm_a, dt_bias, ssm_norm, conv_state, ssm_state):
    """Gated DeltaNet mixer core (inference.rs:2296-2374) over len(qkv) tokens:
    returns (y, new conv_state, new ssm_state)."""
    f = lambda a: np.ascontiguousarray(a, dtype=np.float32)
    qkv, z, alpha, beta = f(qkv), f(z), f(alpha), f(beta)
    cs, ss = f(conv_state).copy(), f(ssm_state).copy()
    n_tokens = qkv.shape[0]
    y = np.zeros((n_tokens, cfg["n_v_heads"] * cfg["d_v"]), np.float32)
    args = [f(conv_w), f(ssm_a), f(dt_bias), f(ssm_norm)]
    rc = lib().oracle_gdn_step(cfg["n_k_heads"], cfg["n_v_heads"], cfg["d_k"], cfg["d_v"], cfg["conv_kernel"],
                               cfg["eps"], n_tokens, _p(qkv, C.c_float), _p(z, C.c_float), _p(alpha, C.c_float),
                               _p(beta, C.c_float), *[_p(a, C.c_float) for a in args], _p(cs, C.c_float),
                               _p(ss, C.c_float), _p(y, C.c_float))
    if rc != 0:
        raise MemoryError("oracle_gdn_step")
    return y, cs, ss


def _p(a: np.ndarray, ct):
    return a.ctypes.data_as(C.POINTER(ct))


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def f16_to_f32(h: int) -> float:
    return lib().oracle_f16_to_f32(h)


def dequantize(raw: np.ndarray, dtype: int, n_elems: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n_elems, dtype=np.float32)
    rc = lib().oracle_dequantize(_p(raw, C.c_uint8), dtype, n_elems, _p(out, C.c_float))
    if rc != 0:
        raise ValueError(f"oracle: dequantization not implemented for type {dtype}")
    return out


def decode_q4k_scales(s12: np.ndarray):
    s12 = np.ascontiguousarray(s12, dtype=np.uint8)
    sc = np.empty(8, np.uint8)
    m = np.empty(8, np.uint8)
    lib().oracle_decode_q4k_scales(_p(s12, C.c_uint8), _p(sc, C.c_uint8), _p(m, C.c_uint8))
    return sc, m


def matmul_batched(raw: np.ndarray, dtype: int, n: int, k: int, x: np.ndarray) -> np.ndarray:
    """The reference's CPU matvec (quantised-x AVX2 path): y [m, n] f32."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    m = x.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    rc = lib().oracle_matmul_batched(_p(raw, C.c_uint8), dtype, n, k, _p(x, C.c_float), m,
                                     _p(out, C.c_float))
    if rc != 0:
        raise ValueError("oracle matmul failed")
    return out


def matmul_f64(raw: np.ndarray, dtype: int, n: int, k: int, x: np.ndarray) -> np.ndarray:
    """fp64 matvec over the bit-exact dequantised weights: y [m, n] f64."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    m = x.shape[0]
    out = np.empty((m, n), dtype=np.float64)
    rc = lib().oracle_matmul_f64(_p(raw, C.c_uint8), dtype, n, k, _p(x, C.c_float), m,
                                 _p(out, C.c_double))
    if rc != 0:
        raise ValueError("oracle matmul_f64 failed")
    return out


# role ids of oracle_model_set (llama_oracle.c)
ROLES = {"token_embd": 0, "output": 1, "output_norm": 2, "attn_norm": 3, "attn_q": 4,
         "attn_k": 5, "attn_v": 6, "attn_output": 7, "ffn_norm": 8, "ffn_gate": 9,
         "ffn_up": 10, "ffn_down": 11, "attn_q.bias": 12, "attn_k.bias": 13, "attn_v.bias": 14}


class Model:
    """The reference Llama forward over borrowed host tensors.

    `tensors` maps GGUF names ("blk.0.attn_q.weight", "output_norm.weight",
    ...) to (dtype, dims[outer.., inner], uint8/float32 array)."""

    def __init__(self, cfg: dict, tensors: dict, kv_capacity: int):
        self.cfg = cfg
        oc = OracleConfig(cfg["n_layers"], cfg["n_embd"], cfg["n_heads"], cfg["n_kv_heads"],
                          cfg["head_dim"], cfg["n_ff"], cfg["n_vocab"], cfg["rms_eps"],
                          cfg["rope_theta"])
        self._h = lib().oracle_model_create(C.byref(oc), kv_capacity)
        self._keep = []
        for name, (dtype, dims, arr) in tensors.items():
            arr = np.ascontiguousarray(arr)
            self._keep.append(arr)
            parts = name.split(".")
            if parts[0] == "blk":
                layer = int(parts[1])
                role = ".".join(parts[2:]).replace(".weight", "")
            else:
                layer = -1
                role = parts[0]
            if role not in ROLES:
                continue
            n = dims[0] if len(dims) > 1 else 1
            k = dims[-1]
            rc = lib().oracle_model_set(self._h, ROLES[role], layer, arr.ctypes.data, dtype, n, k)
            if rc != 0:
                raise ValueError(f"oracle: cannot set {name}")
        if "output.weight" not in tensors:  # tied head falls back to token_embd (inference.rs:2560)
            dtype, dims, arr = tensors["token_embd.weight"]
            lib().oracle_model_set(self._h, ROLES["output"], -1, np.ascontiguousarray(arr).ctypes.data,
                                   dtype, dims[0], dims[-1])

    def clear_state(self):
        lib().oracle_clear_state(self._h)

    def fill_kv(self, n: int, seed: int = 0) -> None:
        """Timing set-up: n positions of seeded synthetic rows in the
        reference path's f32 KV cache (decode steps then run at context n)."""
        if lib().oracle_fill_kv(self._h, n, seed) != 0:
            raise ValueError("oracle fill_kv: n exceeds the KV capacity")

    def forward_ref(self, tokens, start_pos: int) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self.cfg["n_vocab"], dtype=np.float32)
        rc = lib().oracle_forward_ref(self._h, _p(t, C.c_uint32), len(t), start_pos, _p(out, C.c_float))
        if rc != 0:
            raise RuntimeError(f"oracle forward_ref failed: {rc}")
        return out

    def forward_f64(self, tokens, start_pos: int, kv_f16: bool = True) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self.cfg["n_vocab"], dtype=np.float64)
        rc = lib().oracle_forward_f64(self._h, _p(t, C.c_uint32), len(t), start_pos, int(kv_f16),
                                      _p(out, C.c_double))
        if rc != 0:
            raise RuntimeError(f"oracle forward_f64 failed: {rc}")
        return out

    def rope_tables(self):
        half = self.cfg["head_dim"] // 2
        cs = np.ctypeslib.as_array(lib().oracle_rope_table(self._h, 1), shape=(8192 * half,)).copy()
        sn = np.ctypeslib.as_array(lib().oracle_rope_table(self._h, 0), shape=(8192 * half,)).copy()
        return cs, sn

    def __del__(self):
        try:
            if self._h:
                lib().oracle_model_free(self._h)
                self._h = None
        except Exception:
            pass
