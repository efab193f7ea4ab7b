"""GGUF files through the C ABI (b2q_gguf_*): the mirror of the reference's
GgufModelFile (src/inference.rs:235-510).

The parser and the mapping live in libb2q.so; this class only exposes them:
tensor descriptors (dims [outer.., inner], GGML type, absolute offset, byte
length), zero-copy numpy views of tensor bytes, the metadata accessors
get_usize / get_f32 / get_str, and the Llama hyperparameters of from_gguf.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import ModelConfig, check, lib


@dataclass(frozen=True)
class TensorDesc:
    """GgufTensorDesc (inference.rs:236-244)."""
    name: str
    dims: tuple
    dtype: int
    abs_offset: int
    byte_len: int


class GgufFile:
    """A read-only mapped GGUF file (GgufModelFile::open, inference.rs:343-446)."""

    def __init__(self, path):
        h = C.c_void_p()
        check(lib().b2q_gguf_open(str(path).encode(), C.byref(h)))
        self._h = h
        self.path = str(path)

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    @property
    def version(self) -> int:
        return int(lib().b2q_gguf_version(self._h))

    def keys(self) -> list[str]:
        out = []
        for i in range(int(lib().b2q_gguf_n_kv(self._h))):
            k = C.c_char_p()
            check(lib().b2q_gguf_kv_key(self._h, i, C.byref(k), None))
            out.append(k.value.decode())
        return out

    def tensors(self) -> list[TensorDesc]:
        return [self._desc(i) for i in range(int(lib().b2q_gguf_n_tensors(self._h)))]

    def _desc(self, i: int) -> TensorDesc:
        name, t, nd = C.c_char_p(), C.c_int(), C.c_int()
        dims = (C.c_int64 * 8)()
        off, blen = C.c_uint64(), C.c_uint64()
        check(lib().b2q_gguf_tensor_info(self._h, i, C.byref(name), C.byref(t), C.byref(nd), dims,
                                         C.byref(off), C.byref(blen)))
        return TensorDesc(name.value.decode(), tuple(dims[:nd.value]), t.value, off.value, blen.value)

    def tensor(self, name: str) -> TensorDesc:
        i = C.c_int64()
        check(lib().b2q_gguf_find_tensor(self._h, name.encode(), C.byref(i)))
        return self._desc(i.value)

    def has_tensor(self, name: str) -> bool:
        return name in {d.name for d in self.tensors()}

    def tensor_bytes(self, name: str) -> np.ndarray:
        """Zero-copy uint8 view of the tensor's bytes in the mapping (valid
        while this file is open)."""
        i = C.c_int64()
        check(lib().b2q_gguf_find_tensor(self._h, name.encode(), C.byref(i)))
        d = self._desc(i.value)
        ptr = lib().b2q_gguf_tensor_data(self._h, i.value)
        if d.byte_len == 0:
            return np.empty(0, np.uint8)
        return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_uint8)), shape=(d.byte_len,))

    def get_usize(self, key: str) -> int:
        v = C.c_uint64()
        check(lib().b2q_gguf_get_usize(self._h, key.encode(), C.byref(v)))
        return int(v.value)

    def get_f32(self, key: str) -> float:
        v = C.c_float()
        check(lib().b2q_gguf_get_f32(self._h, key.encode(), C.byref(v)))
        return float(v.value)

    def get_str(self, key: str) -> str:
        p, n = C.c_void_p(), C.c_size_t()
        check(lib().b2q_gguf_get_str(self._h, key.encode(), C.byref(p), C.byref(n)))
        return C.string_at(p.value, n.value).decode("utf-8", errors="replace") if n.value else ""

    def llama_config(self, arch: str = "llama") -> dict:
        """Hyperparameters of from_gguf (inference.rs:2513-2537) as the
        dict StandardNativeEngine takes."""
        c = ModelConfig()
        check(lib().b2q_gguf_llama_config(self._h, arch.encode() if arch else None, C.byref(c)))
        return dict(n_layers=c.n_layers, n_embd=c.n_embd, n_heads=c.n_heads, n_kv_heads=c.n_kv_heads,
                    head_dim=c.head_dim, n_ff=c.n_ff, n_vocab=c.n_vocab, rms_eps=c.rms_eps,
                    rope_theta=c.rope_theta)

    def close(self) -> None:
        if self._h:
            lib().b2q_gguf_close(self._h)
            self._h = C.c_void_p(None)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
