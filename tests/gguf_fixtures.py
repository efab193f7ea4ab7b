"""GGUF files for the loader tests.

Two independent writers:
  * `write_ggufpy` -- gguf-py's GGUFWriter (llama.cpp's Python implementation
    of the format), the outside pin for the parser;
  * `write_raw` -- a minimal byte-level writer of our own, for what gguf-py
    cannot produce: version 1/2 containers, duplicate keys or tensor names,
    hand-corrupted files.
Tensors are given as (name, ggml type, dims [outer.., inner], raw bytes).
"""
from __future__ import annotations

import struct

import numpy as np

# GGUF metadata value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?",
           U64: "<Q", I64: "<q", F64: "<d"}


def _len(version: int, n: int) -> bytes:
    return struct.pack("<I" if version == 1 else "<Q", n)


def _str(version: int, s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return _len(version, len(b)) + b


def _value(version: int, vtype: int, v, sub=None) -> bytes:
    if vtype in _SCALAR:
        return struct.pack(_SCALAR[vtype], v)
    if vtype == STRING:
        return _str(version, v)
    if vtype == ARRAY:
        et, items = sub, v
        out = struct.pack("<I", et) + _len(version, len(items))
        for it in items:
            if et == ARRAY:
                out += _value(version, ARRAY, it[1], it[0])
            else:
                out += _value(version, et, it)
        return out
    raise ValueError(vtype)


def raw_bytes(version: int, kvs, tensors, alignment: int = 32):
    """The bytes of a GGUF file.  kvs: (key, vtype, value[, sub_type]);
    tensors: (name, ggml type, dims [outer.., inner], data bytes, [rel offset])."""
    head = b"GGUF" + struct.pack("<I", version) + _len(version, len(tensors)) + _len(version, len(kvs))
    for kv in kvs:
        key, vt, v = kv[0], kv[1], kv[2]
        head += _str(version, key) + struct.pack("<I", vt) + _value(version, vt, v, kv[3] if len(kv) > 3 else None)
    rel, offs = 0, []
    for t in tensors:
        if len(t) > 4:
            offs.append(t[4])
            continue
        offs.append(rel)
        rel += len(t[3])
        rel = (rel + alignment - 1) // alignment * alignment
    for t, off in zip(tensors, offs):
        name, gt, dims = t[0], t[1], t[2]
        head += _str(version, name) + struct.pack("<I", len(dims))
        for d in reversed(dims):
            head += _len(version, d)
        head += struct.pack("<I", gt) + struct.pack("<Q", off)
    pad = (alignment - len(head) % alignment) % alignment
    data_off = len(head) + pad
    body = bytearray(max([o + len(t[3]) for t, o in zip(tensors, offs)], default=0))
    for t, off in zip(tensors, offs):
        body[off:off + len(t[3])] = t[3]
    return bytes(head) + b"\0" * pad + bytes(body), data_off


def write_raw(path, version: int, kvs, tensors, alignment: int = 32):
    data, off = raw_bytes(version, kvs, tensors, alignment)
    with open(path, "wb") as f:
        f.write(data)
    return off


def write_ggufpy(path, arch: str, kvs, tensors, alignment: int | None = None):
    """kvs: (key, gguf-py method name, value); tensors as above."""
    import gguf
    w = gguf.GGUFWriter(str(path), arch)
    if alignment is not None:
        w.add_custom_alignment(alignment)
    for key, meth, v in kvs:
        getattr(w, meth)(key, v)
    for name, gt, dims, data in tensors:
        arr = np.frombuffer(bytes(data), dtype=np.uint8)
        if gt == 0:
            w.add_tensor(name, arr.view(np.float32).reshape(dims))
        elif gt == 1:
            w.add_tensor(name, arr.view(np.float16).reshape(dims))
        else:
            w.add_tensor(name, arr.reshape(dims[0], -1) if len(dims) > 1 else arr,
                         raw_dtype=gguf.GGMLQuantizationType(gt))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def llama_kvs(cfg: dict, arch: str = "llama") -> list:
    return [(f"{arch}.block_count", "add_uint32", cfg["n_layers"]),
            (f"{arch}.embedding_length", "add_uint32", cfg["n_embd"]),
            (f"{arch}.attention.head_count", "add_uint32", cfg["n_heads"]),
            (f"{arch}.attention.head_count_kv", "add_uint32", cfg["n_kv_heads"]),
            (f"{arch}.attention.key_length", "add_uint32", cfg["head_dim"]),
            (f"{arch}.feed_forward_length", "add_uint32", cfg["n_ff"]),
            (f"{arch}.attention.layer_norm_rms_epsilon", "add_float32", cfg["rms_eps"]),
            (f"{arch}.rope.freq_base", "add_float32", cfg["rope_theta"])]


def llama_tensor_list(tensors: dict, drop=(), f16_norms: bool = False) -> list:
    """synth.llama_tensors output -> writer tensor list (optionally without
    some names, or with the 1-D norms stored as F16)."""
    out = []
    for name, (t, dims, arr) in tensors.items():
        if name in drop:
            continue
        a = np.ascontiguousarray(arr)
        if f16_norms and t == 0 and len(dims) == 1:
            out.append((name, 1, list(dims), a.astype(np.float16).tobytes()))
        else:
            out.append((name, t, list(dims), a.tobytes()))
    return out
