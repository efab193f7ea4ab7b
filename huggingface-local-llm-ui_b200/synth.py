"""Seeded synthetic GGUF tensors with the benchmark value distributions.

No checkpoints or datasets are available offline, so every weight is drawn
from a seeded generator with the distributions the decode benchmarks are
quoted on:

* Q8_0: f16 ``d = |N(0,1)| * 0.02 / 127``, 32 int8 codes uniform in [-127, 127].
* Q4_K: f16 ``d`` and ``dmin = |N(0,1)| * 1e-3``, sixteen 6-bit scale/min codes
  uniform in 0..63 packed into the 12-byte K-quant scale field, 128 bytes of
  uniform 4-bit codes.
* Q6_K: 128 bytes of ``ql`` and 64 bytes of ``qh`` uniform random bits, 16 int8
  sub-scales uniform in [-64, 63], f16 ``d = |N(0,1)| * 1e-3``.
* Q5_K / Q4_0: the same recipe extended to their extra bit planes.
* norms: f32 ``N(1, 0.02)``.

These "bench" distributions give strongly biased weights (Q4_K codes are all
non-negative and the mins small: mean weight ~ +0.17; Q6_K weights have std
~0.66), so a random-init decoder built from them is numerically chaotic:
activations grow layer by layer and attention saturates, and even rounding
the KV cache to f16 moves fp64 logits by percents.  Logits tolerance checks
therefore use the "unit" variant of the same block formats: zero-mean codes
(Q4_K mins matched to the sub-block scales) and block scales sized so that a
matvec of width k preserves the activation variance.

Generation is split into row chunks seeded by ``(seed, tensor_id, chunk)``,
so a tensor-parallel rank can generate only its own row range and obtain
exactly the bytes the full tensor would hold there.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import ggml

ROW_CHUNK = 1024  # rows per independently seeded chunk


def _rand_bytes(rng: np.random.Generator, n: int) -> np.ndarray:
    """n uniform random bytes (Generator.bytes is ~20x slower)."""
    words = rng.integers(0, np.iinfo(np.uint64).max, size=(n + 7) // 8, dtype=np.uint64,
                         endpoint=True)
    return words.view(np.uint8)[:n]


def _f16_bits(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint16)


def pack_q4k_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Pack eight 6-bit scales and eight 6-bit mins per block into 12 bytes.

    Inverse of decode_q4k_scales (inference.rs:988-1000): bytes 0..3 hold
    scales 0..3 in their low six bits and the top two bits of scales 4..7;
    bytes 4..7 the same for the mins; bytes 8..11 hold the low nibbles of
    scale j and min j (j = 4..7) as (sc & 15) | (min & 15) << 4.
    """
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.empty(sc.shape[:-1] + (12,), dtype=np.uint8)
    out[..., 0:4] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = mn[..., 0:4] | ((mn[..., 4:8] >> 4) << 6)
    out[..., 8:12] = (sc[..., 4:8] & 0x0F) | ((mn[..., 4:8] & 0x0F) << 4)
    return out


def _blocks_unit(rng: np.random.Generator, dtype: int, nblk: int, k: int) -> np.ndarray:
    """Zero-mean blocks whose dequantised weights have std ~ 1/sqrt(k)."""
    ts = ggml.type_size(dtype)
    out = np.empty((nblk, ts), dtype=np.uint8)
    sig = np.float32(1.0 / np.sqrt(k))
    if dtype == ggml.Q8_0:
        d = np.abs(rng.standard_normal(nblk, dtype=np.float32)) * np.float32(1.25) * sig / np.float32(73.3)
        out[:, 0:2] = _f16_bits(d).reshape(nblk, 1).view(np.uint8)
        out[:, 2:34] = rng.integers(-127, 128, size=(nblk, 32), dtype=np.int8).view(np.uint8)
    elif dtype in (ggml.Q4_K, ggml.Q5_K):
        levels = 16 if dtype == ggml.Q4_K else 32
        half = (levels - 1) / 2.0
        d = np.abs(rng.standard_normal(nblk, dtype=np.float32)) * np.float32(1.25) * sig / np.float32(
            4.6 * 4.8 * (levels / 16))
        sc = rng.integers(1, 9 if levels == 16 else 5, size=(nblk, 8), dtype=np.uint8)
        mn = np.minimum(np.rint(sc * half), 63).astype(np.uint8)
        dd = np.stack([d, d], axis=1)
        out[:, 0:4] = _f16_bits(dd).view(np.uint8).reshape(nblk, 4)
        out[:, 4:16] = pack_q4k_scales(sc, mn)
        nq = ts - 16
        out[:, 16:] = _rand_bytes(rng, nblk * nq).reshape(nblk, nq)
    elif dtype == ggml.Q6_K:
        out[:, 0:192] = _rand_bytes(rng, nblk * 192).reshape(nblk, 192)
        out[:, 192:208] = rng.integers(-64, 64, size=(nblk, 16), dtype=np.int8).view(np.uint8)
        d = np.abs(rng.standard_normal(nblk, dtype=np.float32)) * np.float32(1.25) * sig / np.float32(
            37.0 * 18.5)
        out[:, 208:210] = _f16_bits(d).reshape(nblk, 1).view(np.uint8)
    elif dtype == ggml.Q4_0:
        # codes uniform 0..15 with offset -8: std of (q - 8) ~ 4.6
        d = np.abs(rng.standard_normal(nblk, dtype=np.float32)) * np.float32(1.25) * sig / np.float32(4.6)
        out[:, 0:2] = _f16_bits(d).reshape(nblk, 1).view(np.uint8)
        out[:, 2:18] = _rand_bytes(rng, nblk * 16).reshape(nblk, 16)
    else:
        return _blocks(rng, dtype, nblk)
    return out


def _blocks(rng: np.random.Generator, dtype: int, nblk: int) -> np.ndarray:
    """`nblk` blocks of `dtype` as a [nblk, type_size] uint8 array."""
    ts = ggml.type_size(dtype)
    out = np.empty((nblk, ts), dtype=np.uint8)
    if dtype == ggml.Q8_0:
        d = np.abs(rng.standard_normal(nblk, dtype=np.float32)) * np.float32(0.02 / 127.0)
        out[:, 0:2] = _f16_bits(d).reshape(nblk, 1).view(np.uint8)
        out[:, 2:34] = rng.integers(-127, 128, size=(nblk, 32), dtype=np.int8).view(np.uint8)
    elif dtype in (ggml.Q4_K, ggml.Q5_K):
        dd = np.abs(rng.standard_normal((nblk, 2), dtype=np.float32)) * np.float32(1e-3)
        out[:, 0:4] = _f16_bits(dd).view(np.uint8).reshape(nblk, 4)
        codes = rng.integers(0, 64, size=(nblk, 16), dtype=np.uint8)
        out[:, 4:16] = pack_q4k_scales(codes[:, 0:8], codes[:, 8:16])
        nq = ts - 16
        out[:, 16:] = _rand_bytes(rng, nblk * nq).reshape(nblk, nq)
    elif dtype == ggml.Q6_K:
        out[:, 0:192] = _rand_bytes(rng, nblk * 192).reshape(nblk, 192)
        out[:, 192:208] = rng.integers(-64, 64, size=(nblk, 16), dtype=np.int8).view(np.uint8)
        d = np.abs(rng.standard_normal(nblk, dtype=np.float32)) * np.float32(1e-3)
        out[:, 208:210] = _f16_bits(d).reshape(nblk, 1).view(np.uint8)
    elif dtype == ggml.Q4_0:
        d = np.abs(rng.standard_normal(nblk, dtype=np.float32)) * np.float32(0.02 / 8.0)
        out[:, 0:2] = _f16_bits(d).reshape(nblk, 1).view(np.uint8)
        out[:, 2:18] = _rand_bytes(rng, nblk * 16).reshape(nblk, 16)
    elif dtype == ggml.F16:
        v = rng.standard_normal(nblk, dtype=np.float32) * np.float32(0.02)
        out[:] = _f16_bits(v).view(np.uint8).reshape(nblk, 2)
    elif dtype == ggml.F32:
        v = rng.standard_normal(nblk, dtype=np.float32) * np.float32(0.02)
        out[:] = v.view(np.uint8).reshape(nblk, 4)
    else:
        raise ValueError(f"no synthetic recipe for {ggml.NAMES.get(dtype, dtype)}")
    return out


def tensor_rows(dtype: int, n: int, k: int, seed: int, tensor_id: int,
                row_begin: int = 0, row_end: int | None = None, dist: str = "bench") -> np.ndarray:
    """Rows [row_begin, row_end) of a seeded [n, k] GGUF tensor, as a
    [rows, row_bytes] uint8 array in the raw GGUF block layout.
    `dist`: "bench" (the benchmark distributions) or "unit"."""
    if dist not in ("bench", "unit"):
        raise ValueError(f"unknown distribution {dist!r}")
    row_end = n if row_end is None else row_end
    if not (0 <= row_begin <= row_end <= n):
        raise ValueError("row range out of bounds")
    rb = ggml.row_bytes(dtype, k)
    bpr = k // ggml.block_size(dtype)
    out = np.empty((row_end - row_begin, rb), dtype=np.uint8)
    c0, c1 = row_begin // ROW_CHUNK, (row_end + ROW_CHUNK - 1) // ROW_CHUNK

    def fill(c: int) -> None:
        lo, hi = c * ROW_CHUNK, min(n, (c + 1) * ROW_CHUNK)
        rng = np.random.default_rng([seed, tensor_id, c])
        nblk = (hi - lo) * bpr
        blk = (_blocks(rng, dtype, nblk) if dist == "bench" else
               _blocks_unit(rng, dtype, nblk, k)).reshape(hi - lo, rb)
        a, b = max(lo, row_begin), min(hi, row_end)
        out[a - row_begin:b - row_begin] = blk[a - lo:b - lo]

    if c1 - c0 <= 1:
        for c in range(c0, c1):
            fill(c)
    else:
        with ThreadPoolExecutor(min(c1 - c0, os.cpu_count() or 1)) as ex:
            list(ex.map(fill, range(c0, c1)))
    return out


def norm_weight(n: int, seed: int, tensor_id: int) -> np.ndarray:
    """f32 N(1, 0.02) RMSNorm weight."""
    rng = np.random.default_rng([seed, tensor_id, 0x4E4F524D])
    return (1.0 + 0.02 * rng.standard_normal(n)).astype(np.float32)


def activation(k: int, seed: int, m: int = 1) -> np.ndarray:
    """f32 N(0,1) input vectors, [m, k]."""
    rng = np.random.default_rng([seed, 0x58])
    return rng.standard_normal((m, k), dtype=np.float32)


def llama_specs(cfg: dict, types: dict) -> list:
    """(GGUF name, ggml type, dims [outer.., inner], tensor id) of a Llama
    decoder with the names from_gguf reads (inference.rs:2551-2587)."""
    E, F, V = cfg["n_embd"], cfg["n_ff"], cfg["n_vocab"]
    hd, H, KV = cfg["head_dim"], cfg["n_heads"], cfg["n_kv_heads"]
    specs = [("token_embd.weight", types["token_embd"], [V, E]),
             ("output_norm.weight", ggml.F32, [E]),
             ("output.weight", types["output"], [V, E])]
    for i in range(cfg["n_layers"]):
        p = f"blk.{i}"
        specs += [(f"{p}.attn_norm.weight", ggml.F32, [E]),
                  (f"{p}.attn_q.weight", types["attn_q"], [H * hd, E]),
                  (f"{p}.attn_k.weight", types["attn_k"], [KV * hd, E]),
                  (f"{p}.attn_v.weight", types["attn_v"], [KV * hd, E]),
                  (f"{p}.attn_output.weight", types["attn_output"], [E, H * hd]),
                  (f"{p}.ffn_norm.weight", ggml.F32, [E]),
                  (f"{p}.ffn_gate.weight", types["ffn_gate"], [F, E]),
                  (f"{p}.ffn_up.weight", types["ffn_up"], [F, E]),
                  (f"{p}.ffn_down.weight", types["ffn_down"], [E, F])]
    return [(name, t, dims, tid) for tid, (name, t, dims) in enumerate(specs)]


def llama_tensor(spec, seed: int, row_begin: int = 0, row_end: int | None = None,
                 dist: str = "bench") -> np.ndarray:
    """Data of one spec entry: f32 norms as float32 [E]; quantised weights as
    raw GGUF rows [rows, row_bytes] uint8 (rows [row_begin, row_end))."""
    name, t, dims, tid = spec
    if t == ggml.F32 and len(dims) == 1:
        return norm_weight(dims[0], seed, tid)
    if name == "token_embd.weight" and dist == "unit":
        # embedding rows are the residual stream itself: unit scale, not 1/sqrt(k)
        return _embedding_unit(t, dims, seed, tid, row_begin, row_end)
    return tensor_rows(t, dims[0], dims[-1], seed, tid, row_begin, row_end, dist=dist)


def _embedding_unit(t, dims, seed, tid, row_begin, row_end):
    # rows generated as a width-1 matvec would be: std ~ 1 per element
    n, k = dims[0], dims[-1]
    rb = ggml.row_bytes(t, k)
    bpr = k // ggml.block_size(t)
    row_end = n if row_end is None else row_end
    out = np.empty((row_end - row_begin, rb), dtype=np.uint8)
    for c in range(row_begin // ROW_CHUNK, (row_end + ROW_CHUNK - 1) // ROW_CHUNK):
        lo, hi = c * ROW_CHUNK, min(n, (c + 1) * ROW_CHUNK)
        rng = np.random.default_rng([seed, tid, c])
        blk = _blocks_unit(rng, t, (hi - lo) * bpr, 1).reshape(hi - lo, rb)
        a, b = max(lo, row_begin), min(hi, row_end)
        out[a - row_begin:b - row_begin] = blk[a - lo:b - lo]
    return out


def llama_tensors(cfg: dict, types: dict, seed: int, dist: str = "bench") -> dict:
    """All tensors of a synthetic Llama: name -> (type, dims, array)."""
    return {s[0]: (s[1], s[2], llama_tensor(s, seed, dist=dist)) for s in llama_specs(cfg, types)}
