"""Python mirror of the reference's Llama engine (src/inference.rs:2406-2905).

``StandardNativeEngine`` keeps the reference's entry points -- construction
from GGUF-named tensors, ``forward(tokens, start_pos)`` returning the logits
of the last position, ``clear_state()`` -- over the C ABI of libb2q, which
keeps the weights, activations and the f16 KV cache on the device.
``generate_greedy`` is the decode loop of LocalLlm at temperature 0
(inference.rs:3190-3231 prefill, :3354 decode, :1620-1630 greedy sampling).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import ggml
from ._lib import ModelConfig, check, lib
from .engine import CudaEngine

LLAMA3_8B = dict(n_layers=32, n_embd=4096, n_heads=32, n_kv_heads=8, head_dim=128, n_ff=14336,
                 n_vocab=128256, rms_eps=1e-5, rope_theta=500000.0)
LLAMA3_70B = dict(n_layers=80, n_embd=8192, n_heads=64, n_kv_heads=8, head_dim=128, n_ff=28672,
                  n_vocab=128256, rms_eps=1e-5, rope_theta=500000.0)


def tp_shard_rows(cfg: dict, name: str, n: int, tp_rank: int, tp_size: int) -> tuple[int, int]:
    """Rows [begin, end) of tensor `name` ([n][...]) owned by `tp_rank` of
    `tp_size` (b2q_tp_shard_rows; no device needed)."""
    c = ModelConfig(cfg["n_layers"], cfg["n_embd"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                    cfg["n_ff"], cfg["n_vocab"], cfg["rms_eps"], cfg["rope_theta"], 8, tp_rank, tp_size, 0)
    b, e = C.c_int64(), C.c_int64()
    check(lib().b2q_tp_shard_rows(C.byref(c), name.encode(), n, C.byref(b), C.byref(e)))
    return b.value, e.value


def tp_shard_cols(cfg: dict, name: str, k: int, tp_rank: int, tp_size: int) -> tuple[int, int]:
    """Columns [begin, end) of tensor `name` ([...][k]) kept by `tp_rank` of
    `tp_size` (b2q_tp_shard_cols; no device needed)."""
    c = ModelConfig(cfg["n_layers"], cfg["n_embd"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                    cfg["n_ff"], cfg["n_vocab"], cfg["rms_eps"], cfg["rope_theta"], 8, tp_rank, tp_size, 0)
    b, e = C.c_int64(), C.c_int64()
    check(lib().b2q_tp_shard_cols(C.byref(c), name.encode(), k, C.byref(b), C.byref(e)))
    return b.value, e.value


def tp_unique_id() -> bytes:
    buf = (C.c_ubyte * 128)()
    check(lib().b2q_tp_unique_id(buf))
    return bytes(buf)


class StandardNativeEngine:
    """Llama-family decoder on one device, or one tensor-parallel rank."""

    # single-token step modes (b2q_model_config.no_graph)
    DECODE_MODES = {"persistent": 0, "eager": 1, "graph": 2}

    def __init__(self, engine: CudaEngine, cfg: dict, max_seq: int = 8192, tp_rank: int = 0,
                 tp_size: int = 1, tp_id: bytes | None = None, use_graph: bool = True,
                 decode: str | None = None):
        """`decode` picks how single-token steps run: "persistent" (default:
        one persistent kernel per token, on one GPU or across the
        tensor-parallel ranks; the captured graph where the model does not
        fit it), "graph" (the captured graph of the per-layer kernels) or
        "eager" (the same kernels launched one by one; also use_graph=False).
        All three give the same logits bit for bit."""
        self.engine = engine
        self.cfg = dict(cfg)
        self.max_seq = max_seq
        mode = decode or ("persistent" if use_graph else "eager")
        if mode not in self.DECODE_MODES:
            raise ValueError(f"decode must be one of {sorted(self.DECODE_MODES)}")
        self.decode_mode = mode
        c = ModelConfig(cfg["n_layers"], cfg["n_embd"], cfg["n_heads"], cfg["n_kv_heads"],
                        cfg["head_dim"], cfg["n_ff"], cfg["n_vocab"], cfg["rms_eps"],
                        cfg["rope_theta"], max_seq, tp_rank, tp_size, self.DECODE_MODES[mode])
        h = C.c_void_p()
        idbuf = (C.c_ubyte * 128).from_buffer_copy(tp_id) if tp_id else None
        check(lib().b2q_model_create(engine.handle, C.byref(c), idbuf, C.byref(h)))
        self._h = h
        self._logits_ptr = None  # (address, ctypes pointer) of forward_into's last logits buffer
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.current_pos = 0

    # -- loading (from_gguf, inference.rs:2513-2620) -----------------------
    def shard_rows(self, name: str, n: int) -> tuple[int, int]:
        b, e = C.c_int64(), C.c_int64()
        check(lib().b2q_model_shard_rows(self._h, name.encode(), n, C.byref(b), C.byref(e)))
        return b.value, e.value

    def set_tensor(self, name: str, dtype: int, dims, data: np.ndarray, row_begin: int | None = None,
                   row_end: int | None = None) -> None:
        arr = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        d = (C.c_int64 * len(dims))(*[int(v) for v in dims])
        if row_begin is None:
            check(lib().b2q_model_set_tensor(self._h, name.encode(), dtype, d, len(dims),
                                             arr.ctypes.data, arr.size))
        else:
            check(lib().b2q_model_set_tensor_rows(self._h, name.encode(), dtype, d, len(dims),
                                                  row_begin, row_end, arr.ctypes.data, arr.size))

    def finalize(self) -> None:
        check(lib().b2q_model_finalize(self._h))

    @classmethod
    def from_tensors(cls, engine: CudaEngine, cfg: dict, tensors: dict, max_seq: int = 8192,
                     **tp) -> "StandardNativeEngine":
        """`tensors`: GGUF name -> (ggml type, dims [outer.., inner], array)."""
        m = cls(engine, cfg, max_seq=max_seq, **tp)
        for name, (dtype, dims, arr) in tensors.items():
            m.set_tensor(name, dtype, dims, arr)
        m.finalize()
        return m

    @classmethod
    def from_gguf(cls, engine: CudaEngine, gguf, arch: str = "llama", max_seq: int = 8192,
                  **kw) -> "StandardNativeEngine":
        """StandardNativeEngine::from_gguf (inference.rs:2513-2620): the
        hyperparameters and every tensor from a GGUF file (a path or an open
        GgufFile); under tensor parallelism each rank uploads its own rows."""
        from .gguf_file import GgufFile
        f = gguf if isinstance(gguf, GgufFile) else GgufFile(gguf)
        try:
            m = cls(engine, f.llama_config(arch), max_seq=max_seq, **kw)
            check(lib().b2q_model_load_gguf(m._h, f.handle))
            m.finalize()
        finally:
            if f is not gguf:
                f.close()
        return m

    @property
    def weight_bytes(self) -> int:
        return int(lib().b2q_model_weight_bytes(self._h))

    @property
    def step_path(self) -> str:
        """How single-token steps run: "persistent", "eager" or "graph"."""
        return {0: "persistent", 1: "eager", 2: "graph"}.get(int(lib().b2q_model_step_path(self._h)), "none")

    # -- inference --------------------------------------------------------
    def forward(self, tokens, start_pos: int) -> np.ndarray:
        """Logits [n_vocab] of the last position (inference.rs:2695-2860)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        logits = np.empty(self.cfg["n_vocab"], dtype=np.float32)
        check(lib().b2q_forward(self._h, t.ctypes.data_as(C.POINTER(C.c_uint32)), t.size, start_pos,
                                logits.ctypes.data_as(C.POINTER(C.c_float)), None))
        return logits

    def forward_into(self, tokens, start_pos: int, logits: np.ndarray) -> int:
        """forward with the logits written into the caller's float32 array
        (page-locked host memory makes the copy a direct DMA) and the greedy
        next token (the library's device argmax, first index of the maximum)
        returned."""
        if logits.dtype != np.float32 or logits.size < self.cfg["n_vocab"] or not logits.flags.c_contiguous:
            raise ValueError("logits must be a contiguous float32 array of n_vocab elements")
        # a decode loop calls this once per token: one id goes in a ctypes
        # array, and the logits pointer is converted once per buffer address
        if type(tokens) is list and len(tokens) == 1 and type(tokens[0]) is int and 0 <= tokens[0] < 1 << 32:
            tp, nt = (C.c_uint32 * 1)(tokens[0]), 1
        else:
            t = np.ascontiguousarray(tokens, dtype=np.uint32)
            tp, nt = t.ctypes.data_as(C.POINTER(C.c_uint32)), t.size
        addr = logits.ctypes.data
        lp = self._logits_ptr
        if lp is None or lp[0] != addr:
            lp = self._logits_ptr = (addr, C.cast(addr, C.POINTER(C.c_float)))
        out = C.c_uint32()
        check(lib().b2q_forward(self._h, tp, nt, start_pos, lp[1], C.byref(out)))
        return int(out.value)

    def forward_argmax(self, tokens, start_pos: int) -> int:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = C.c_uint32()
        check(lib().b2q_forward(self._h, t.ctypes.data_as(C.POINTER(C.c_uint32)), t.size, start_pos,
                                None, C.byref(out)))
        return int(out.value)

    def forward_dev(self, tokens_ptr: int, n: int, start_pos: int, logits_ptr: int = 0,
                    argmax_ptr: int = 0, stream: int = 0) -> None:
        check(lib().b2q_forward_dev(self._h, tokens_ptr, n, start_pos, logits_ptr or None,
                                    argmax_ptr or None, stream or None))

    def forward_sample(self, tokens, start_pos: int, temperature: float, top_p: float, state: int) -> tuple[int, int]:
        """forward, then SelfMadeSampler::sample (inference.rs:1619-1681) on
        the device: (next token, new sampler state)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        st = C.c_uint64(state)
        out = C.c_uint32()
        check(lib().b2q_forward_sample(self._h, t.ctypes.data_as(C.POINTER(C.c_uint32)), t.size, start_pos,
                                       temperature, top_p, C.byref(st), C.byref(out)))
        return int(out.value), int(st.value)

    def generate(self, prompt, max_tokens: int, temperature: float = 0.7, top_p: float = 0.9,
                 seed: int = 0) -> list[int]:
        """Prompt pass, then `max_tokens` sampled tokens (LocalLlm's generate
        loop over forward + SelfMadeSampler).  temperature <= 1e-5 is greedy."""
        prompt = list(prompt)
        if not prompt:
            raise ValueError("no tokens to prefill")
        state = int(lib().b2q_sampler_state(seed))
        nxt = None
        for off in range(0, len(prompt), 256):
            chunk = prompt[off:off + 256]
            nxt, state = self.forward_sample(chunk, self.current_pos, temperature, top_p, state)
            self.current_pos += len(chunk)
        out = []
        for _ in range(max_tokens):
            out.append(nxt)
            nxt, state = self.forward_sample([nxt], self.current_pos, temperature, top_p, state)
            self.current_pos += 1
        return out

    def fill_kv(self, start: int, n: int, seed: int = 0, scale: float = 1.0) -> None:
        """Seeded synthetic K/V rows for positions [start, start + n) of every
        layer (benchmark set-up for a long context; b2q_model_fill_kv)."""
        check(lib().b2q_model_fill_kv(self._h, start, n, seed, scale))

    def clear_state(self) -> None:
        check(lib().b2q_clear_state(self._h))
        self.current_pos = 0

    def generate_greedy(self, prompt, max_tokens: int, prefill_chunk: int = 256) -> list[int]:
        """Chunked prefill, then greedy decode of `max_tokens` tokens."""
        prompt = list(prompt)
        if not prompt:
            raise ValueError("no tokens to prefill")
        nxt = None
        for off in range(0, len(prompt), prefill_chunk):
            chunk = prompt[off:off + prefill_chunk]
            nxt = self.forward_argmax(chunk, self.current_pos)
            self.current_pos += len(chunk)
        out = []
        for _ in range(max_tokens):
            out.append(nxt)
            nxt = self.forward_argmax([nxt], self.current_pos)
            self.current_pos += 1
        return out

    def close(self) -> None:
        if self._h:
            lib().b2q_model_destroy(self._h)
            self._h = C.c_void_p(None)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def q4_k_m_types() -> dict:
    """GGML types per tensor role of the Llama Q4_K_M layout used here."""
    return {"token_embd": ggml.Q4_K, "output": ggml.Q6_K, "attn_q": ggml.Q4_K, "attn_k": ggml.Q4_K,
            "attn_v": ggml.Q6_K, "attn_output": ggml.Q4_K, "ffn_gate": ggml.Q4_K,
            "ffn_up": ggml.Q4_K, "ffn_down": ggml.Q6_K}
