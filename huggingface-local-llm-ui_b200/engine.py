"""Python mirror of the reference's GPU accelerator interface (src/gpu.rs).

``CudaEngine`` / ``CudaWeightBuffer`` keep the reference's names and argument
meaning (gpu.rs:183-735) over the C ABI of libb2q.  Differences, by design:
* failures raise ``B2QError`` instead of returning ``None`` -- there is no CPU
  fallback behind this interface;
* ``try_upload_weight`` also takes the tensor's ``[n, k]`` shape, because the
  library repacks the GGUF blocks for the GEMV at upload time (the reference
  passed the shape at every launch instead, gpu.rs:522-535).
"""
from __future__ import annotations

import ctypes as C
import threading

import numpy as np

from . import ggml
from ._lib import B2QError, check, lib

_MIB = 1024 * 1024


class CudaWeightBuffer:
    """A weight tensor resident on the device (gpu.rs:212-238)."""

    def __init__(self, engine: "CudaEngine", handle: int, byte_len: int, dtype: int, n: int, k: int):
        self.engine = engine
        self._h = C.c_void_p(handle)
        self.byte_len = byte_len
        self.dtype = dtype
        self.n = n
        self.k = k

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def free(self) -> None:
        if self._h:
            lib().b2q_weight_free(self._h)
            self.engine.offloaded_bytes -= self.byte_len
            self.engine.offloaded_tensors -= 1
            self._h = C.c_void_p(None)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class CudaEngine:
    """The device engine (gpu.rs:183-207): one per CUDA device."""

    _global: dict[int, "CudaEngine"] = {}
    _global_lock = threading.Lock()

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(lib().b2q_init(device, C.byref(h)))
        self._h = h
        self.device = device
        name = C.create_string_buffer(256)
        free, total = C.c_size_t(), C.c_size_t()
        check(lib().b2q_device_info(h, name, 256, C.byref(free), C.byref(total)))
        self.device_name = name.value.decode()
        self.total_vram = total.value
        self.offloaded_bytes = 0
        self.offloaded_tensors = 0

    @classmethod
    def global_(cls, device: int = 0) -> "CudaEngine":
        """CudaEngine::global (gpu.rs:238-241)."""
        with cls._global_lock:
            if device not in cls._global:
                cls._global[device] = CudaEngine(device)
            return cls._global[device]

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def mem_info(self) -> tuple[int, int]:
        free, total = C.c_size_t(), C.c_size_t()
        check(lib().b2q_device_info(self._h, None, 0, C.byref(free), C.byref(total)))
        return free.value, total.value

    # -- allocation policy (gpu.rs:403-464) -------------------------------
    @staticmethod
    def safe_alloc_policy(bytes_: int, free_vram: int, total_vram: int, offloaded: int) -> bool:
        """The reference's can_safely_alloc rule: never offload more than 58 %
        of VRAM, and keep max(total/5, 1600 MiB) free (gpu.rs:421-436)."""
        if bytes_ == 0:
            return True
        if offloaded + bytes_ > total_vram * 58 // 100:
            return False
        reserve = max(total_vram // 5, 1600 * _MIB)
        return free_vram > bytes_ + reserve

    def can_safely_alloc(self, bytes_: int) -> bool:
        free, total = self.mem_info()
        return self.safe_alloc_policy(bytes_, free, total, self.offloaded_bytes)

    # -- weights ----------------------------------------------------------
    def try_upload_weight(self, data, dtype: int, n: int, k: int) -> CudaWeightBuffer:
        """Upload the raw GGUF bytes of an [n, k] tensor (gpu.rs:468-507)."""
        arr = np.ascontiguousarray(np.frombuffer(memoryview(data), dtype=np.uint8)
                                   if not isinstance(data, np.ndarray) else data.view(np.uint8).reshape(-1))
        if arr.size == 0:
            raise B2QError(1, "empty weight")
        h = C.c_void_p()
        check(lib().b2q_upload_weight(self._h, arr.ctypes.data, arr.size, dtype, n, k, C.byref(h)))
        self.offloaded_bytes += arr.size
        self.offloaded_tensors += 1
        return CudaWeightBuffer(self, h.value, arr.size, dtype, n, k)

    # -- matvec entry points ----------------------------------------------
    def matmul_batched(self, buf: CudaWeightBuffer, x: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
        """y[m, n] = x[m, k] . W[n, k]^T (gpu.rs:557-589)."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(m, k)
        y = np.empty((m, n), dtype=np.float32)
        check(lib().b2q_matmul(self._h, buf.handle, x.ctypes.data_as(C.POINTER(C.c_float)),
                               y.ctypes.data_as(C.POINTER(C.c_float)), m, n, k))
        return y

    def matmul_group_same_input(self, targets, x: np.ndarray, m: int, k: int) -> list[np.ndarray]:
        """Several weights sharing one input (gpu.rs:593-650); each result is
        its own [m, n_i] array, in order."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(m, k)
        cnt = len(targets)
        ws = (C.c_void_p * cnt)(*[t[0].handle.value for t in targets])
        ns = (C.c_int * cnt)(*[int(t[1]) for t in targets])
        total = sum(int(t[1]) for t in targets)
        flat = np.empty(m * total, dtype=np.float32)
        check(lib().b2q_matmul_group(self._h, ws, ns, cnt, x.ctypes.data_as(C.POINTER(C.c_float)),
                                     m, k, flat.ctypes.data_as(C.POINTER(C.c_float))))
        out, off = [], 0
        for _, n in targets:
            out.append(flat[off:off + m * n].reshape(m, n))
            off += m * n
        return out

    def ffn_swiglu_fused(self, gate: CudaWeightBuffer, up: CudaWeightBuffer, down: CudaWeightBuffer,
                         ffn_in: np.ndarray, m: int, n_embd: int, ffn_inter: int) -> np.ndarray:
        """down . (silu(gate . x) * (up . x)) (gpu.rs:657-734)."""
        x = np.ascontiguousarray(ffn_in, dtype=np.float32).reshape(m, n_embd)
        y = np.empty((m, n_embd), dtype=np.float32)
        check(lib().b2q_ffn_swiglu(self._h, gate.handle, up.handle, down.handle,
                                   x.ctypes.data_as(C.POINTER(C.c_float)), m, n_embd, ffn_inter,
                                   y.ctypes.data_as(C.POINTER(C.c_float))))
        return y

    # -- device-pointer forms (torch tensors or raw addresses) -------------
    def sample_dev(self, logits_ptr: int, n: int, temperature: float, top_p: float, state: int,
                   stream: int = 0) -> tuple[int, int]:
        """SelfMadeSampler::sample (inference.rs:1619-1681) on device logits:
        (token, new sampler state)."""
        st = C.c_uint64(state)
        out = C.c_uint32()
        check(lib().b2q_sample_dev(self._h, logits_ptr, n, temperature, top_p, C.byref(st), C.byref(out),
                                   stream or None))
        return int(out.value), int(st.value)

    def matmul_dev(self, buf: CudaWeightBuffer, x_ptr: int, y_ptr: int, m: int, n: int, k: int,
                   stream: int = 0) -> None:
        check(lib().b2q_matmul_dev(self._h, buf.handle, x_ptr, y_ptr, m, n, k, stream or None))

    def matmul_group_dev(self, targets, x_ptr: int, y_ptr: int, m: int, k: int, stream: int = 0) -> None:
        cnt = len(targets)
        ws = (C.c_void_p * cnt)(*[t[0].handle.value for t in targets])
        ns = (C.c_int * cnt)(*[int(t[1]) for t in targets])
        check(lib().b2q_matmul_group_dev(self._h, ws, ns, cnt, x_ptr, m, k, y_ptr, stream or None))

    def ffn_swiglu_dev(self, gate, up, down, x_ptr: int, y_ptr: int, m: int, n_embd: int,
                       ffn_inter: int, stream: int = 0) -> None:
        check(lib().b2q_ffn_swiglu_dev(self._h, gate.handle, up.handle, down.handle, x_ptr, m, n_embd,
                                       ffn_inter, y_ptr, stream or None))

    def dequantize_dev(self, raw_ptr: int, dtype: int, n_elems: int, out_ptr: int, stream: int = 0) -> None:
        check(lib().b2q_dequantize_dev(self._h, raw_ptr, dtype, n_elems, out_ptr, stream or None))

    def time_gemv(self, bufs, x_ptr: int, k: int, reps: int, stream: int = 0, chained: bool = False) -> float:
        """Average device milliseconds of one GEMV launch, rotating `bufs`;
        chained: each launch a programmatic dependent launch of the last."""
        cnt = len(bufs)
        ws = (C.c_void_p * cnt)(*[b.handle.value for b in bufs])
        ms = C.c_float()
        check(lib().b2q_time_gemv(self._h, ws, cnt, x_ptr, k, reps, stream or None, C.byref(ms), int(chained)))
        return float(ms.value)

    def kernel_launches(self) -> int:
        return int(lib().b2q_kernel_launch_count(self._h))

    def check_device_error(self) -> None:
        check(lib().b2q_check_device_error(self._h))


def row_bytes(dtype: int, k: int) -> int:
    return ggml.row_bytes(dtype, k)
