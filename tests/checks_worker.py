"""One GPU run over every kernel family, written for the debug-bounds build
(launched by tests/test_gpu_checks.py, once with B2Q_CHECKS=1 -- the
library with the kernels' index and layout checks compiled in -- and once
with the regular library):
  * GEMVs of Q4_K / Q6_K / Q8_0 rows for 1 and 5 tokens, and the tensor-core
    matmul for 20 tokens;
  * a 2-layer model of Llama-3-8B widths: a 270-token prompt (a 256-token
    tensor-core chunk and a 14-token GEMV chunk), then greedy single-token
    steps on the persistent kernel and on the captured per-kernel graph;
  * the same model with its KV cache filled to 4096 tokens, then steps (the
    grouped long-context attention, double-buffered tiles for G = 4 off).
Saves every output to --out (npz) with the library's check status; the test
compares the two runs bit for bit and requires no failed check."""
from __future__ import annotations

import argparse
import ctypes as C
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    from conftest import load_pkg
    load_pkg()
    from hf_llm_b200 import _lib, ggml, model, synth
    from hf_llm_b200.engine import CudaEngine

    L = _lib.lib()
    eng = CudaEngine(0)
    out = {"checks_enabled": np.array(L.b2q_debug_checks_enabled())}

    for dtype in (ggml.Q4_K, ggml.Q6_K, ggml.Q8_0):
        n, k = 1024, 4096
        raw = synth.tensor_rows(dtype, n, k, 5, 31)
        buf = eng.try_upload_weight(raw, dtype, n, k)
        for m in (1, 5, 20):
            x = synth.activation(k, 40 + m, m)
            out[f"gemv_{dtype}_{m}"] = eng.matmul_batched(buf, x, m, n, k)

    cfg = dict(model.LLAMA3_8B, n_layers=2, n_vocab=32000)
    full = synth.llama_tensors(cfg, model.q4_k_m_types(), 9, dist="unit")
    rng = np.random.default_rng(4)
    prompt = rng.integers(0, cfg["n_vocab"], 270).tolist()
    for decode in ("persistent", "graph"):
        mm = model.StandardNativeEngine.from_tensors(eng, cfg, full, max_seq=4160, decode=decode)
        logits = mm.forward(prompt, 0)
        out[f"{decode}_prompt"] = logits
        pos, tok = len(prompt), int(np.argmax(logits))
        for s in range(3):
            lg = mm.forward([tok], pos)
            out[f"{decode}_step{s}"] = lg
            pos, tok = pos + 1, int(np.argmax(lg))
        mm.fill_kv(0, 4096, seed=3, scale=1.0)
        pos, tok = 4096, 7
        for s in range(2):
            lg = mm.forward([tok], pos)
            out[f"{decode}_long{s}"] = lg
            pos, tok = pos + 1, int(np.argmax(lg))
        mm.close()

    site = C.c_int(0)
    _lib.check(L.b2q_debug_check_site(eng._h, C.byref(site)))
    out["check_site"] = np.array(site.value)
    status = L.b2q_check_device_error(eng._h)
    out["device_error"] = np.array(status)
    np.savez(args.out, **out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
