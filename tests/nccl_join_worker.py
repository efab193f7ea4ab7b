"""One process, one GPU: rank 0 of a two-rank tensor-parallel model whose
rank 1 never joins (launched by tests/test_gpu_timeouts.py).  The NCCL
communicator set-up is non-blocking with a host-side timeout, so model
creation must end with B2Q_ETIMEOUT within that timeout (after
ncclCommAbort) instead of hanging, and the engine must stay usable: a GEMV
on the same device afterwards matches the fp64 oracle.  Prints one JSON
line."""
from __future__ import annotations

import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))


def main() -> int:
    from conftest import load_oracle, load_pkg
    load_pkg()
    from hf_llm_b200 import build, ggml, model, synth
    build.build()
    from hf_llm_b200._lib import B2QError, check, lib
    from hf_llm_b200.engine import CudaEngine
    orc = load_oracle()
    eng = CudaEngine(0)
    timeout_ms = int(sys.argv[1]) if len(sys.argv) > 1 else 3000
    check(lib().b2q_set_tp_init_timeout_ms(timeout_ms))
    cfg = dict(n_layers=1, n_embd=512, n_heads=8, n_kv_heads=2, head_dim=128, n_ff=512, n_vocab=512,
               rms_eps=1e-5, rope_theta=500000.0)
    uid = model.tp_unique_id()
    status, msg = 0, ""
    t0 = time.time()
    try:
        m = model.StandardNativeEngine(eng, cfg, max_seq=16, tp_rank=0, tp_size=2, tp_id=uid)
        m.close()
    except B2QError as e:
        status, msg = e.status, str(e)
    waited = time.time() - t0
    # the device is still usable
    n, k = 512, 4096
    raw = synth.tensor_rows(ggml.Q4_K, n, k, 3, 3)
    x = synth.activation(k, 4)
    y = eng.matmul_batched(eng.try_upload_weight(raw, ggml.Q4_K, n, k), x, 1, n, k)
    y64 = orc.matmul_f64(raw, ggml.Q4_K, n, k, x)
    err = float(np.linalg.norm(y - y64) / np.linalg.norm(y64))
    print(json.dumps({"status": status, "message": msg, "waited_s": waited, "gemv_rel_l2_after": err}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
