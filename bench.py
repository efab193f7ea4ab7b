"""Decode benchmark: Llama-3-8B-shaped Q4_K_M decoder at batch 1 (the headline),
plus the Llama-3-70B-shaped decoder at an 8192-token context.

Workload (the metric "decode tok/s at Llama-3-8B Q4_K_M shape; dequant-GEMV
HBM GB/s vs 8 TB/s"): a random-init 32-layer Llama-3-8B-shaped decoder
(hidden 4096, 32/8 heads, head_dim 128, FFN 14336, vocab 128256; attn_q/k/
output and ffn_gate/up Q4_K, attn_v / ffn_down / output Q6_K, token_embd
Q4_K, f32 norms, f16 KV cache), weights drawn from the seeded benchmark
distributions (synthetic: no checkpoints offline).  A 512-token random-id
prompt is prefilled, then one step = one greedy decode token at batch 1.

* value    -- decode tok/s with everything resident in HBM: one step is one
              launch of the persistent decode kernel (the whole single-token
              forward); the next token id is the argmax that kernel writes on
              the device (no host round trip).  CUDA events on the launching
              stream, max over ranks.  After the host barrier and sync that
              open the timed region, one untimed step runs first: its
              all-rank barriers line the ranks' streams up on the device, so
              host start skew stays out of every rank's events.  4.9 GB of
              weights are read per step, far above L2 (126 MB).
* e2e      -- the same through the host API b2q_forward: the token id copied
              in from host memory and the logits [128256] f32 copied back into
              a page-locked array every step, with the greedy next token that
              b2q_forward returns beside them; host wall clock, max over ranks.
* roofline -- the dominant kernel, decode_kernel (the only kernel of a step):
              algorithmic bytes of one step on this rank (the weight rows or
              columns it owns, one token_embd row, the norms and the f16 K/V
              rows of its KV heads at the mean timed context) / event time
              per step; `traffic` from the committed ncu capture.
* gemv_roofline / gemv_shapes -- the standalone GEMV per matvec config shape
              (rank 0), weights rotated over copies larger than L2.
* output_head -- the Q6_K output head (128256 x 4096) row-sharded over the N
              ranks: the GEMV of one rank's rows, max over ranks.
* prefill  -- the 512-token prompt pass (tensor cores), its projection flops
              against the measured bf16 peak.
* tp_parity -- after the timed region, a fixed-seed 2-layer model of
              Llama-3-8B widths (unit distribution) runs a 20-token prompt and
              three single-token steps through the same path on the same
              ranks; rank 0 compares the logits with the fp64 oracle
              (rel-L2 <= 1e-3).
* cpu_baseline -- the reference's CPU path (the oracle's restatement of the
              AVX2/FMA Rayon matvec and the Llama forward), rank 0 at N = 1:
              all host cores, and the reference governor's thread count
              min(3/4 cores, cores - 2) (hardware.rs:157-166); `matvec_shapes`:
              the same CPU matvec per gemv_shapes config shape, weight copies
              rotated past 256 MB.
* model_70b -- the Llama-3-70B-shaped decoder (80 layers, hidden 8192, 64/8
              heads, FFN 28672, same quant mix, 44 GB): the f16 KV cache is
              filled with seeded synthetic rows (b2q_model_fill_kv) up to the
              8192-token context, then the same value / e2e / roofline.  Host
              generation shortcut: one seeded layer's bytes are uploaded into
              each of the 80 layers' own device buffers, so every step still
              reads 44 GB of distinct device memory.

--gpus N > 1 (launched under torchrun): tensor-parallel decode of the same
model on N GPUs (KV heads, gate/up and the head by rows, attn_output and
ffn_down by columns, partial sums exchanged over NVLink by the persistent
kernel); the model is fixed, so scaling is strong.
--impl reference: the reference's CPU path (the oracle restatement) on the
same workload -- the same prompt ids, prefill length, warm-up and timed steps
-- on rank 0 with all host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
PKG_DIR = REPO / "huggingface-local-llm-ui_b200"

HBM_FALLBACK_GBS = 6650.0


def load_pkg():
    import importlib.util
    name = "hf_llm_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle  # noqa: E402
    oracle.build()
    return oracle


def measured_peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return HBM_FALLBACK_GBS, "fallback"


def load_peaks() -> dict:
    """MEASURED_PEAKS.json (driver-measured copy bandwidth and bf16 GEMM
    throughput on this pool's B200s), or the fallback figures."""
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {"hbm_gbs": HBM_FALLBACK_GBS, "bf16_tflops": 1590.0}


def profile_traffic(name: str = "gemv_q4k_14336x4096.md",
                    key: str = "traffic_bytes_per_launch") -> float | None:
    """DRAM bytes per launch from a committed ncu summary under profiles/
    (its "traffic_bytes_per_launch:" line, or another `key:` line), if one
    has been captured."""
    p = REPO / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


def scaled_profile_traffic(name: str, step_bytes: int) -> float | None:
    """DRAM bytes of a full launch from a capture of a smaller case of the
    same kernel: the capture's traffic / algorithmic-bytes ratio times this
    launch's algorithmic bytes (traffic grows with the layers and keys in
    proportion; the summary under profiles/ records both figures)."""
    t = profile_traffic(name)
    a = profile_traffic(name, "algorithmic_bytes_per_launch")
    if not t or not a:
        return None
    return round(t / a * step_bytes)


def governor_threads(cores: int) -> int:
    """The reference's CPU thread count: min(3/4 cores, cores - 2), at least 1
    (ResourceGovernor, hardware.rs:157-166)."""
    return max(1, min(cores * 3 // 4, cores - 2))


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"b2q_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        try:
            for line in self.path.read_text().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx.append(float(f[2]))
                except ValueError:
                    continue
                names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
                for name, v in zip(names, f[5:9]):
                    if v.lower() == "active":
                        reasons.add(name)
        except FileNotFoundError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def model_cfg(name: str, layers: int | None = None) -> dict:
    from hf_llm_b200 import model
    base = model.LLAMA3_70B if name == "70b" else model.LLAMA3_8B
    return dict(base, n_layers=layers or base["n_layers"])


def workload_config(name: str, cfg: dict, prefill: int, context: str | None = None) -> dict:
    """The workload as both arms report it (no implementation keys)."""
    c = {"workload": f"llama3-{name}-q4_k_m-decode", "layers": cfg["n_layers"], "hidden": cfg["n_embd"],
         "heads": f"{cfg['n_heads']}/{cfg['n_kv_heads']}", "ffn": cfg["n_ff"], "vocab": cfg["n_vocab"],
         "prefill": prefill, "batch": 1,
         "l2": "inputs larger than L2: every step reads all weights (GBs) from memory"}
    if context:
        c["context"] = context
    return c


def build_model(engine, cfg, seed, rank, size, tp_id, max_seq, dist="bench", decode="persistent",
                keep_host=False, share_layers=False):
    """Upload this rank's shards of a synthetic Llama.  share_layers: every
    layer gets the bytes of layer 0's tensors (generated once; each layer
    still has its own device buffers)."""
    from hf_llm_b200 import model, synth
    m = model.StandardNativeEngine(engine, cfg, max_seq=max_seq, tp_rank=rank, tp_size=size, tp_id=tp_id,
                                   decode=decode)
    host = {}
    cache = {}
    specs = synth.llama_specs(cfg, model.q4_k_m_types())
    by_name = {s[0]: s for s in specs}
    for spec in specs:
        name, t, dims, _ = spec
        src = spec
        if share_layers and name.startswith("blk."):
            role = name.split(".", 2)[2]
            src = by_name[f"blk.0.{role}"]
        if len(dims) == 1:
            arr = synth.llama_tensor(src, seed, dist=dist)
            m.set_tensor(name, t, dims, arr)
            if keep_host:
                host[name] = (t, dims, arr)
            continue
        b, e = m.shard_rows(name, dims[0])
        key = (src[0], b, e)
        arr = cache.get(key) if share_layers else None
        if arr is None:
            arr = synth.llama_tensor(src, seed, b, e, dist=dist)
            if share_layers and src[0].startswith("blk."):
                cache[key] = arr
        m.set_tensor(name, t, dims, arr, b, e)
        if keep_host:
            host[name] = (t, dims, arr)
        del arr
    cache.clear()
    m.finalize()
    return m, host


def step_algorithmic_bytes(cfg, rank: int, world: int, ctx: int) -> int:
    """Bytes one single-token step must read on `rank`: the part of every
    matvec weight it owns (its rows, or for attn_output / ffn_down its
    columns) and of the output head, one row of token_embd, the norms, and
    the f16 K/V rows of its KV heads for `ctx` cached tokens."""
    from hf_llm_b200 import ggml, model, synth
    total = 0
    for name, t, dims, _ in synth.llama_specs(cfg, model.q4_k_m_types()):
        if len(dims) == 1:
            total += 4 * dims[0]
            continue
        n, k = dims
        if name == "token_embd.weight":
            total += ggml.row_bytes(t, k)
            continue
        b, e = model.tp_shard_rows(cfg, name, n, rank, world)
        cb, ce = model.tp_shard_cols(cfg, name, k, rank, world)
        total += (e - b) * ggml.row_bytes(t, ce - cb)
    total += cfg["n_layers"] * 2 * (cfg["n_kv_heads"] // world) * cfg["head_dim"] * 2 * ctx
    return total


def prefill_matmul_params(cfg, rank: int, world: int) -> int:
    """Weights (elements) of the per-layer projections this rank multiplies
    in a prompt pass: q, k, v, o, gate, up, down of every layer."""
    from hf_llm_b200 import model, synth
    total = 0
    for name, t, dims, _ in synth.llama_specs(cfg, model.q4_k_m_types()):
        if len(dims) == 2 and name.startswith("blk."):
            b, e = model.tp_shard_rows(cfg, name, dims[0], rank, world)
            cb, ce = model.tp_shard_cols(cfg, name, dims[1], rank, world)
            total += (e - b) * (ce - cb)
    return total


def prompt_ids(cfg, seed: int, n: int) -> np.ndarray:
    """The benchmark prompt: n random token ids (both arms use these)."""
    return np.random.default_rng(seed).integers(0, cfg["n_vocab"], n).astype(np.int32)


def cpu_decode(orc, cfg, host, prompt, phases) -> list[dict]:
    """The reference CPU path on one model at the benchmark's context: its
    f32 KV cache holds len(prompt) - 1 positions of seeded synthetic rows (the
    context the GPU arm reaches with its prompt pass; a 512-token CPU prompt
    pass takes minutes), the last prompt token is run through the forward,
    then for each (threads, warmup, steps) of `phases` untimed and timed
    greedy steps."""
    m = orc.Model(cfg, host, kv_capacity=len(prompt) + sum(w + s for _, w, s in phases) + 1)
    m.fill_kv(len(prompt) - 1, seed=len(prompt))
    orc.set_threads(phases[0][0])
    logits = m.forward_ref([int(prompt[-1])], len(prompt) - 1)
    pos = len(prompt)
    out = []
    for threads, warm, steps in phases:
        orc.set_threads(threads)
        for _ in range(warm):
            logits = m.forward_ref([int(np.argmax(logits))], pos)
            pos += 1
        t0 = time.perf_counter()
        for _ in range(steps):
            logits = m.forward_ref([int(np.argmax(logits))], pos)
            pos += 1
        dt = time.perf_counter() - t0
        out.append({"value": steps / dt, "unit": "tok/s", "cores": threads, "kind": "port", "steps": steps})
    return out


GEMV_SHAPES = {  # key: (ggml type, n, k, copies rotated to exceed L2)
    "q4k_14336x4096": (12, 14336, 4096, 24), "q4k_4096x14336": (12, 4096, 14336, 24),
    "q4k_4096x4096": (12, 4096, 4096, 48), "q4k_1024x4096": (12, 1024, 4096, 96),
    "q6k_128256x4096": (14, 128256, 4096, 2), "q6k_4096x14336": (14, 4096, 14336, 16),
    "q8_0_4096x4096": (8, 4096, 4096, 48),
    "q5k_14336x4096": (13, 14336, 4096, 20), "q4_0_4096x4096": (2, 4096, 4096, 48),
}


def time_gemv_shape(engine, synth, key, seed, dev, sp, copies=None, reps=None, chained=False):
    """Average device ms of one GEMV launch of a config shape, rotating weight
    copies larger than L2; chained: programmatic dependent launches (as the
    per-kernel decode path chains its GEMVs), else plain back-to-back ones."""
    import torch
    t, n, k, cp = GEMV_SHAPES[key]
    copies = copies or cp
    raw = synth.tensor_rows(t, n, k, seed, 900)
    bufs = [engine.try_upload_weight(raw, t, n, k) for _ in range(copies)]
    x = torch.randn(k, device=dev)
    engine.time_gemv(bufs, x.data_ptr(), k, 2, sp, chained)  # warm-up
    reps = reps or max(2, 400 // copies)
    ms_l = engine.time_gemv(bufs, x.data_ptr(), k, reps, sp, chained)
    alg = n * raw.shape[1] + 4 * k + 4 * n
    for b in bufs:
        b.free()
    return ms_l, alg


CPU_ROTATE_BYTES = 256 << 20  # weight copies rotated by the CPU matvec timing (past the host's LLC)


def cpu_matvec_shape(orc, synth, key, seed, threads: list[int], min_s: float = 0.25, max_reps: int = 64) -> dict:
    """The reference CPU matvec (matmul_batched, inference.rs:589-760: x
    quantised to Q8_K / Q8_0, then the AVX2/FMA row dots over the threads) on
    one config shape, per thread count: wall time per call, rotating weight
    copies that together exceed the host's last-level cache, so the rows come
    from DRAM as they do on the GPU side."""
    t, n, k, _ = GEMV_SHAPES[key]
    raw = synth.tensor_rows(t, n, k, seed, 900)
    copies = [raw] + [raw.copy() for _ in range(max(0, -(-CPU_ROTATE_BYTES // raw.nbytes) - 1))]
    x = np.random.default_rng(seed).standard_normal(k).astype(np.float32)
    alg = n * raw.shape[1] + 4 * k + 4 * n
    out = {"bytes": alg, "copies": len(copies)}
    for th in threads:
        orc.set_threads(th)
        orc.matmul_batched(raw, t, n, k, x)  # warm-up
        reps = 0
        t0 = time.perf_counter()
        while True:
            orc.matmul_batched(copies[reps % len(copies)], t, n, k, x)
            reps += 1
            dt = time.perf_counter() - t0
            if (dt >= min_s and reps >= len(copies)) or reps >= max_reps:
                break
        us = dt / reps * 1e6
        out[f"threads_{th}"] = {"us": round(us, 1), "GBps": round(alg / (us * 1e-6) / 1e9, 2), "reps": reps}
    return out


def time_head_shard(engine, synth, world, rank, seed, dev, sp, dist, peak, peak_kind):
    """The Q6_K output head (128256 x 4096) row-sharded over the ranks as the
    model shards it: every rank times the GEMV of its rows (chained launches,
    weight copies rotated past L2), max over ranks.  The logit slices are
    then exchanged inside the persistent kernel's epilogue (each rank stores
    its slice into every rank's logits over NVLink), not by a collective."""
    import torch
    t, n, k = 14, 128256, 4096
    rows = -(-n // world)
    rows = -(-rows // 8) * 8  # the model's V_loc: 8-row groups
    r0 = min(n, rank * rows)
    nl = max(8, min(rows, n - r0))
    raw = synth.tensor_rows(t, n, k, seed, 901, r0, r0 + nl)
    copies = max(2, -(-400_000_000 // raw.nbytes))
    bufs = [engine.try_upload_weight(raw, t, nl, k) for _ in range(copies)]
    x = torch.randn(k, device=dev)
    engine.time_gemv(bufs, x.data_ptr(), k, 2, sp, True)
    ms = engine.time_gemv(bufs, x.data_ptr(), k, max(4, 400 // copies), sp, True)
    for b in bufs:
        b.free()
    alg = raw.nbytes + 4 * k + 4 * nl
    if dist:
        tt = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    ach = alg / (ms * 1e-3) / 1e9
    return {"rows_per_rank": nl, "us": round(ms * 1000, 3), "GBps_per_rank": round(ach, 1),
            "GBps_all_ranks": round(ach * world, 1), "frac": round(ach / peak, 4), "peak_kind": peak_kind,
            "note": "Q6_K 128256x4096 row-sharded; GEMV of one rank's rows, chained launches, max over ranks; "
                    "the logit slices go to every rank by peer stores in the persistent kernel's epilogue"}


def run_gemv_only(args):
    """One GEMV shape, its weights rotated over `--copies` copies: the
    workload of the kernel profiles (ncu) under profiles/."""
    import torch
    load_pkg()
    from hf_llm_b200 import build as bld
    bld.build()
    from hf_llm_b200 import synth
    from hf_llm_b200.engine import CudaEngine
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    engine = CudaEngine(0)
    stream = torch.cuda.Stream(device=dev)
    ms_l, alg = time_gemv_shape(engine, synth, args.gemv_only, args.seed, dev, stream.cuda_stream,
                                args.copies, args.reps, chained=args.chained)
    peak, kind = measured_peaks()
    gbs = alg / (ms_l * 1e-3) / 1e9
    print(json.dumps({"gemv": args.gemv_only, "us_per_launch": round(ms_l * 1000, 3),
                      "algorithmic_bytes": alg, "GBps": round(gbs, 1), "frac": round(gbs / peak, 4),
                      "peak": peak, "peak_kind": kind, "copies": args.copies, "reps": args.reps}))
    return 0


def run_reference_arm(args):
    """The reference's CPU path (oracle restatement) on the GPU arm's workload:
    the same model, prompt ids, prefill, warm-up and timed steps."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    load_pkg()
    orc = load_oracle()
    from hf_llm_b200 import model, synth
    cfg = model_cfg(args.model, args.layers)
    host = synth.llama_tensors(cfg, model.q4_k_m_types(), args.seed)
    threads = os.cpu_count() or 1
    prompt = prompt_ids(cfg, args.seed, args.prefill)
    r = cpu_decode(orc, cfg, host, prompt, [(threads, args.warmup, args.steps)])[0]
    r["sample"] = (f"context of the GPU arm's {args.prefill}-token prompt (f32 KV cache filled with seeded "
                   f"rows, the last prompt token run through the forward), {args.warmup} warm-up and "
                   f"{args.steps} timed greedy decode steps, {threads} threads (OpenMP), quantised-x "
                   f"AVX2/FMA matvecs, f32 KV cache as the reference keeps it")
    line = {"metric": f"decode tok/s at Llama-3-{args.model.upper()} Q4_K_M shape", "value": r["value"],
            "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 / r["value"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8/f32", "data": "synthetic",
            "config": workload_config(args.model, cfg, args.prefill),
            "cpu_baseline": r,
            "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def timed_decode(m, tok, pos, steps, sp, stream, dist, dev, clk_dev):
    """K timed single-token steps (device argmax feeds the next step), CUDA
    events on `stream`, max over ranks.  Returns (ms, pos, clocks, library
    kernel launches inside the timed region)."""
    import torch

    def step(p):
        m.forward_dev(tok.data_ptr(), 1, p, 0, tok.data_ptr(), sp)

    stream.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    # untimed: its all-rank barriers align the ranks' streams on the device
    step(pos)
    pos += 1
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = m.engine.kernel_launches()
    with ClockSampler(clk_dev) as clk:
        ev0.record(stream)
        for _ in range(steps):
            step(pos)
            pos += 1
        ev1.record(stream)
        ev1.synchronize()
    launches = m.engine.kernel_launches() - launches0
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, pos, clk.summary(), launches


def timed_e2e(m, tok0, pos, steps, dist, dev):
    """b2q_forward with host token ids and host logits every step (into a
    page-locked array; the next token is the library's greedy argmax, which
    b2q_forward returns beside the logits); host wall clock, max over
    ranks."""
    import torch
    nxt = tok0
    logits = torch.empty(m.cfg["n_vocab"], dtype=torch.float32, pin_memory=True).numpy()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        nxt = m.forward_into([nxt], pos, logits)
        pos += 1
    s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        s = float(t.item())
    return s, pos


def tp_parity(engine, orc, rank, world, dist, seed=0x7A):
    """Fixed-seed 2-layer model of Llama-3-8B widths (unit distribution) on
    the same ranks and step path as the benchmark: a 20-token prompt and three
    single-token steps, logits against the fp64 oracle on rank 0."""
    from hf_llm_b200 import model, synth
    cfg = model_cfg("8b", 2)
    tp_id = None
    if world > 1:
        obj = [model.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        tp_id = obj[0]
    m, _ = build_model(engine, cfg, seed, rank, world, tp_id, 64, dist="unit")
    ref = None
    if rank == 0:
        full = synth.llama_tensors(cfg, model.q4_k_m_types(), seed, dist="unit")
        ref = orc.Model(cfg, full, kv_capacity=64)
    prompt = [int(v) for v in prompt_ids(cfg, seed, 20)]
    errs, toks, pos = [], [prompt], 0
    for s in range(4):
        a = m.forward(toks[-1], pos)
        nxt = 0
        if rank == 0:
            b = ref.forward_f64(toks[-1], pos, kv_f16=True)
            errs.append(float(np.linalg.norm(a - b) / np.linalg.norm(b)))
            nxt = int(np.argmax(b))
        if dist:
            o = [nxt]
            dist.broadcast_object_list(o, src=0)
            nxt = o[0]
        pos += len(toks[-1])
        toks.append([nxt])
    path = m.step_path
    m.close()
    if rank != 0:
        return None
    return {"rel_l2": max(errs), "rel_l2_per_step": [round(e, 8) for e in errs], "tol": 1e-3,
            "ok": bool(max(errs) <= 1e-3), "tp": world, "step_path": path,
            "model": "Llama-3-8B widths, 2 layers, unit distribution; 20-token prompt + 3 single-token steps",
            "oracle": "fp64 forward over the bit-exact dequantised weights, f16 KV"}


def run_model(args, name, engine, rank, world, local, dist, dev, stream, orc):
    """One model's decode measurements on this rank; returns the fields of
    its bench block (rank 0) and the host tensors (N = 1, 8B only)."""
    import torch
    from hf_llm_b200 import model
    cfg = model_cfg(name, args.layers)
    is70 = name == "70b"
    steps = args.steps
    e2e_steps = args.e2e_steps_70b if is70 else args.e2e_steps
    tp_id = None
    if world > 1:
        obj = [model.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        tp_id = obj[0]
    max_seq = 8192 if is70 else args.prefill + args.warmup + steps + e2e_steps + 8
    t_load = time.perf_counter()
    m, host = build_model(engine, cfg, args.seed, rank, world, tp_id, max_seq, decode=args.decode,
                          keep_host=(world == 1 and not is70 and not args.no_cpu), share_layers=is70)
    t_load = time.perf_counter() - t_load
    sp = stream.cuda_stream
    tok = torch.zeros(2, dtype=torch.int32, device=dev)
    prefill = None
    if is70:
        # an 8192-token context: seeded synthetic K/V rows up to the first step
        pos = max_seq - (args.warmup + 1 + steps + e2e_steps + 1)
        m.fill_kv(0, pos, seed=args.seed, scale=1.0)
        tok.fill_(int(prompt_ids(cfg, args.seed, 1)[0]))
    else:
        prompt = torch.tensor(prompt_ids(cfg, args.seed, args.prefill), device=dev)
        with torch.cuda.stream(stream):
            m.forward_dev(prompt.data_ptr(), args.prefill, 0, 0, tok.data_ptr(), sp)
        stream.synchronize()
        pos = args.prefill
    for _ in range(args.warmup):
        m.forward_dev(tok.data_ptr(), 1, pos, 0, tok.data_ptr(), sp)
        pos += 1
    pos_t0 = pos + 1  # after the aligning step
    ms, pos, clocks, launches = timed_decode(m, tok, pos, steps, sp, stream, dist, dev, local)
    ms_step = ms / steps
    value = steps / (ms / 1000.0)
    e2e_s, pos = timed_e2e(m, int(tok[0].item()), pos, e2e_steps, dist, dev)
    e2e = {"value": e2e_steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4,
           "d2h_bytes_per_step": 4 * cfg["n_vocab"] + 4,
           "note": "b2q_forward with host token ids and host logits (a page-locked array) and the greedy "
                   "argmax it returns; host wall clock, max over ranks"}
    peak, peak_kind = measured_peaks()
    ctx = pos_t0 + steps // 2
    step_bytes = step_algorithmic_bytes(cfg, rank, world, ctx)
    step_gbs = step_bytes / (ms_step * 1e-3) / 1e9
    roof = None
    if m.decode_mode == "persistent":
        traffic = None
        if world == 1 and not is70 and cfg["n_layers"] == 32:
            traffic = profile_traffic("decode_kernel_llama3_8b.md")
        elif world == 1 and is70 and cfg["n_layers"] == 80:
            traffic = scaled_profile_traffic("decode_kernel_llama3_70b_2layers_8192ctx.md", step_bytes)
        traffic_source = (None if traffic is None else
                          "ncu capture of this launch" if not is70 else
                          "ncu capture of the 2-layer 8192-key case, its traffic/algorithmic ratio (1.0025) "
                          "times this launch's algorithmic bytes")
        roof = {"bound": "hbm", "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                "frac": round(step_gbs / peak, 4), "traffic": traffic, "traffic_source": traffic_source,
                "kernel": "decode_kernel (persistent single-token step)",
                "algorithmic_bytes_per_launch": int(step_bytes), "peak_kind": peak_kind,
                "launch_us": round(ms_step * 1000, 2), "context": ctx}
    if not is70 and args.prefill >= 16:
        reps = 3
        with torch.cuda.stream(stream):
            m.forward_dev(prompt.data_ptr(), args.prefill, 0, 0, tok.data_ptr(), sp)  # warm-up
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.synchronize()
        if dist:
            dist.barrier()
        e0.record(stream)
        for _ in range(reps):
            m.forward_dev(prompt.data_ptr(), args.prefill, 0, 0, tok.data_ptr(), sp)
        e1.record(stream)
        e1.synchronize()
        pms = e0.elapsed_time(e1) / reps
        if dist:
            t = torch.tensor([pms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            pms = float(t.item())
        flops = 2.0 * args.prefill * prefill_matmul_params(cfg, rank, world)
        tf = flops / (pms * 1e-3) / 1e12
        pk = load_peaks().get("bf16_tflops")
        prefill = {"tokens": args.prefill, "ms": round(pms, 3), "tok_s": round(args.prefill / (pms * 1e-3), 1),
                   "matmul_tflops_rank0": round(tf, 1),
                   "frac_of_bf16_peak": round(tf / pk, 4) if pk else None,
                   "note": "whole prompt pass (norms, attention, f16 tensor-core projections); "
                           "flops = 2 x tokens x projection weights of the layers (head excluded)"}
    decode_path = m.decode_mode
    m.close()
    block = {"value": round(value, 2), "ms_per_step": round(ms_step, 4), "steps": steps,
             "roofline": roof, "e2e": e2e, "gpu_launches": int(launches), "clocks": clocks,
             "decode_step": {"bytes_per_step_rank0": int(step_bytes), "GBps_rank0": round(step_gbs, 1)},
             "config": workload_config(name, cfg, 0 if is70 else args.prefill,
                                       f"{ctx} cached tokens (f16 KV rows: seeded synthetic fill)" if is70 else None),
             "decode_path": decode_path, "load_s": round(t_load, 1)}
    if prefill:
        block["prefill"] = prefill
    return block, host, cfg


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b2q", choices=["b2q", "reference"])
    ap.add_argument("--prefill", type=int, default=512)
    ap.add_argument("--seed", type=int, default=0x5EED)
    ap.add_argument("--cpu-steps", type=int, default=6, help="timed CPU-baseline steps per thread count")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--e2e-steps-70b", type=int, default=16)
    ap.add_argument("--model", default="8b", choices=["8b", "70b"],
                    help="headline model: Llama-3-8B (the metric's workload) or, for profiles, Llama-3-70B")
    ap.add_argument("--no-70b", action="store_true", help="skip the Llama-3-70B block")
    ap.add_argument("--no-parity", action="store_true", help="skip the tp_parity check")
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder layers (default: the model's; fewer only for kernel profiles on a small case)")
    ap.add_argument("--decode", default="persistent", choices=["persistent", "graph", "eager"],
                    help="single-token step: one persistent kernel, the captured kernel graph, or eager")
    ap.add_argument("--no-gemv-shapes", action="store_true", help="skip the per-shape GEMV timings")
    ap.add_argument("--gemv-only", default=None,
                    help="time one GEMV shape only (e.g. q4k_14336x4096), for kernel profiling")
    ap.add_argument("--copies", type=int, default=24, help="weight copies rotated by --gemv-only")
    ap.add_argument("--reps", type=int, default=20, help="rotations timed by --gemv-only")
    ap.add_argument("--chained", action="store_true", help="--gemv-only: chain launches (programmatic dependent launch)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.gemv_only:
        return run_gemv_only(args)

    import torch
    load_pkg()
    from hf_llm_b200 import build as bld
    bld.build()
    from hf_llm_b200 import synth
    from hf_llm_b200.engine import CudaEngine

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        world = args.gpus if world == 1 else world
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
        local = 0
    dev = torch.device("cuda", local)
    engine = CudaEngine(local)
    stream = torch.cuda.Stream(device=dev)
    sp = stream.cuda_stream
    orc = load_oracle() if rank == 0 else None

    head, host, cfg = run_model(args, args.model, engine, rank, world, local, dist, dev, stream, orc)

    # the standalone GEMV (Q4_K, FFN gate shape) and the other matvec shapes
    peak, peak_kind = measured_peaks()
    gemv_roof = None
    gemv_shapes = {}
    if rank == 0:
        keys = ["q4k_14336x4096"] if args.no_gemv_shapes else list(GEMV_SHAPES)
        for key in keys:
            ms_l, alg = time_gemv_shape(engine, synth, key, args.seed, dev, sp)
            ms_c, _ = time_gemv_shape(engine, synth, key, args.seed, dev, sp, chained=True)
            gemv_shapes[key] = {"us": round(ms_l * 1000, 3), "GBps": round(alg / (ms_l * 1e-3) / 1e9, 1),
                                "us_chained": round(ms_c * 1000, 3),
                                "GBps_chained": round(alg / (ms_c * 1e-3) / 1e9, 1), "bytes": alg}
            if key == "q4k_14336x4096":
                ach = alg / (ms_c * 1e-3) / 1e9
                gemv_roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(ach / peak, 4), "traffic": profile_traffic(),
                             "kernel": "gemv_kernel (Q4_K, 14336x4096), launches chained by programmatic "
                                       "dependent launch as in the per-kernel decode path",
                             "algorithmic_bytes_per_launch": alg, "peak_kind": peak_kind,
                             "launch_us": round(ms_c * 1000, 3),
                             "single_launch": {"launch_us": round(ms_l * 1000, 3),
                                               "achieved": round(alg / (ms_l * 1e-3) / 1e9, 1),
                                               "frac": round(alg / (ms_l * 1e-3) / 1e9 / peak, 4)}}

    # the Q6_K output head, row-sharded over the ranks (every rank)
    head_shard = time_head_shard(engine, synth, world, rank, args.seed, dev, sp, dist, peak, peak_kind)

    cpu = None
    if rank == 0 and world == 1 and host:
        try:
            cores = os.cpu_count() or 1
            gov = governor_threads(cores)
            prompt = prompt_ids(cfg, args.seed, args.prefill)
            r_gov, r_all = cpu_decode(orc, cfg, host, prompt, [(gov, 1, args.cpu_steps), (cores, 1, args.cpu_steps)])
            cpu = dict(r_all)
            cpu["sample"] = (f"context of the {args.prefill}-token prompt (f32 KV cache filled with seeded rows), "
                             f"then {args.cpu_steps} timed greedy decode steps per thread count, full "
                             f"{cfg['n_layers']}-layer model, quantised-x AVX2/FMA matvecs; value at all {cores} "
                             f"host threads")
            cpu["governor_threads"] = {"cores": gov, "value": r_gov["value"], "unit": "tok/s",
                                       "rule": "min(3/4 cores, cores - 2), hardware.rs:157-166"}
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "error": str(ex)}
        try:  # the matvec config shapes on the same CPU path, beside gemv_shapes
            cores = os.cpu_count() or 1
            keys = ["q4k_14336x4096"] if args.no_gemv_shapes else list(GEMV_SHAPES)
            cpu["matvec_shapes"] = {key: cpu_matvec_shape(orc, synth, key, args.seed,
                                                          sorted({governor_threads(cores), cores}))
                                    for key in keys}
            cpu["matvec_note"] = ("oracle matmul_batched (x quantised, AVX2/FMA row dots) per call, weight copies "
                                  "rotated past 256 MB; GBps = the GPU side's algorithmic bytes / call time")
        except Exception as ex:
            cpu["matvec_shapes"] = {"error": str(ex)}
    host = None

    parity = None
    if not args.no_parity and args.decode == "persistent":
        parity = tp_parity(engine, orc, rank, world, dist)

    m70 = None
    if not args.no_70b and args.model == "8b" and args.layers is None:
        m70, _, _ = run_model(args, "70b", engine, rank, world, local, dist, dev, stream, orc)

    if rank == 0:
        line = {"metric": f"decode tok/s at Llama-3-{args.model.upper()} Q4_K_M shape", "value": head["value"],
                "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": head["ms_per_step"], "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None,
                "dtype": "int16xint8 dp2a, f32 accum", "data": "synthetic",
                "config": head["config"],
                "parallelism": f"tp{world}", "kv_cache": "f16", "decode_path": head["decode_path"],
                "decode_step": head["decode_step"],
                "roofline": head["roofline"], "gemv_roofline": gemv_roof, "gemv_shapes": gemv_shapes,
                "output_head": head_shard,
                "prefill": head.get("prefill"), "cpu_baseline": cpu, "e2e": head["e2e"],
                "tp_parity": parity, "model_70b": m70,
                "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
                "load_s": head["load_s"]}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
