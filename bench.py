"""Decode benchmark: Llama-3-8B-shaped Q4_K_M decoder, batch 1.

Workload (the metric "decode tok/s at Llama-3-8B Q4_K_M shape; dequant-GEMV
HBM GB/s vs 8 TB/s"): a random-init 32-layer Llama-3-8B-shaped decoder
(hidden 4096, 32/8 heads, head_dim 128, FFN 14336, vocab 128256; attn_q/k/
output and ffn_gate/up Q4_K, attn_v / ffn_down / output Q6_K, token_embd
Q4_K, f32 norms, f16 KV cache), weights drawn from the seeded benchmark
distributions (synthetic: no checkpoints offline).  A 512-token random-id
prompt is prefilled, then one step = one greedy decode token at batch 1.

* value  -- decode tok/s with everything resident in HBM: each step replays
            the captured decode graph; the next token id is the device argmax
            of the previous step (no host round trip).  CUDA events on the
            launching stream; weights (4.9 GB) far exceed L2.
* e2e    -- the same through the host API b2q_forward: token id copied from
            host, logits [128256] f32 copied back every step.
* roofline -- the dominant kernel family, the dequant-GEMV: Q4_K at the FFN
            gate shape 14336x4096 (33.1 MB per launch), launches timed with
            CUDA events while rotating 24 weight copies (794 MB > L2).
* cpu_baseline -- the reference's own CPU path (the oracle's restatement of
            the AVX2/FMA Rayon matvec + Llama forward) on the host cores.

--gpus N > 1 (launched under torchrun): tensor-parallel decode of the same
model, weights row-sharded over N GPUs, NCCL all-gathers; strong scaling.
--impl reference: the reference's CPU path on the same workload (rank 0).
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


def profile_traffic(name: str = "gemv_q4k_14336x4096.md") -> float | None:
    """DRAM bytes per launch from a committed ncu summary under profiles/
    (its "traffic_bytes_per_launch:" line), if one has been captured."""
    p = REPO / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


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


def build_model(pkg, engine, cfg, seed, rank, size, tp_id, max_seq, dist="bench", decode="persistent"):
    from hf_llm_b200 import model, synth
    m = model.StandardNativeEngine(engine, cfg, max_seq=max_seq, tp_rank=rank, tp_size=size, tp_id=tp_id,
                                   decode=decode)
    host = {}
    for spec in synth.llama_specs(cfg, model.q4_k_m_types()):
        name, t, dims, _ = spec
        if len(dims) == 1:
            arr = synth.llama_tensor(spec, seed, dist=dist)
            m.set_tensor(name, t, dims, arr)
            host[name] = (t, dims, arr)
            continue
        b, e = m.shard_rows(name, dims[0])
        arr = synth.llama_tensor(spec, seed, b, e, dist=dist)
        m.set_tensor(name, t, dims, arr, b, e)
        if size == 1:
            host[name] = (t, dims, arr)
        del arr
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


def cpu_decode_rate(orc, cfg, host, steps: int, warmup: int, threads: int) -> dict:
    """The reference CPU path: decode tok/s of the same model (prefill 8
    tokens, then `steps` timed greedy decode steps)."""
    orc.set_threads(threads)
    m = orc.Model(cfg, host, kv_capacity=8 + warmup + steps + 1)
    rng = np.random.default_rng(7)
    logits = m.forward_ref(rng.integers(0, cfg["n_vocab"], 8).tolist(), 0)
    pos = 8
    for _ in range(warmup):
        logits = m.forward_ref([int(np.argmax(logits))], pos)
        pos += 1
    t0 = time.perf_counter()
    for _ in range(steps):
        logits = m.forward_ref([int(np.argmax(logits))], pos)
        pos += 1
    dt = time.perf_counter() - t0
    return {"value": steps / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{steps} greedy decode steps after an 8-token prefill, full 32-layer model, "
                      f"{threads} threads (OpenMP), quantised-x AVX2/FMA matvecs"}


GEMV_SHAPES = {  # key: (ggml type, n, k, copies rotated to exceed L2)
    "q4k_14336x4096": (12, 14336, 4096, 24), "q4k_4096x14336": (12, 4096, 14336, 24),
    "q4k_4096x4096": (12, 4096, 4096, 48), "q4k_1024x4096": (12, 1024, 4096, 96),
    "q6k_128256x4096": (14, 128256, 4096, 2), "q6k_4096x14336": (14, 4096, 14336, 16),
    "q8_0_4096x4096": (8, 4096, 4096, 48),
    "q5k_14336x4096": (13, 14336, 4096, 20), "q4_0_4096x4096": (2, 4096, 4096, 48),
}


def time_gemv_shape(engine, synth, key, seed, dev, sp, copies=None, reps=None):
    import torch
    t, n, k, cp = GEMV_SHAPES[key]
    copies = copies or cp
    raw = synth.tensor_rows(t, n, k, seed, 900)
    bufs = [engine.try_upload_weight(raw, t, n, k) for _ in range(copies)]
    x = torch.randn(k, device=dev)
    engine.time_gemv(bufs, x.data_ptr(), k, 2, sp)  # warm-up
    reps = reps or max(2, 400 // copies)
    ms_l = engine.time_gemv(bufs, x.data_ptr(), k, reps, sp)
    alg = n * raw.shape[1] + 4 * k + 4 * n
    for b in bufs:
        b.free()
    return ms_l, alg


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
                                args.copies, args.reps)
    peak, kind = measured_peaks()
    gbs = alg / (ms_l * 1e-3) / 1e9
    print(json.dumps({"gemv": args.gemv_only, "us_per_launch": round(ms_l * 1000, 3),
                      "algorithmic_bytes": alg, "GBps": round(gbs, 1), "frac": round(gbs / peak, 4),
                      "peak": peak, "peak_kind": kind, "copies": args.copies, "reps": args.reps}))
    return 0


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    pkg = load_pkg()
    orc = load_oracle()
    from hf_llm_b200 import model, synth
    cfg = dict(model.LLAMA3_70B if args.model == "70b" else model.LLAMA3_8B)
    host = synth.llama_tensors(cfg, model.q4_k_m_types(), args.seed)
    threads = os.cpu_count() or 1
    steps = max(1, min(args.steps, args.cpu_steps))
    warm = max(0, min(args.warmup, 1))
    r = cpu_decode_rate(orc, cfg, host, steps, warm, threads)
    line = {"metric": f"decode tok/s at Llama-3-{args.model.upper()} Q4_K_M shape", "value": r["value"],
            "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus, "steps": steps, "warmup": warm,
            "ms_per_step": 1000.0 / r["value"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8/f32", "data": "synthetic",
            "config": {"workload": f"llama3-{args.model}-q4_k_m-decode", "prefill": 8, "batch": 1},
            "cpu_baseline": r,
            "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b2q", choices=["b2q", "reference"])
    ap.add_argument("--prefill", type=int, default=512)
    ap.add_argument("--seed", type=int, default=0x5EED)
    ap.add_argument("--cpu-steps", type=int, default=6)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--model", default="8b", choices=["8b", "70b"],
                    help="Llama-3-8B (the headline workload) or Llama-3-70B shape")
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder layers (default: the model's; fewer only for kernel profiles on a small case)")
    ap.add_argument("--decode", default="persistent", choices=["persistent", "graph", "eager"],
                    help="single-token step: captured kernel graph, one persistent kernel, or eager")
    ap.add_argument("--no-gemv-shapes", action="store_true", help="skip the per-shape GEMV timings")
    ap.add_argument("--gemv-only", default=None,
                    help="time one GEMV shape only (e.g. q4k_14336x4096), for kernel profiling")
    ap.add_argument("--copies", type=int, default=24, help="weight copies rotated by --gemv-only")
    ap.add_argument("--reps", type=int, default=20, help="rotations timed by --gemv-only")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.gemv_only:
        return run_gemv_only(args)

    import torch
    pkg = load_pkg()
    from hf_llm_b200 import build as bld
    bld.build()
    from hf_llm_b200 import model, synth
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
    tp_id = None
    if world > 1:
        obj = [model.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        tp_id = obj[0]

    base = model.LLAMA3_70B if args.model == "70b" else model.LLAMA3_8B
    cfg = dict(base, n_layers=args.layers or base["n_layers"])
    max_seq = args.prefill + args.warmup + args.steps + args.e2e_steps + 8
    t_load = time.perf_counter()
    m, host = build_model(pkg, engine, cfg, args.seed, rank, world, tp_id, max_seq, decode=args.decode)
    t_load = time.perf_counter() - t_load

    stream = torch.cuda.Stream(device=dev)
    sp = stream.cuda_stream
    rng = np.random.default_rng(args.seed)
    prompt = torch.tensor(rng.integers(0, cfg["n_vocab"], args.prefill).astype(np.int32), device=dev)
    tok = torch.zeros(2, dtype=torch.int32, device=dev)
    with torch.cuda.stream(stream):
        m.forward_dev(prompt.data_ptr(), args.prefill, 0, 0, tok.data_ptr(), sp)
    stream.synchronize()
    pos = args.prefill

    def step(p):
        # greedy: the argmax of this step is the input of the next one
        m.forward_dev(tok.data_ptr(), 1, p, 0, tok.data_ptr(), sp)

    for _ in range(args.warmup):
        step(pos)
        pos += 1
    stream.synchronize()
    if dist:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = engine.kernel_launches()
    with ClockSampler(local) as clk:
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_push("decode")
        ev0.record(stream)
        for _ in range(args.steps):
            step(pos)
            pos += 1
        ev1.record(stream)
        ev1.synchronize()
        torch.cuda.nvtx.range_pop()
    launches = engine.kernel_launches() - launches0
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = args.steps / (ms / 1000.0)

    # ---- e2e through the host API (token id in, logits out, every step) ----
    logits_host = np.empty(cfg["n_vocab"], np.float32)
    nxt = int(tok[0].item())
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        logits_host = m.forward([nxt], pos)
        nxt = int(np.argmax(logits_host))
        pos += 1
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = {"value": args.e2e_steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4,
           "d2h_bytes_per_step": 4 * cfg["n_vocab"],
           "note": "b2q_forward with host token ids and host logits; host wall clock"}

    # ---- roofline of the dominant kernel ----
    # persistent path: the decode kernel itself (the only kernel of a step);
    # bytes = what one step must read (weights it owns + KV rows) per launch
    peak, peak_kind = measured_peaks()
    ctx = args.prefill + args.warmup + args.steps // 2
    step_bytes = step_algorithmic_bytes(cfg, rank, world, ctx)
    step_gbs = step_bytes / (ms_step * 1e-3) / 1e9
    roof = None
    if m.decode_mode == "persistent":
        roof = {"bound": "hbm", "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                "frac": round(step_gbs / peak, 4),
                "traffic": profile_traffic(f"decode_kernel_llama3_{args.model}.md") if world == 1 else None,
                "kernel": "decode_kernel (persistent single-token step)",
                "algorithmic_bytes_per_launch": int(step_bytes), "peak_kind": peak_kind,
                "launch_us": round(ms_step * 1000, 2)}
    # the standalone GEMV (Q4_K, FFN gate shape) and the other matvec shapes
    gemv_roof = None
    gemv_shapes = {}
    if rank == 0:
        keys = ["q4k_14336x4096"] if args.no_gemv_shapes else list(GEMV_SHAPES)
        for key in keys:
            ms_l, alg = time_gemv_shape(engine, synth, key, args.seed, dev, sp)
            gemv_shapes[key] = {"us": round(ms_l * 1000, 3), "GBps": round(alg / (ms_l * 1e-3) / 1e9, 1),
                                "bytes": alg}
            if key == "q4k_14336x4096":
                ach = alg / (ms_l * 1e-3) / 1e9
                gemv_roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(ach / peak, 4), "traffic": profile_traffic(),
                             "kernel": "gemv_kernel (Q4_K, 14336x4096), one launch",
                             "algorithmic_bytes_per_launch": alg, "peak_kind": peak_kind,
                             "launch_us": round(ms_l * 1000, 3)}
    if roof is None:
        roof = gemv_roof

    # ---- prompt pass (prefill) on the tensor cores: the same prompt again ----
    prefill = None
    if args.prefill >= 16:
        reps = 3
        with torch.cuda.stream(stream):
            m.forward_dev(prompt.data_ptr(), args.prefill, 0, 0, tok.data_ptr(), sp)  # warm-up
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            orc = load_oracle()
            cpu = cpu_decode_rate(orc, cfg, host, args.cpu_steps, 1, os.cpu_count() or 1)
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "error": str(ex)}
    del host

    if rank == 0:
        line = {"metric": f"decode tok/s at Llama-3-{args.model.upper()} Q4_K_M shape", "value": round(value, 2),
                "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms_step, 4), "higher_is_better": True,
                "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
                "dtype": "int16xint8 dp2a, f32 accum", "data": "synthetic",
                "config": {"workload": f"llama3-{args.model}-q4_k_m-decode", "layers": cfg["n_layers"],
                           "hidden": cfg["n_embd"], "heads": f"{cfg['n_heads']}/{cfg['n_kv_heads']}",
                           "ffn": cfg["n_ff"], "vocab": cfg["n_vocab"], "prefill": args.prefill,
                           "batch": 1, "kv_cache": "f16", "tp": world, "decode": m.decode_mode,
                           "l2": f"inputs larger than L2 ({step_bytes / 1e9:.1f} GB read per step)"},
                "decode_step": {"bytes_per_step_rank0": int(step_bytes), "GBps_rank0": round(step_gbs, 1)},
                "roofline": roof, "gemv_roofline": gemv_roof, "gemv_shapes": gemv_shapes, "prefill": prefill,
                "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": int(launches), "clocks": clk.summary(),
                "load_s": round(t_load, 1)}
        print(json.dumps(line), flush=True)
    m.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
