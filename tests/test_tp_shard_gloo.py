"""Tensor-parallel host logic on CPU, as world_size-2 gloo ranks.

Each rank asks the library for its row ranges (b2q_tp_shard_rows, no device),
computes its rows of every weight's matvec with the oracle, and the ranks
all-gather the slices with torch.distributed -- the exchange the device path
performs with NCCL after each row-sharded matvec.  Rank 0 checks that the
ranges tile every tensor exactly (heads kept whole, KV groups aligned with
their query heads) and that the gathered product equals the unsharded one.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

CFG = dict(n_layers=1, n_embd=512, n_heads=8, n_kv_heads=4, head_dim=64, n_ff=1024, n_vocab=640,
           rms_eps=1e-5, rope_theta=10000.0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int) -> None:
    import sys
    from pathlib import Path
    import torch.distributed as dist
    here = Path(__file__).resolve().parent
    sys.path.insert(0, str(here))
    from conftest import load_oracle, load_pkg
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        load_pkg()
        orc = load_oracle()
        from hf_llm_b200 import model, synth
        specs = synth.llama_specs(CFG, model.q4_k_m_types())
        x = synth.activation(CFG["n_embd"], 3)
        mine = {}
        for spec in specs:
            name, dtype, dims, _ = spec
            if len(dims) != 2:
                continue
            n, k = dims
            b, e = model.tp_shard_rows(CFG, name, n, rank, world)
            if k != CFG["n_embd"] or name == "token_embd.weight":
                mine[name] = (b, e, None)
                continue
            raw = synth.llama_tensor(spec, 5, b, e)  # this rank's rows only
            mine[name] = (b, e, orc.matmul_f64(raw, dtype, e - b, k, x)[0])
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        if rank == 0:
            for spec in specs:
                name, dtype, dims, _ = spec
                if len(dims) != 2:
                    continue
                n, k = dims
                parts = [g[name] for g in gathered]
                if name == "token_embd.weight":
                    assert all(p[:2] == (0, n) for p in parts), name  # replicated
                    continue
                # contiguous, ordered, exact tiling of [0, n)
                assert parts[0][0] == 0 and parts[-1][1] == n, name
                for a, c in zip(parts, parts[1:]):
                    assert a[1] == c[0], name
                if name.startswith("blk.0.attn_") and name.split(".")[2] in ("attn_q", "attn_k", "attn_v"):
                    hd = CFG["head_dim"]
                    assert all((p[1] - p[0]) % hd == 0 for p in parts), name  # whole heads
                if parts[0][2] is not None:
                    full = orc.matmul_f64(synth.llama_tensor(spec, 5), dtype, n, k, x)[0]
                    cat = np.concatenate([p[2] for p in parts])
                    assert np.array_equal(cat, full), name
            # q heads of rank r are exactly the query heads of its KV heads
            G = CFG["n_heads"] // CFG["n_kv_heads"]
            hd = CFG["head_dim"]
            for r, g in enumerate(gathered):
                qb, qe, _ = g["blk.0.attn_q.weight"]
                kb, ke, _ = g["blk.0.attn_k.weight"]
                assert (qb // hd, qe // hd) == (G * (kb // hd), G * (ke // hd)), r
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_tp_shards_tile_and_gather_gloo():
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)
