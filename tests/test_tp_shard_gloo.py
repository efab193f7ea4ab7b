"""Tensor-parallel host logic on CPU, as world_size-2 gloo ranks.

Each rank asks the library for its row and column ranges (b2q_tp_shard_rows,
b2q_tp_shard_cols; no device) and computes its part of every weight's matvec
with the oracle: its rows for the row-split tensors, partial sums over its
columns for attn_output and ffn_down.  The ranks all-gather the parts with
torch.distributed -- the exchanges the device path performs.  Rank 0 checks
that the ranges tile every tensor exactly (heads kept whole, KV groups
aligned with their query heads, attn_output columns = the rank's query heads,
ffn_down columns = its ffn_gate/up rows), that the gathered rows equal the
unsharded product and that the partial sums add up to it.
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
        mine = {}
        for spec in specs:
            name, dtype, dims, _ = spec
            if len(dims) != 2:
                continue
            n, k = dims
            x = synth.activation(k, 3)
            b, e = model.tp_shard_rows(CFG, name, n, rank, world)
            cb, ce = model.tp_shard_cols(CFG, name, k, rank, world)
            if name == "token_embd.weight":
                mine[name] = (b, e, cb, ce, None)
                continue
            raw = synth.llama_tensor(spec, 5, b, e)  # this rank's rows only
            w = orc.dequantize(raw.reshape(-1), dtype, (e - b) * k).reshape(e - b, k).astype(np.float64)
            part = w[:, cb:ce] @ x[0, cb:ce].astype(np.float64)  # rows, or a partial sum over columns
            mine[name] = (b, e, cb, ce, part)
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
                    assert all(p[:4] == (0, n, 0, k) for p in parts), name  # replicated
                    continue
                x = synth.activation(k, 3)
                full = orc.matmul_f64(synth.llama_tensor(spec, 5), dtype, n, k, x)[0]
                role = name.split(".")[2] if name.startswith("blk.") else name
                if role in ("attn_output", "ffn_down"):
                    # every row on every rank; contiguous, ordered, exact tiling of the columns
                    assert all(p[:2] == (0, n) for p in parts), name
                    assert parts[0][2] == 0 and parts[-1][3] == k, name
                    for a, c in zip(parts, parts[1:]):
                        assert a[3] == c[2], name
                    total = sum(p[4] for p in parts)
                    assert np.allclose(total, full, rtol=1e-12, atol=1e-12 * np.abs(full).max()), name
                    continue
                # contiguous, ordered, exact tiling of [0, n), all columns
                assert all(p[2:4] == (0, k) for p in parts), name
                assert parts[0][0] == 0 and parts[-1][1] == n, name
                for a, c in zip(parts, parts[1:]):
                    assert a[1] == c[0], name
                if role in ("attn_q", "attn_k", "attn_v"):
                    hd = CFG["head_dim"]
                    assert all((p[1] - p[0]) % hd == 0 for p in parts), name  # whole heads
                cat = np.concatenate([p[4] for p in parts])
                assert np.allclose(cat, full, rtol=1e-12, atol=1e-12 * np.abs(full).max()), name
            # q heads of rank r are exactly the query heads of its KV heads
            G = CFG["n_heads"] // CFG["n_kv_heads"]
            hd = CFG["head_dim"]
            for r, g in enumerate(gathered):
                qb, qe = g["blk.0.attn_q.weight"][:2]
                kb, ke = g["blk.0.attn_k.weight"][:2]
                assert (qb // hd, qe // hd) == (G * (kb // hd), G * (ke // hd)), r
                # attn_output's columns are this rank's query heads, ffn_down's its gate/up rows
                assert g["blk.0.attn_output.weight"][2:4] == (qb, qe), r
                assert g["blk.0.ffn_down.weight"][2:4] == g["blk.0.ffn_gate.weight"][:2], r
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_tp_shards_tile_and_gather_gloo():
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)
