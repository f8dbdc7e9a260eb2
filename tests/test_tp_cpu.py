"""Tensor-parallel host logic on CPU with two gloo ranks (no GPU).

The decode engine shards its NVFP4 linears like the reference's parallel linears
(adallm/ops/linear.py:116-215) and picks the greedy token over a vocab-parallel lm_head.
Each rank builds its shards with the engine's own functions; the ranks then reproduce the
unsharded results with the collectives the engine uses:
  * column-parallel qkv / gate_up: gathered per-part output blocks == the full output
  * row-parallel o_proj / down: all-reduce of partial products == the full product
  * vocab-parallel embedding rows == rows of the full table
  * vocab-parallel greedy pick == argmax over the full vocabulary (first maximum on ties)
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import nvfp4 as nv

HIDDEN, HQ, HKV, D, INTER, VOCAB = 256, 4, 2, 64, 512, 1000


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dq(packed: torch.Tensor, scale: torch.Tensor, s2: float) -> np.ndarray:
    return nv.dequant_nvfp4(packed.numpy(), scale.float().numpy(), s2).astype(np.float64)


def _worker(rank: int, world: int, port: int, q):
    from adallm_b200.decode_step import sharded_nvfp4, fill_rows, vocab_parallel_pick
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = torch.Generator().manual_seed(123)
        x = torch.randn((3, HIDDEN), generator=g, dtype=torch.float64)
        errs = {}

        # column-parallel fused qkv: rank r holds [q_r; k_r; v_r]
        parts = [("q", HQ * D), ("k", HKV * D), ("v", HKV * D)]
        full = sharded_nvfp4(7, "qkv", 0, parts, HIDDEN, False, 1, 0, "cpu")
        mine = sharded_nvfp4(7, "qkv", 0, parts, HIDDEN, False, world, rank, "cpu")
        y_full = x.numpy() @ _dq(*full).T
        y_mine = torch.from_numpy(x.numpy() @ _dq(*mine).T)
        got = [torch.empty_like(y_mine) for _ in range(world)]
        dist.all_gather(got, y_mine)
        cols, base = [], 0
        for _, rows in parts:  # reassemble [q_0 q_1 | k_0 k_1 | v_0 v_1]
            r = rows // world
            for rk in range(world):
                cols.append(got[rk][:, base:base + r])
            base += r
        errs["column"] = float(np.abs(torch.cat(cols, 1).numpy() - y_full).max())

        # row-parallel down: rank r holds K slice r; partial products are summed
        full = sharded_nvfp4(7, "down", 0, [("down", HIDDEN)], INTER, True, 1, 0, "cpu")
        mine = sharded_nvfp4(7, "down", 0, [("down", HIDDEN)], INTER, True, world, rank, "cpu")
        xi = torch.randn((3, INTER), generator=g, dtype=torch.float64)
        kk = INTER // world
        part = torch.from_numpy(xi[:, rank * kk:(rank + 1) * kk].numpy() @ _dq(*mine).T)
        dist.all_reduce(part)
        errs["row"] = float(np.abs(part.numpy() - xi.numpy() @ _dq(*full).T).max())
        errs["scale_2_shared"] = float(mine[2] != full[2])

        # vocab-parallel embedding shard == rows of the full table
        shard = VOCAB // world
        tab_full = torch.empty((VOCAB, 32), dtype=torch.bfloat16)
        fill_rows(tab_full, 5, "embed", 0, chunk=96)
        tab_mine = torch.empty((shard, 32), dtype=torch.bfloat16)
        fill_rows(tab_mine, 5, "embed", rank * shard, chunk=96)
        errs["embed"] = float(not torch.equal(tab_mine, tab_full[rank * shard:(rank + 1) * shard]))

        # vocab-parallel greedy pick, with a tie across the two shards in row 1
        logits = torch.randn((4, VOCAB), generator=g)
        logits[1, 10] = 50.0
        logits[1, shard + 10] = 50.0
        logits[2, VOCAB - 1] = 60.0
        loc = logits[:, rank * shard:(rank + 1) * shard]
        lmax, lidx = loc.max(dim=1).values, loc.argmax(dim=1)
        pick = vocab_parallel_pick(lmax, lidx, rank, shard, world)
        errs["pick"] = float(not torch.equal(pick, logits.argmax(dim=1)))
        q.put((rank, errs))
        dist.destroy_process_group()
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, {"exception": repr(exc)}))


def test_tensor_parallel_sharding_gloo_world2():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, errs = q.get(timeout=180)
        results[rank] = errs
    for p in procs:
        p.join(timeout=60)
    for rank, errs in results.items():
        assert "exception" not in errs, (rank, errs)
        assert errs["column"] < 1e-9 and errs["row"] < 1e-9, (rank, errs)
        assert errs["scale_2_shared"] == 0 and errs["embed"] == 0 and errs["pick"] == 0, (rank, errs)


def _ep_rank(rank, world, port, q):
    """Expert parallelism host logic on gloo: each rank owns a contiguous expert block and
    contributes only the routed slots of its experts; the all-reduce of the shares equals the
    full weighted sum."""
    import os
    import torch
    import torch.distributed as dist
    from adallm_b200.moe import expert_shard
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        e, t, k, h = 8, 5, 3, 4
        g = torch.Generator().manual_seed(0)
        ids = torch.stack([torch.randperm(e, generator=g)[:k] for _ in range(t)])
        w = torch.rand((t, k), generator=g)
        expert_out = torch.randn((e, t, h), generator=g)  # what expert x would give token t
        base, cnt = expert_shard(e, world, rank)
        mine = (ids >= base) & (ids < base + cnt)
        share = torch.zeros((t, h))
        for i in range(t):
            for j in range(k):
                if mine[i, j]:
                    share[i] += w[i, j] * expert_out[ids[i, j], i]
        dist.all_reduce(share)
        full = torch.zeros((t, h))
        for i in range(t):
            for j in range(k):
                full[i] += w[i, j] * expert_out[ids[i, j], i]
        q.put((rank, float((share - full).abs().max())))
        dist.destroy_process_group()
    except Exception as exc:
        q.put((rank, repr(exc)))


def test_expert_parallel_shares_all_reduce_to_full_gloo():
    import socket
    import torch.multiprocessing as mp
    from adallm_b200.moe import expert_shard
    assert expert_shard(128, 8, 3) == (48, 16)
    with pytest.raises(ValueError):
        expert_shard(10, 4, 0)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ep_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert isinstance(res[r], float) and res[r] < 1e-5, res[r]
