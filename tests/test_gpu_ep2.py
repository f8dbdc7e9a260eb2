"""Expert-parallel MoE block on two GPUs (skipped with fewer than two GPUs).

Two processes, one per GPU, NCCL for the all-reduce of the ranks' shares (NVLS off).  Each rank
holds half of the experts (moe.expert_shard); the all-reduced output of moe_block_ep equals, on
both ranks, the single-GPU block over all experts within 1e-2 relative L2 (the shares are
rounded to bf16 before the sum)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(e, n, k, seed, d):
    from tests.test_gpu_nvfp4 import random_weight
    ws = [random_weight(n, k, seed=seed + i, realistic=False) for i in range(e)]
    return (torch.stack([torch.from_numpy(w[0]) for w in ws]).to(d),
            torch.stack([torch.from_numpy(w[2]) for w in ws]).to(d),
            torch.tensor([w[3] for w in ws], dtype=torch.float32, device=d))


def _run(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from adallm_b200.moe import expert_shard, moe_block_ep
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        d = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=d)
        t, e, k, hid, inter = 16, 16, 4, 512, 256
        gu = _weights(e, 2 * inter, hid, 700, d)
        dn = _weights(e, hid, inter, 800, d)
        g = torch.Generator().manual_seed(11)
        x = torch.randn((t, hid), generator=g).to(torch.bfloat16).to(d)
        logits = torch.randn((t, e), generator=g).to(torch.bfloat16).to(d)
        base, cnt = expert_shard(e, world, rank)
        sl = lambda p: tuple(a[base:base + cnt].contiguous() for a in p)
        out = moe_block_ep(x, logits, k, True, sl(gu), sl(dn), base, group=dist.group.WORLD)
        full = moe_block_ep(x, logits, k, True, gu, dn, 0)
        torch.cuda.synchronize()
        rel = float((out.float() - full.float()).norm() / full.float().norm())
        outs = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(outs, out)
        same = bool(torch.equal(outs[0], outs[1]))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, {"rel": rel, "same": same}))
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, {"exception": repr(exc)}))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep2_block_matches_single_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, out = q.get(timeout=600)
        res[rank] = out
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert "exception" not in res[r], res[r]
        assert res[r]["same"]
        assert res[r]["rel"] < 1e-2, res[r]
