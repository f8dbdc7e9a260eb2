"""Two-GPU tensor parallelism of the decode engine (skipped with fewer than two GPUs).

Two processes, one per GPU, NCCL for the embedding all-reduce and the vocab-parallel pick,
NVLink peer memory for the row-parallel projections (GEMM epilogues write every rank's inbox;
the RMSNorm on each rank waits for the count and sums all ranks' planes).  With the same token
fed to every step, the gathered TP2 logits match the TP1 engine's within 2e-2 relative L2 (the
K splits are summed in a different order), both ranks hold identical hidden states, and no
peer wait timed out."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

LAYERS, B, STEPS = 3, 4, 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens(step):
    return torch.tensor([(7 * step + 3 * i + 1) % 1000 for i in range(B)])


def _run(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from adallm_b200 import _native as N
    from adallm_b200.decode_step import Qwen3DecodeEngine, DecodeSession
    from tests.decode_check import small_config
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        d = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=d)
        cfg = small_config(LAYERS)
        cfg.tp_size, cfg.tp_rank = world, rank
        eng = Qwen3DecodeEngine(cfg, d, B, max_ctx=32, seed=7, group=dist.group.WORLD)
        assert eng.tp_peer
        sess = DecodeSession(eng, seed=7)
        logits, hidden = [], []
        for s in range(STEPS):
            sess.prepare(_tokens(s))
            sess.upload()
            eng.forward()
            sess.download()
            sess.commit()
            parts = [torch.empty_like(eng.logits) for _ in range(world)]
            dist.all_gather(parts, eng.logits)
            logits.append(torch.cat(parts, 1).float().cpu())
            hidden.append(eng.xnorm.float().cpu())
        torch.cuda.synchronize()
        ws = eng.gemm_only_ws[:4].view(torch.int32).item()
        eng.close()
        out = {"logits": torch.stack(logits).numpy(), "xnorm": torch.stack(hidden).numpy(), "err": ws}
        if rank == 0:
            cfg1 = small_config(LAYERS)
            e1 = Qwen3DecodeEngine(cfg1, d, B, max_ctx=32, seed=7)
            s1 = DecodeSession(e1, seed=7)
            ref = []
            for s in range(STEPS):
                s1.prepare(_tokens(s))
                s1.upload()
                e1.forward()
                s1.download()
                s1.commit()
                ref.append(e1.logits.float().cpu())
            out["ref"] = torch.stack(ref).numpy()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out))  # numpy arrays: sent by value, the process may exit before they are read
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, {"exception": repr(exc)}))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_engine_matches_tp1():
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
        assert res[r]["err"] == 0
    assert (res[0]["xnorm"] == res[1]["xnorm"]).all()
    assert (res[0]["logits"] == res[1]["logits"]).all()
    got, ref = torch.from_numpy(res[0]["logits"]), torch.from_numpy(res[0]["ref"])
    rel = float((got - ref).norm() / ref.norm())
    assert rel < 2e-2, rel
