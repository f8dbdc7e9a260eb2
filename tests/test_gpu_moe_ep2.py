"""Expert parallelism of the MoE decode engine on two GPUs (skipped with fewer than two).

Two processes, one per GPU: each holds half of the 128 experts of every layer (ep_size 2), runs
the same attention and routing, the grouped GEMMs over the rows routed to its own experts, sums
its slots in fp32 and all-reduces them in fp32 (NCCL) before the one rounding to bf16.  With the
same tokens fed to every step, both ranks hold identical logits, which match the single-GPU engine
holding every expert within 1e-2 relative L2 (only the order of the fp32 additions differs; a bf16
all-reduce of per-rank rounded sums measured 2.2e-2 here), and no bounded wait ran out."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

LAYERS, B, STEPS = 3, 16, 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens(step):
    return torch.tensor([(7 * step + 3 * i + 1) % 1000 for i in range(B)])


def _steps(eng, sess):
    out = []
    for s in range(STEPS):
        sess.prepare(_tokens(s))
        sess.upload()
        eng.forward()
        sess.download()
        sess.commit()
        out.append(eng.logits.float().cpu())
    return torch.stack(out)


def _run(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from adallm_b200.decode_step import DecodeSession
    from adallm_b200.moe_step import Qwen3MoeDecodeEngine
    from tests.decode_check import moe_test_config
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        d = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=d)
        cfg = moe_test_config(LAYERS)
        cfg.ep_size, cfg.ep_rank = world, rank
        eng = Qwen3MoeDecodeEngine(cfg, d, B, max_ctx=32, seed=7, group=dist.group.WORLD)
        logits = _steps(eng, DecodeSession(eng, seed=7))
        eng.check_errors()
        out = {"logits": logits.numpy()}
        if rank == 0:
            e1 = Qwen3MoeDecodeEngine(moe_test_config(LAYERS), d, B, max_ctx=32, seed=7)
            out["ref"] = _steps(e1, DecodeSession(e1, seed=7)).numpy()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out))
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, {"exception": repr(exc)}))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_moe_ep2_engine_matches_single_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, out = q.get(timeout=900)
        res[rank] = out
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert "exception" not in res[r], res[r]
    assert (res[0]["logits"] == res[1]["logits"]).all()
    got, ref = torch.from_numpy(res[0]["logits"]), torch.from_numpy(res[0]["ref"])
    rel = float((got - ref).norm() / ref.norm())
    assert rel < 1e-2, rel
