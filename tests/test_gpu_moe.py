"""MoE routing and combine kernels against the reference's torch ops
(Qwen3MoeSparseMoeBlock.forward, adallm/architectures/qwen3.py:1026-1032), and one MoE expert
projection end to end: route -> grouped NVFP4 GEMM -> weighted combine, against the oracle."""
import numpy as np
import pytest
import torch

from oracle import nvfp4 as nv
from adallm_b200.moe import route_topk, combine
from adallm_b200.nvfp4_gemm import nvfp4_linear_gather
from tests.gpu_util import dev, rel_l2
from tests.test_gpu_nvfp4 import random_weight

pytestmark = pytest.mark.gpu


def _torch_route(logits, k, norm):
    w = torch.softmax(logits.float(), dim=1, dtype=torch.float32)
    w, ids = torch.topk(w, k, dim=-1)
    if norm:
        w = w / w.sum(dim=-1, keepdim=True)
    return ids, w.to(logits.dtype)


@pytest.mark.parametrize("t,e,k,norm", [(16, 128, 8, True), (5, 64, 4, False), (33, 1024, 2, True), (1, 8, 8, True)])
def test_route_topk_matches_torch(t, e, k, norm):
    d = dev()
    g = torch.Generator().manual_seed(t + e)
    # distinct logits (multiples of 1/256, exact in fp16), so the top-k has no ties to order
    logits = torch.stack([(torch.randperm(e, generator=g) - e // 2).float() / 256 for _ in range(t)])
    logits = logits.to(torch.float16).to(d)
    ids, w = route_topk(logits, k, norm)
    rid, rw = _torch_route(logits, k, norm)
    torch.cuda.synchronize()
    assert torch.equal(ids.long(), rid)
    assert torch.allclose(w.float(), rw.float(), rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("t,e,k,norm", [(16, 128, 8, True), (7, 64, 4, False)])
def test_route_topk_matches_cpu_oracle(t, e, k, norm):
    """Against the CPU restatement of qwen3.py:1026-1032 (oracle.moe) on N(0, 1) bf16 logits (the
    config-4 router): identical experts in identical order, weights within one bf16 ulp."""
    from oracle.moe import route_topk as oracle_route
    d = dev()
    g = torch.Generator().manual_seed(100 + t)
    logits = torch.randn((t, e), generator=g).to(torch.bfloat16)
    ids, w = route_topk(logits.to(d), k, norm)
    rid, rw = oracle_route(logits, k, norm)
    torch.cuda.synchronize()
    assert torch.equal(ids.long().cpu(), rid)
    assert torch.allclose(w.float().cpu(), rw.float(), rtol=2 ** -8, atol=0)


def test_combine_weighted_sum():
    d = dev()
    t, k, h = 7, 8, 2048
    y = torch.randn((t * k, h), device=d, dtype=torch.bfloat16)
    w = torch.rand((t, k), device=d, dtype=torch.bfloat16)
    out = combine(y, w, k)
    ref = (y.float().view(t, k, h) * w.float().unsqueeze(-1)).sum(1)
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 4e-3


def test_combine_expert_parallel_fp32_shares():
    """Two ranks' fp32 shares (ada_moe_combine_ep_f32), summed in fp32 and rounded once, give the
    single-GPU combine up to the order of the fp32 additions: within one bf16 ulp everywhere, and
    the same bf16 value almost everywhere; the bf16 share entry agrees with the fp32 one rounded."""
    d = dev()
    t, k, h, e = 16, 8, 2048, 128
    g = torch.Generator().manual_seed(21)
    y = torch.randn((t * k, h), generator=g).to(torch.bfloat16).to(d)
    w = torch.rand((t, k), generator=g).to(torch.bfloat16).to(d)
    ids = torch.stack([torch.randperm(e, generator=g)[:k] for _ in range(t)]).to(torch.int32).to(d)
    full = combine(y, w, k)
    s0 = combine(y, w, k, expert_ids=ids, expert_base=0, num_local=e // 2, fp32=True)
    s1 = combine(y, w, k, expert_ids=ids, expert_base=e // 2, num_local=e // 2, fp32=True)
    b0 = combine(y, w, k, expert_ids=ids, expert_base=0, num_local=e // 2)
    torch.cuda.synchronize()
    assert s0.dtype == torch.float32 and torch.equal(b0, s0.to(torch.bfloat16))
    summed = (s0 + s1).to(torch.bfloat16).float()
    ulp = full.float().abs().clamp(min=2.0 ** -100).log2().floor().exp2() * 2.0 ** -7
    assert bool(((summed - full.float()).abs() <= ulp).all())
    assert float((summed == full.float()).float().mean()) > 0.99


def test_moe_projection_end_to_end():
    d = dev()
    t, e, k, hid, n = 16, 32, 4, 512, 256
    ws = [random_weight(n, hid, seed=300 + i, realistic=False) for i in range(e)]
    wp = torch.stack([torch.from_numpy(w[0]) for w in ws]).to(d)
    sc = torch.stack([torch.from_numpy(w[2]) for w in ws]).to(d)
    s2 = torch.tensor([w[3] for w in ws], dtype=torch.float32, device=d)
    g = torch.Generator().manual_seed(5)
    x = torch.randn((t, hid), generator=g).to(torch.bfloat16).to(d)
    logits = torch.randn((t, e), generator=g).to(torch.bfloat16).to(d)
    ids, w = route_topk(logits, k, True)
    h = nvfp4_linear_gather(x.repeat_interleave(k, 0), wp, sc, s2, ids.reshape(-1), 16)
    out = combine(h, w, k)
    torch.cuda.synchronize()
    xr = x.float().cpu().numpy()
    idn, wn = ids.cpu().numpy(), w.float().cpu().numpy()
    ref = np.zeros((t, n), np.float32)
    for i in range(t):
        for j in range(k):
            wt = ws[idn[i, j]]
            ref[i] += wn[i, j] * nv.linear_ref(xr[i:i + 1], wt[0], wt[2].astype(np.float32), wt[3])[0]
    assert rel_l2(out.float().cpu(), torch.from_numpy(ref)) < 1e-2


def _experts(e, n, k, seed):
    ws = [random_weight(n, k, seed=seed + i, realistic=False) for i in range(e)]
    d = dev()
    return (torch.stack([torch.from_numpy(w[0]) for w in ws]).to(d),
            torch.stack([torch.from_numpy(w[2]) for w in ws]).to(d),
            torch.tensor([w[3] for w in ws], dtype=torch.float32, device=d)), ws


def test_expert_parallel_block_sums_to_the_full_block():
    """Experts split over two emulated ranks on one GPU (the all-reduce replaced by a sum of the
    ranks' outputs): the sum equals the single-rank block, and both match the oracle (dequantised
    weights, bf16 activations, SiLU(gate) * up, routing weights)."""
    from adallm_b200.moe import expert_shard, moe_block_ep
    d = dev()
    t, e, k, hid, inter, world = 16, 16, 4, 512, 256, 2
    gu, gu_np = _experts(e, 2 * inter, hid, 700)
    dn, dn_np = _experts(e, hid, inter, 800)
    g = torch.Generator().manual_seed(11)
    x = torch.randn((t, hid), generator=g).to(torch.bfloat16).to(d)
    logits = torch.randn((t, e), generator=g).to(torch.bfloat16).to(d)
    full = moe_block_ep(x, logits, k, True, gu, dn, 0)
    parts = []
    for r in range(world):
        base, cnt = expert_shard(e, world, r)
        sl = lambda p: tuple(a[base:base + cnt] for a in p)
        parts.append(moe_block_ep(x, logits, k, True, sl(gu), sl(dn), base).float())
    torch.cuda.synchronize()
    summed = parts[0] + parts[1]
    assert torch.isfinite(summed).all()
    assert rel_l2(summed.cpu(), full.float().cpu()) < 1e-2
    ids, w = route_topk(logits, k, True)
    ids, w = ids.cpu().numpy(), w.float().cpu().numpy()
    xr = x.float().cpu().numpy()
    ref = np.zeros((t, hid), np.float32)
    for i in range(t):
        for j in range(k):
            ex = int(ids[i, j])
            a = gu_np[ex]
            h = nv.linear_ref(xr[i:i + 1], a[0], a[2].astype(np.float32), a[3])
            gate, up = h[:, :inter], h[:, inter:]
            act = (gate / (1 + np.exp(-gate)) * up).astype(np.float32)
            act = torch.from_numpy(act).to(torch.bfloat16).float().numpy()
            b = dn_np[ex]
            ref[i] += w[i, j] * nv.linear_ref(act, b[0], b[2].astype(np.float32), b[3])[0]
    assert rel_l2(summed.cpu(), torch.from_numpy(ref)) < 2e-2
    assert rel_l2(full.float().cpu(), torch.from_numpy(ref)) < 2e-2
