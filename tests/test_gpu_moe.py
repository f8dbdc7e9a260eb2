"""MoE routing and combine kernels against the reference's torch ops
(Qwen3MoeSparseMoeBlock.forward, adallm/architectures/qwen3.py:1026-1032), and one MoE expert
projection end to end: route -> grouped NVFP4 GEMM -> weighted combine, against the oracle."""
import numpy as np
import pytest
import torch

from oracle import nvfp4 as nv
from adallm_b200 import _native as N
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


@pytest.mark.parametrize("t,e,k,hid,inter,base,cnt,terms", [(16, 32, 8, 2048, 768, 0, 32, 4),
                                                            (16, 32, 8, 2048, 768, 16, 16, 4),
                                                            (5, 8, 2, 512, 256, 0, 8, 1)])
def test_moe_experts_matches_the_grouped_pipeline(t, e, k, hid, inter, base, cnt, terms):
    """ada_moe_experts (one routing, the gather folded into the quantiser, SiLU*up quantised
    straight into the down operand) against the unfused pipeline -- row gather, grouped gate_up,
    SiLU*up, grouped down, each through its own entry point: bit-identical rows for the experts
    held ([base, base + cnt)), other rows untouched, no error."""
    from adallm_b200.activation import gated_act
    d = dev()
    gu, _ = _experts(cnt, 2 * inter, hid, 900 + base)
    dn, _ = _experts(cnt, hid, inter, 950 + base)
    g = torch.Generator().manual_seed(t + e)
    x = torch.randn((t, hid), generator=g).to(torch.bfloat16).to(d)
    ids = torch.stack([torch.randperm(e, generator=g)[:k] for _ in range(t)]).to(torch.int32).to(d)
    flat = ids.reshape(-1)
    h = nvfp4_linear_gather(x.repeat_interleave(k, 0), gu[0], gu[1], gu[2], flat, 16, expert_base=base, terms=terms)
    a = gated_act(h, 0)
    y_ref = nvfp4_linear_gather(a, dn[0], dn[1], dn[2], flat, 16, expert_base=base, terms=terms)
    from adallm_b200.nvfp4_gemm import prepack_scales
    sf_gu = prepack_scales(gu[1].reshape(cnt * 2 * inter, hid // 16), cnt * 2 * inter, hid)
    sf_dn = prepack_scales(dn[1].reshape(cnt * hid, inter // 16), cnt * hid, inter)
    lib = N.lib()
    ws = torch.zeros(int(lib.ada_moe_experts_workspace_size(t, k, hid, inter, terms, cnt)), dtype=torch.uint8, device=d)
    y = torch.full((t * k, hid), 7.0, dtype=torch.bfloat16, device=d)
    st = lib.ada_moe_experts(x.data_ptr(), 0, x.stride(0), t, k, flat.data_ptr(), cnt, base, int(cnt == e),
                             gu[0].data_ptr(), gu[0].stride(1), sf_gu.data_ptr(), gu[2].data_ptr(), dn[0].data_ptr(),
                             dn[0].stride(1), sf_dn.data_ptr(), dn[2].data_ptr(), inter, hid, 0, y.data_ptr(),
                             y.stride(0), terms, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    N.check(st, "moe experts")
    torch.cuda.synchronize()
    local = ((flat >= base) & (flat < base + cnt)).cpu()
    assert int(ws[:4].view(torch.int32).item()) == 0
    assert torch.equal(y.cpu()[local], y_ref.cpu()[local])
    assert bool((y.cpu()[~local] == 7.0).all())


def _router_case(t, e, h, seed, exact):
    g = torch.Generator().manual_seed(seed)
    if exact:  # small integers times powers of two: every product and sum is exact in fp32 and bf16
        x = torch.randint(-2, 3, (t, h), generator=g).float() * 0.25
        w = torch.randint(-2, 3, (e, h), generator=g).float() * 0.125
    else:  # the config-4 router: N(0, 1/H) weights, so logits ~ N(0, 1)
        x = torch.randn((t, h), generator=g)
        w = torch.randn((e, h), generator=g) * h ** -0.5
    return x.to(torch.bfloat16), w.to(torch.bfloat16)


@pytest.mark.parametrize("t,e,h,k,norm", [(16, 128, 2048, 8, True), (5, 64, 512, 4, False), (3, 256, 1024, 8, True),
                                          (2, 24, 256, 2, True)])
def test_router_topk_fused_exact(t, e, h, k, norm):
    """The fused router GEMM + routing on exactly representable inputs: identical experts, order
    and weights to ada_moe_route_topk over the exact logits (rounded to bf16, as F.linear)."""
    d = dev()
    x, w = _router_case(t, e, h, 31 + t, exact=True)
    logits = (x.double() @ w.double().t()).to(torch.bfloat16)
    rid, rw = route_topk(logits.to(d), k, norm)
    ids = torch.empty((t, k), dtype=torch.int32, device=d)
    wts = torch.empty((t, k), dtype=torch.bfloat16, device=d)
    err = torch.zeros(1, dtype=torch.int32, device=d)
    xd, wd = x.to(d), w.to(d)
    N.check(N.lib().ada_moe_router_topk(xd.data_ptr(), 0, h, t, wd.data_ptr(), h, h, e, k, int(norm), ids.data_ptr(),
                                        wts.data_ptr(), err.data_ptr(), torch.cuda.current_stream().cuda_stream),
            "router")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(ids.long(), rid.long().view(t, k))
    assert torch.equal(wts, rw.view(t, k))


def test_router_topk_fused_config4():
    """N(0, 1) router logits (config 4): the fused kernel's fp32 sums differ from an fp64 product
    only in order, so its routing equals the routing of the fp64 logits rounded to bf16 except
    where two logits sit within one bf16 rounding of each other."""
    d = dev()
    t, e, h, k = 16, 128, 2048, 8
    x, w = _router_case(t, e, h, 5, exact=False)
    logits = (x.double() @ w.double().t()).to(torch.bfloat16)
    rid, rw = route_topk(logits.to(d), k, True)
    ids = torch.empty((t, k), dtype=torch.int32, device=d)
    wts = torch.empty((t, k), dtype=torch.bfloat16, device=d)
    err = torch.zeros(1, dtype=torch.int32, device=d)
    xd, wd = x.to(d), w.to(d)
    N.check(N.lib().ada_moe_router_topk(xd.data_ptr(), 0, h, t, wd.data_ptr(), h, h, e, k, 1, ids.data_ptr(),
                                        wts.data_ptr(), err.data_ptr(), torch.cuda.current_stream().cuda_stream),
            "router")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    same = (ids.long() == rid.long().view(t, k)).float().mean().item()
    assert same >= 0.97, same
    assert torch.allclose(wts.float(), rw.view(t, k).float(), atol=2e-2)
