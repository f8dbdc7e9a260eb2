"""FP8 paged decode attention: CUDA kernel (through the C ABI) vs the CPU oracle
(restating adallm/ops/attention.py:126-233 with an exact fp64 softmax).
Tolerance: rel-L2 <= 1e-2 in bf16; typical ~1e-3."""
import numpy as np
import pytest
import torch

from oracle import attention as oa
from adallm_b200.attention import paged_decode, Attention
from adallm_b200.context import set_context, reset_context
from tests.gpu_util import dev, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _run(case, window=0, dtype=torch.bfloat16, page=None):
    d = dev()
    q = torch.from_numpy(case["q"]).to(dtype).to(d)
    k = torch.from_numpy(case["k"]).to(d).view(torch.float8_e4m3fn)
    v = torch.from_numpy(case["v"]).to(d).view(torch.float8_e4m3fn)
    bt = torch.from_numpy(case["block_tables"]).to(d)
    ctx = torch.from_numpy(case["context_lens"]).to(d)
    out = paged_decode(q, k, v, bt, ctx, case["scale"], window, case["k_scale"], case["v_scale"])
    torch.cuda.synchronize()
    ref = oa.paged_decode(q.float().cpu().numpy(), case["k"], case["v"], case["block_tables"],
                          case["context_lens"], case["scale"], window, case["k_scale"], case["v_scale"])
    return out.float().cpu(), torch.from_numpy(ref)


@pytest.mark.parametrize("seed", [0, 1])
def test_config1_shape(seed):
    # B16, Hq32/Hkv8, D128, page 16, ctx U[512, 8192]
    case = oa.make_paged_case(seed, batch=16, hq=32, hkv=8, d=128, page=16, ctx_lo=512, ctx_hi=8192)
    out, ref = _run(case)
    assert rel_l2(out, ref) < TOL


@pytest.mark.parametrize("page", [16, 32, 256])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (32, 16), (32, 4), (8, 8)])
def test_pages_and_groups(page, hq, hkv):
    case = oa.make_paged_case(7, batch=5, hq=hq, hkv=hkv, d=128, page=page, ctx_lo=1, ctx_hi=700, extra_cols=3)
    out, ref = _run(case)
    assert rel_l2(out, ref) < TOL


@pytest.mark.parametrize("window", [1, 17, 1024])
@pytest.mark.parametrize("hkv,ctx_hi", [(16, 3000), (8, 1000)])  # split-K path / short-cache one-cluster path
def test_sliding_window(window, hkv, ctx_hi):
    case = oa.make_paged_case(11, batch=6, hq=32, hkv=hkv, d=128, page=16, ctx_lo=1, ctx_hi=ctx_hi)
    out, ref = _run(case, window=window)
    assert rel_l2(out, ref) < TOL


def test_kv_scales_and_fp16_query():
    case = oa.make_paged_case(5, batch=4, hq=32, hkv=8, d=128, page=16, ctx_lo=100, ctx_hi=900,
                              k_scale=0.25, v_scale=2.0)
    out, ref = _run(case, dtype=torch.float16)
    assert rel_l2(out, ref) < TOL


def test_edge_lengths_and_padding():
    # ctx 0 -> zeros; ctx 1, 16, 17, 256, 257 cross tile / split boundaries
    case = oa.make_paged_case(2, batch=7, hq=32, hkv=8, d=128, page=16, ctx_lo=1, ctx_hi=2, extra_cols=20)
    lens = np.array([0, 1, 16, 17, 256, 257, 300], np.int32)
    npages = (lens + 15) // 16
    pool = case["k"].shape[0]
    rng = np.random.default_rng(0)
    need = int(npages.sum())
    kk = rng.standard_normal((need, 16, 8, 128)).astype(np.float32)
    from oracle.nvfp4 import e4m3_encode
    case["k"] = e4m3_encode(kk)
    case["v"] = e4m3_encode(rng.standard_normal((need, 16, 8, 128)).astype(np.float32))
    perm = rng.permutation(need).astype(np.int32)
    bt = -np.ones((7, 25), np.int32)
    off = 0
    for i, n in enumerate(npages):
        bt[i, :n] = perm[off:off + n]
        off += n
    case["block_tables"], case["context_lens"] = bt, lens
    del pool
    out, ref = _run(case)
    assert torch.all(out[0] == 0)
    assert rel_l2(out[1:], ref[1:]) < TOL


def test_negative_block_ids_are_masked():
    case = oa.make_paged_case(9, batch=3, hq=8, hkv=2, d=128, page=16, ctx_lo=64, ctx_hi=64)
    case["block_tables"][1, 1] = -1  # a hole inside the context: the reference kernel masks it
    out, ref = _run(case)
    assert rel_l2(out, ref) < TOL


def test_attention_module_decode_branch():
    d = dev()
    case = oa.make_paged_case(4, batch=4, hq=32, hkv=8, d=128, page=16, ctx_lo=40, ctx_hi=200)
    attn = Attention(32, 128, case["scale"], 8)
    k = torch.from_numpy(case["k"]).to(d).view(torch.float8_e4m3fn)
    v = torch.from_numpy(case["v"]).to(d).view(torch.float8_e4m3fn)
    attn.k_cache, attn.v_cache = k, v
    ctx = torch.from_numpy(case["context_lens"]).to(d)
    bt = torch.from_numpy(case["block_tables"]).to(d)
    # the new token of each sequence goes to its last position (slot = page*16 + off)
    last = case["context_lens"] - 1
    slots = np.array([case["block_tables"][i, last[i] // 16] * 16 + last[i] % 16 for i in range(4)], np.int32)
    q = torch.randn(4, 32 * 128, device=d, dtype=torch.bfloat16)
    kn = torch.randn(4, 8, 128, device=d, dtype=torch.bfloat16)
    vn = torch.randn(4, 8, 128, device=d, dtype=torch.bfloat16)
    set_context(False, slot_mapping=torch.from_numpy(slots).to(d), context_lens=ctx, block_tables=bt)
    try:
        out = attn(q.view(4, 32, 128), kn, vn)
    finally:
        reset_context()
    torch.cuda.synchronize()
    kb = k.view(torch.uint8).cpu().numpy()
    vb = v.view(torch.uint8).cpu().numpy()
    ref = oa.paged_decode(q.view(4, 32, 128).float().cpu().numpy(), kb, vb, case["block_tables"],
                          case["context_lens"], case["scale"])
    assert rel_l2(out.float().cpu(), torch.from_numpy(ref)) < TOL
