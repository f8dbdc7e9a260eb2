"""Causal prefill attention over the FP8 paged cache (ada_fp8_paged_prefill) against the oracle.

The oracle restates the reference's prefix-cache prefill (attention.py:335-358: gather the
e4m3 pages to fp16, then flash-attn varlen with a bottom-right causal mask and window (W, 0)).
Tolerance: 1e-2 relative L2 (bf16/fp16 output; fp16 probabilities in P.V), as for decode.
Size-independent checks at a long context: a prefill split into a cached prefix and a new
chunk gives bit-identical rows to the unsplit prefill, and sampled rows equal the decode
oracle for a context ending at that row's position."""
import numpy as np
import pytest
import torch

from adallm_b200.attention import paged_prefill
from oracle.attention import make_prefill_case, paged_decode, paged_prefill as ref_prefill
from tests.gpu_util import dev, rel_l2

pytestmark = pytest.mark.gpu


def _run(c, window=0, k_scale=1.0, v_scale=1.0, dtype=torch.bfloat16, out_dtype=None, cu_k=None):
    d = dev()
    q = torch.from_numpy(c["q"]).to(dtype).to(d)
    kc = torch.from_numpy(c["k"]).to(d).view(torch.float8_e4m3fn)
    vc = torch.from_numpy(c["v"]).to(d).view(torch.float8_e4m3fn)
    bt = torch.from_numpy(c["block_tables"]).to(d)
    cu_q = torch.from_numpy(c["cu_q"]).to(d)
    cu_k = torch.from_numpy(cu_k if cu_k is not None else c["cu_k"]).to(d)
    err = torch.zeros(1, dtype=torch.int32, device=d)
    out = None
    if out_dtype is not None:
        out = torch.empty(q.shape, dtype=out_dtype, device=d)
    o = paged_prefill(q, kc, vc, bt, cu_q, cu_k, c["max_seqlen_q"], c["scale"], window, k_scale, v_scale,
                      out=out, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return o


CASES = [
    # cached, new, hq, hkv, page, window, holes
    ([0, 37, 300, 5], [50, 1, 129, 0], 32, 8, 16, 0, 0),
    ([0, 37, 300, 5], [50, 1, 129, 0], 32, 8, 16, 40, 0),
    ([100, 0], [77, 200], 32, 4, 64, 0, 0),
    ([15], [70], 12, 4, 32, 0, 0),
    ([3], [130], 4, 4, 16, 17, 0),
    ([64, 200, 31], [16, 90, 33], 16, 8, 16, 0, 3),
    ([1024], [512], 32, 8, 16, 0, 0),
]


@pytest.mark.parametrize("cached,new,hq,hkv,page,window,holes", CASES)
def test_prefill_matches_oracle(cached, new, hq, hkv, page, window, holes):
    """Prefix and no prefix, single new token, empty sequence, sliding window, GQA groups
    1 / 3 (a padded row block) / 4 / 8, pages 16-64, holes in the block table."""
    c = make_prefill_case(len(cached) + hq + page, cached, new, hq, hkv, 128, page, extra_pages=4, holes=holes)
    o = _run(c, window)
    ref = ref_prefill(c["q"], c["k"], c["v"], c["block_tables"], c["cu_q"], c["cu_k"], c["scale"], window)
    assert o.dtype == torch.bfloat16
    assert torch.isfinite(o).all()
    assert rel_l2(o.float().cpu(), torch.from_numpy(ref)) < 1e-2


def test_prefill_fp16_scales_and_strided_out():
    """fp16 q and output written into a strided view; per-tensor k / v scales."""
    c = make_prefill_case(5, [40, 0], [33, 70], 32, 8, 128, 16)
    d = dev()
    q = torch.from_numpy(c["q"]).to(torch.float16).to(d)
    wide = torch.zeros((q.shape[0], 40, 128), dtype=torch.float16, device=d)
    out = wide[:, 4:36]
    kc = torch.from_numpy(c["k"]).to(d).view(torch.float8_e4m3fn)
    vc = torch.from_numpy(c["v"]).to(d).view(torch.float8_e4m3fn)
    o = paged_prefill(q, kc, vc, torch.from_numpy(c["block_tables"]).to(d), torch.from_numpy(c["cu_q"]).to(d),
                      torch.from_numpy(c["cu_k"]).to(d), c["max_seqlen_q"], c["scale"], 0, 0.5, 2.0, out=out)
    torch.cuda.synchronize()
    assert o.data_ptr() == out.data_ptr()
    ref = ref_prefill(c["q"], c["k"], c["v"], c["block_tables"], c["cu_q"], c["cu_k"], c["scale"], 0, 0.5, 2.0)
    assert rel_l2(out.float().cpu(), torch.from_numpy(ref)) < 1e-2
    assert (wide[:, :4] == 0).all() and (wide[:, 36:] == 0).all()


def test_prefill_rows_without_keys_are_zero():
    """len_k < len_q: the first len_q - len_k rows see no key (bottom-right causal mask)."""
    c = make_prefill_case(9, [0, 10], [50, 20], 32, 8, 128, 16)
    cu_k = c["cu_k"].copy()
    cu_k[1] = 40  # sequence 0: 40 keys for 50 queries
    cu_k[2] = cu_k[1] + 30
    o = _run(c, cu_k=cu_k)
    ref = ref_prefill(c["q"], c["k"], c["v"], c["block_tables"], c["cu_q"], cu_k, c["scale"])
    assert (o[:10].float() == 0).all()
    assert rel_l2(o.float().cpu(), torch.from_numpy(ref)) < 1e-2


@pytest.mark.parametrize("window", [0, 300])
def test_long_prefill_chunked_is_bit_identical_and_rows_match_decode(window):
    """8192-token prefill (Qwen3-8B heads): the last 1024 rows computed with the first 7168
    tokens as a cached prefix are bit-identical to the same rows of the whole prefill; eight
    sampled rows equal the decode oracle with the context ending at that row (window W covers
    W + 1 keys here, W + 1 in the decode convention)."""
    L, chunk = 8192, 1024
    c = make_prefill_case(11, [0], [L], 32, 8, 128, 16)
    full = _run(c, window)
    c2 = dict(c)
    c2["q"] = c["q"][L - chunk:]
    c2["cu_q"] = np.asarray([0, chunk], np.int32)
    c2["max_seqlen_q"] = chunk
    part = _run(c2, window)
    assert torch.equal(full[L - chunk:], part)
    rows = [0, 1, 15, 16, 777, 4095, 7000, L - 1]
    ctx = np.asarray([r + 1 for r in rows], np.int32)
    bt = np.repeat(c["block_tables"], len(rows), axis=0)
    ref = paged_decode(c["q"][rows], c["k"], c["v"], bt, ctx, c["scale"], window + 1 if window else 0)
    assert rel_l2(full[rows].float().cpu(), torch.from_numpy(ref)) < 1e-2


def test_attention_module_prefix_prefill():
    """Attention.forward in a prefix-cache prefill context: stores the new K/V rows into the
    e4m3 cache, then attends over cached prefix + new rows (the reference's prefill branch)."""
    from adallm_b200.attention import Attention
    from adallm_b200.context import reset_context, set_context
    from oracle.attention import store_kvcache as ref_store
    d = dev()
    hq, hkv, page, cached, new = 32, 8, 16, [20, 0], [30, 17]
    c = make_prefill_case(21, cached, new, hq, hkv, 128, page)
    g = torch.Generator().manual_seed(5)
    k_new = torch.randn((sum(new), hkv, 128), generator=g).to(torch.bfloat16)
    v_new = torch.randn((sum(new), hkv, 128), generator=g).to(torch.bfloat16)
    slots = []
    for b in range(len(new)):
        for t in range(cached[b], cached[b] + new[b]):
            slots.append(int(c["block_tables"][b, t // page]) * page + t % page)
    slots = np.asarray(slots, np.int32)
    kb, vb = c["k"].copy(), c["v"].copy()
    ref_store(k_new.float().numpy(), v_new.float().numpy(), kb, vb, slots)
    ref = ref_prefill(c["q"], kb, vb, c["block_tables"], c["cu_q"], c["cu_k"], c["scale"])

    m = Attention(hq, 128, float(c["scale"]), hkv)
    m.k_cache = torch.from_numpy(c["k"]).to(d).view(torch.float8_e4m3fn)
    m.v_cache = torch.from_numpy(c["v"]).to(d).view(torch.float8_e4m3fn)
    try:
        set_context(True, torch.from_numpy(c["cu_q"]).to(d), torch.from_numpy(c["cu_k"]).to(d), c["max_seqlen_q"],
                    int(np.diff(c["cu_k"]).max()), torch.from_numpy(slots).to(d), None,
                    torch.from_numpy(c["block_tables"]).to(d))
        o = m.forward(torch.from_numpy(c["q"]).to(torch.bfloat16).to(d).view(sum(new), hq * 128), k_new.to(d),
                      v_new.to(d))
        torch.cuda.synchronize()
    finally:
        reset_context()
    assert torch.equal(m.k_cache.view(torch.uint8).cpu(), torch.from_numpy(kb))
    assert rel_l2(o.float().cpu(), torch.from_numpy(ref)) < 1e-2
