"""FP8 paged decode and prefix-cache prefill attention + FP8 KV-cache store oracle.
Test infrastructure only.

Reference anchors (paths inside the reference project):
  * store_kvcache_kernel / store_kvcache   adallm/ops/attention.py:11-31, :236-251
  * fp8_kv_decode_group_kernel             adallm/ops/attention.py:126-233
  * _gather_kv_from_blocks                 adallm/ops/attention.py:254-286
  * decode launch (q -> fp16, out fp16)    adallm/ops/attention.py:314-324, :359-414
  * slot = page_id * page + offset         adallm/runtime/model_runner.py:262-267, :291
  * prefix-cache prefill                   adallm/ops/attention.py:335-358 (gather, then
                                           flash_attn_varlen_func causal, window (W, 0));
                                           metadata from model_runner.py:240-276

Cache layout (reference): k_cache / v_cache are e4m3fn [num_pages, page, Hkv, D];
block_tables int32 [B, max_pages] padded with -1; context_lens int32 [B]
counts the current token.  Token t of sequence b sits in page
block_tables[b, t // page], row t % page.
"""
from __future__ import annotations

import numpy as np
import torch

from .nvfp4 import e4m3_decode, e4m3_encode


def store_kvcache(key, value, k_cache_bits, v_cache_bits, slot_mapping, k_scale=1.0, v_scale=1.0):
    """In-place e4m3 store of key/value rows (attention.py:11-31 / :236-251).

    key, value: float arrays [T, Hkv, D] holding bf16 values.
    k_cache_bits, v_cache_bits: uint8 [num_pages, page, Hkv, D] (modified).
    Slots equal to -1 are skipped.  The reference has no KV scale (1.0)."""
    key = np.asarray(key, np.float32)
    value = np.asarray(value, np.float32)
    t, hkv, d = key.shape
    kc = k_cache_bits.reshape(-1, hkv * d)
    vc = v_cache_bits.reshape(-1, hkv * d)
    for i in range(t):
        slot = int(slot_mapping[i])
        if slot == -1:
            continue
        kc[slot] = e4m3_encode((key[i].reshape(-1) / np.float32(k_scale)).astype(np.float32))
        vc[slot] = e4m3_encode((value[i].reshape(-1) / np.float32(v_scale)).astype(np.float32))


def gather_kv_from_blocks(k_cache: np.ndarray, v_cache: np.ndarray, block_tables, context_lens):
    """Restates attention.py:254-286: concatenate each sequence's first ctx
    tokens (decoded cache values) -> ([total, Hkv, D], [total, Hkv, D], cu_seqlens)."""
    page = k_cache.shape[1]
    ks, vs, cu = [], [], [0]
    for i in range(block_tables.shape[0]):
        ctx = int(context_lens[i])
        if ctx == 0:
            cu.append(cu[-1])
            continue
        nb = (ctx + page - 1) // page
        blocks = np.asarray(block_tables[i, :nb], np.int64)
        ks.append(k_cache[blocks].reshape(nb * page, *k_cache.shape[2:])[:ctx])
        vs.append(v_cache[blocks].reshape(nb * page, *v_cache.shape[2:])[:ctx])
        cu.append(cu[-1] + ctx)
    hkv, d = k_cache.shape[2], k_cache.shape[3]
    k_out = np.concatenate(ks) if ks else np.zeros((0, hkv, d), k_cache.dtype)
    v_out = np.concatenate(vs) if vs else np.zeros((0, hkv, d), v_cache.dtype)
    return k_out, v_out, np.asarray(cu, np.int32)


def paged_decode(q, k_cache_bits, v_cache_bits, block_tables, context_lens, scale,
                 window: int = 0, k_scale: float = 1.0, v_scale: float = 1.0):
    """Decode attention for one query token per sequence (attention.py:126-233).

    q: [B, Hq, D] (bf16 values as fp32; rounded to fp16 as the reference does
    at attention.py:314-324).  Pages whose block id is negative are masked
    like the reference kernel's ``block_id >= 0`` test.  A zero-length
    sequence yields zeros.  Returns fp32 [B, Hq, D]."""
    q = torch.as_tensor(np.asarray(q, np.float32)).to(torch.float16).to(torch.float64)
    page = k_cache_bits.shape[1]
    hkv = k_cache_bits.shape[2]
    b, hq, d = q.shape
    group = hq // hkv
    out = torch.zeros((b, hq, d), dtype=torch.float64)
    bt = np.asarray(block_tables)
    head_map = torch.arange(hq) // group
    for i in range(b):
        ctx = int(context_lens[i])
        if ctx == 0:
            continue
        start = max(ctx - window, 0) if window > 0 else 0
        toks = np.arange(start, ctx)
        pages = bt[i, toks // page]
        valid = pages >= 0
        toks, pages = toks[valid], pages[valid]
        if toks.size == 0:
            continue
        # decode only the cache rows this sequence reads (e4m3 -> value is elementwise)
        kf = torch.from_numpy(e4m3_decode(k_cache_bits[pages, toks % page])).to(torch.float64) * float(k_scale)
        vf = torch.from_numpy(e4m3_decode(v_cache_bits[pages, toks % page])).to(torch.float64) * float(v_scale)
        kk = kf[:, head_map]  # [n, Hq, D] (GQA repeat)
        vv = vf[:, head_map]
        s = torch.einsum("nhd,hd->nh", kk, q[i]) * float(scale)
        p = torch.softmax(s, dim=0)
        out[i] = torch.einsum("nh,nhd->hd", p, vv)
    return out.to(torch.float32).numpy()


def paged_decode_fp16_kernel(q, k_cache_bits, v_cache_bits, block_tables, context_lens, scale,
                             window: int = 0, block_t: int = 64):
    """The reference decode kernel's own arithmetic (fp8_kv_decode_group_kernel,
    adallm/ops/attention.py:165-233), for measuring how far the reference itself sits from the
    fp64 softmax of paged_decode: q rounded to fp16; e4m3 K/V widened to fp16 (exact); per tile
    of block_t consecutive tokens (aligned, as the kernel walks a page in BLOCK_T = 64 steps) the
    fp32 scores q.k * scale, an online softmax in fp32 whose probabilities are rounded to fp16
    before the P.V product (fp32 accumulation), and the output acc / l rounded to fp16
    (:229-233).  Masked tokens (past ctx, before the window start, pages < 0) are -inf.
    Returns fp32 [B, Hq, D] holding fp16 values."""
    q = torch.as_tensor(np.asarray(q, np.float32)).to(torch.float16).to(torch.float32)
    page = k_cache_bits.shape[1]
    hkv = k_cache_bits.shape[2]
    b, hq, d = q.shape
    group = hq // hkv
    out = torch.zeros((b, hq, d), dtype=torch.float32)
    bt = np.asarray(block_tables)
    head_map = torch.arange(hq) // group
    for i in range(b):
        ctx = int(context_lens[i])
        if ctx == 0:
            continue
        start = max(ctx - window, 0) if window > 0 else 0
        m = torch.full((hq,), -float("inf"))
        l = torch.zeros(hq)
        acc = torch.zeros((hq, d))
        for t0 in range((start // block_t) * block_t, ctx, block_t):
            toks = np.arange(t0, min(t0 + block_t, ctx))
            toks = toks[toks >= start]
            pages = bt[i, toks // page]
            valid = pages >= 0
            toks, pages = toks[valid], pages[valid]
            if toks.size == 0:
                continue
            kk = torch.from_numpy(e4m3_decode(k_cache_bits[pages, toks % page])).float()[:, head_map]  # [n, Hq, D]
            vv = torch.from_numpy(e4m3_decode(v_cache_bits[pages, toks % page])).float()[:, head_map]
            s = torch.einsum("nhd,hd->hn", kk, q[i]) * float(scale)
            m_new = torch.maximum(m, s.max(dim=1).values)
            e = torch.exp(s - m_new[:, None])
            alpha = torch.exp(m - m_new)
            l = l * alpha + e.sum(dim=1)
            acc = acc * alpha[:, None] + torch.einsum("hn,nhd->hd", e.to(torch.float16).float(), vv)
            m = m_new
        out[i] = (acc / l[:, None]).to(torch.float16).float()
    return out.numpy()


def paged_prefill(q, k_cache_bits, v_cache_bits, block_tables, cu_seqlens_q, cu_seqlens_k, scale,
                  window: int = 0, k_scale: float = 1.0, v_scale: float = 1.0):
    """Prefix-cache prefill attention (attention.py:335-358).

    The reference gathers each sequence's first len_k = cu_seqlens_k[b+1] - cu_seqlens_k[b]
    cached tokens to fp16 (_gather_kv_from_blocks, :254-286; e4m3 -> fp16 is exact) and calls
    flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, causal=True,
    window_size=(W, 0)).  flash-attn's published masking for varlen causal attention aligns
    the mask to the bottom right: query i of the len_q new tokens sees key j iff
    j <= i + len_k - len_q, and with W > 0 also j >= i + len_k - len_q - W.  A row that sees
    no key is zero.  Keys on a page whose block id is outside [0, num_pages) are masked (the
    reference would fail on such a table; the kernel treats it like the decode path does).

    q: [total_q, Hq, D] float (bf16 values), rounded to fp16 as the reference does
    (:319-324).  Returns fp32 [total_q, Hq, D]."""
    q = torch.as_tensor(np.asarray(q, np.float32)).to(torch.float16).to(torch.float64)
    kf = torch.from_numpy(e4m3_decode(k_cache_bits)).to(torch.float64) * float(k_scale)
    vf = torch.from_numpy(e4m3_decode(v_cache_bits)).to(torch.float64) * float(v_scale)
    num_pages, page, hkv = k_cache_bits.shape[0], k_cache_bits.shape[1], k_cache_bits.shape[2]
    total_q, hq, d = q.shape
    group = hq // hkv
    head_map = torch.arange(hq) // group
    out = torch.zeros((total_q, hq, d), dtype=torch.float64)
    bt = np.asarray(block_tables)
    cu_q = np.asarray(cu_seqlens_q, np.int64)
    cu_k = np.asarray(cu_seqlens_k, np.int64)
    for b in range(len(cu_q) - 1):
        q0, len_q = int(cu_q[b]), int(cu_q[b + 1] - cu_q[b])
        len_k = int(cu_k[b + 1] - cu_k[b])
        if len_q <= 0 or len_k <= 0:
            continue
        keys = np.arange(len_k)
        keys = keys[keys < bt.shape[1] * page]
        pages = bt[b, keys // page].astype(np.int64)
        ok = (pages >= 0) & (pages < num_pages)
        pi = torch.from_numpy(np.where(ok, pages, 0))
        ti = torch.from_numpy(keys % page)
        kk = kf[pi, ti][:, head_map]  # [n, Hq, D]
        vv = vf[pi, ti][:, head_map]
        vv[torch.from_numpy(~ok)] = 0.0
        off = len_k - len_q
        i = torch.arange(len_q)[:, None]
        j = torch.from_numpy(keys)[None, :]
        vis = (j <= i + off) & torch.from_numpy(ok)[None, :]
        if window > 0:
            vis &= j >= i + off - window
        s = torch.einsum("qhd,khd->hqk", q[q0:q0 + len_q], kk) * float(scale)
        s = s.masked_fill(~vis[None], float("-inf"))
        p = torch.softmax(s, dim=-1)
        p = torch.nan_to_num(p, nan=0.0)  # rows with no visible key
        out[q0:q0 + len_q] = torch.einsum("hqk,khd->qhd", p, vv)
    return out.to(torch.float32).numpy()


def make_prefill_case(seed: int, cached: list, new: list, hq: int, hkv: int, d: int, page: int,
                      extra_pages: int = 0, holes: int = 0):
    """Seeded prefix-cache prefill case: sequence b has cached[b] tokens already in the cache
    and new[b] new query tokens (all len_k = cached + new tokens stored, as store_kvcache does
    before attention); pages from a random permutation of a pool with `extra_pages` unused
    pages; `holes` random table entries inside the used range set to -1.  K, V ~ N(0,1) cast
    to e4m3, q ~ N(0,1) bf16."""
    g = torch.Generator().manual_seed(seed)
    len_k = np.asarray([c + n for c, n in zip(cached, new)], np.int64)
    npages = (len_k + page - 1) // page
    pool = int(npages.sum()) + extra_pages
    perm = torch.randperm(max(pool, 1), generator=g).numpy().astype(np.int32)
    max_pages = max(int(npages.max()) if len(npages) else 1, 1)
    bt = -np.ones((len(new), max_pages), np.int32)
    o = 0
    for b in range(len(new)):
        bt[b, :npages[b]] = perm[o:o + npages[b]]
        o += int(npages[b])
    for _ in range(holes):
        b = int(torch.randint(0, len(new), (1,), generator=g))
        if npages[b]:
            bt[b, int(torch.randint(0, int(npages[b]), (1,), generator=g))] = -1
    kbits = e4m3_encode(torch.randn((max(pool, 1), page, hkv, d), generator=g).numpy())
    vbits = e4m3_encode(torch.randn((max(pool, 1), page, hkv, d), generator=g).numpy())
    cu_q = np.concatenate([[0], np.cumsum(new)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(len_k)]).astype(np.int32)
    q = torch.randn((int(cu_q[-1]), hq, d), generator=g).to(torch.bfloat16).to(torch.float32).numpy()
    return dict(q=q, k=kbits, v=vbits, block_tables=bt, cu_q=cu_q, cu_k=cu_k,
                max_seqlen_q=int(max(new)) if len(new) else 0, scale=1.0 / np.sqrt(d))


def make_paged_case(seed: int, batch: int, hq: int, hkv: int, d: int, page: int,
                    ctx_lo: int, ctx_hi: int, extra_cols: int = 0, k_scale: float = 1.0,
                    v_scale: float = 1.0):
    """Seeded synthetic decode-attention case (BASELINE config 1 generator):
    context lengths ~ U{ctx_lo..ctx_hi}; a pool of exactly sum(pages) pages is
    assigned by a random permutation; the table is padded with -1; K, V ~
    N(0,1) cast to e4m3 (after division by the per-tensor scale); q ~ N(0,1) bf16."""
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(ctx_lo, ctx_hi + 1, (batch,), generator=g).numpy().astype(np.int32)
    npages = (ctx + page - 1) // page
    pool = int(npages.sum())
    perm = torch.randperm(max(pool, 1), generator=g).numpy().astype(np.int32)
    max_pages = int(npages.max()) + extra_cols if batch else 1
    bt = -np.ones((batch, max(max_pages, 1)), np.int32)
    off = 0
    for i in range(batch):
        bt[i, : npages[i]] = perm[off: off + npages[i]]
        off += npages[i]
    kf = torch.randn((max(pool, 1), page, hkv, d), generator=g)
    vf = torch.randn((max(pool, 1), page, hkv, d), generator=g)
    kbits = e4m3_encode((kf / k_scale).numpy())
    vbits = e4m3_encode((vf / v_scale).numpy())
    q = torch.randn((batch, hq, d), generator=g).to(torch.bfloat16).to(torch.float32).numpy()
    return dict(q=q, k=kbits, v=vbits, block_tables=bt, context_lens=ctx,
                scale=1.0 / np.sqrt(d), k_scale=k_scale, v_scale=v_scale)
