"""FP8 paged decode attention + FP8 KV-cache store oracle.  Test infrastructure only.

Reference anchors (paths inside the reference project):
  * store_kvcache_kernel / store_kvcache   adallm/ops/attention.py:11-31, :236-251
  * fp8_kv_decode_group_kernel             adallm/ops/attention.py:126-233
  * _gather_kv_from_blocks                 adallm/ops/attention.py:254-286
  * decode launch (q -> fp16, out fp16)    adallm/ops/attention.py:314-324, :359-414
  * slot = page_id * page + offset         adallm/runtime/model_runner.py:262-267, :291

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
    kf = torch.from_numpy(e4m3_decode(k_cache_bits)).to(torch.float64) * float(k_scale)
    vf = torch.from_numpy(e4m3_decode(v_cache_bits)).to(torch.float64) * float(v_scale)
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
        pi = torch.from_numpy(pages.astype(np.int64))
        ti = torch.from_numpy(toks % page)
        kk = kf[pi, ti][:, head_map]  # [n, Hq, D] (GQA repeat)
        vv = vf[pi, ti][:, head_map]
        s = torch.einsum("nhd,hd->nh", kk, q[i]) * float(scale)
        p = torch.softmax(s, dim=0)
        out[i] = torch.einsum("nh,nhd->hd", p, vv)
    return out.to(torch.float32).numpy()


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
