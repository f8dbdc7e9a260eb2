"""Timed CPU baseline: the reference's own CPU-runnable decode path (dequantise-then-
compute, adallm/infra/loader.py:92-102 + F.linear at adallm/ops/linear.py:74, KV gather
+ fp32 softmax per adallm/ops/attention.py:254-286) restated by oracle.decode, timed on
the host cores.  Test / benchmark infrastructure only (bench.py's cpu_baseline leg and
``--impl reference``); never part of the product path.

A full Qwen3-8B-shape step on the CPU reads ~16 GB of dequantised bf16 weights, so the
sample is bounded: one of the decoder layers (full-size weights) plus the full lm_head,
timed over repeated steps, scaled to all layers:
    t_step = t_lm_head + num_layers * (t_one_layer_step - t_lm_head)
"""
from __future__ import annotations

import os
import time
from types import SimpleNamespace

import numpy as np
import torch

from .decode import OracleDecoder
from .layers import rope_cache


def _random_layer(cfg, g):
    D = cfg.head_dim

    def nvfp4(n, k):
        packed = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.int32).to(torch.uint8)
        sb = torch.randint(0x30, 0x41, (n, k // 16), generator=g, dtype=torch.int32).to(torch.uint8)
        return packed, sb.view(torch.float8_e4m3fn).to(torch.float16), 1.0 / (k ** 0.5 * 3.2)

    qkv_n = (cfg.num_heads + 2 * cfg.num_kv_heads) * D
    return dict(qkv=nvfp4(qkv_n, cfg.hidden), o=nvfp4(cfg.hidden, cfg.num_heads * D),
                gate_up=nvfp4(2 * cfg.intermediate, cfg.hidden), down=nvfp4(cfg.hidden, cfg.intermediate),
                in_norm=torch.ones(cfg.hidden, dtype=torch.bfloat16),
                post_norm=torch.ones(cfg.hidden, dtype=torch.bfloat16),
                q_norm=torch.ones(D, dtype=torch.bfloat16), k_norm=torch.ones(D, dtype=torch.bfloat16))


class CpuDecodeSample:
    """One full-size decoder layer + lm_head of the decode step, dequantised to bf16 once."""

    def __init__(self, num_layers, hidden, num_heads, num_kv_heads, head_dim, intermediate, vocab, batch, ctx,
                 page=16, threads=None, seed=0):
        self.threads = threads or os.cpu_count()
        torch.set_num_threads(self.threads)
        self.num_layers = num_layers
        cfg = SimpleNamespace(num_layers=1, hidden=hidden, num_heads=num_heads, num_kv_heads=num_kv_heads,
                              head_dim=head_dim, intermediate=intermediate, rms_eps=1e-6, page_size=page)
        g = torch.Generator().manual_seed(seed)
        weights = dict(layers=[_random_layer(cfg, g)],
                       # the embedding lookup is not timed work: a small table stands in for it
                       embed=(torch.randn((1024, hidden), generator=g) * 0.02).to(torch.bfloat16),
                       lm_head=(torch.randn((vocab, hidden), generator=g) * 0.02).to(torch.bfloat16),
                       final_norm=torch.ones(hidden, dtype=torch.bfloat16),
                       cos_sin=rope_cache(head_dim, 4096, 1e6))
        self.dec = OracleDecoder(cfg, weights, exact=False)
        self.B = batch
        pages_per_seq = -(-(ctx + 1) // page)
        self.pages = batch * pages_per_seq
        self.kc = [np.zeros((self.pages, page, num_kv_heads, head_dim), np.uint8)]
        self.vc = [np.zeros_like(self.kc[0])]
        rng = np.random.default_rng(seed)
        self.kc[0][:] = rng.integers(0, 0x70, self.kc[0].shape, dtype=np.uint8)  # finite e4m3 bytes
        self.vc[0][:] = rng.integers(0, 0x70, self.vc[0].shape, dtype=np.uint8)
        self.bt = np.arange(self.pages, dtype=np.int32).reshape(batch, pages_per_seq)
        self.ctx = ctx
        self.page = page
        self.vocab = vocab
        self.x = torch.randn((batch, hidden), generator=g).to(torch.bfloat16)

    def one_step(self) -> float:
        B, page = self.B, self.page
        pos = np.full(B, self.ctx - 1, np.int64)
        slots = (self.bt[np.arange(B), pos // page] * page + pos % page).astype(np.int32)
        ids = np.arange(B, dtype=np.int64) % 1024
        t0 = time.perf_counter()
        self.dec.step(torch.from_numpy(ids), torch.from_numpy(pos), slots, np.full(B, self.ctx, np.int32), self.bt,
                      self.kc, self.vc)
        return time.perf_counter() - t0

    def lm_head_time(self) -> float:
        t0 = time.perf_counter()
        torch.nn.functional.linear(self.x, self.dec.lm_head)
        return time.perf_counter() - t0

    def estimate_step_seconds(self, reps: int) -> tuple[float, float, float]:
        """(estimated full-step seconds, one-layer-step seconds, lm_head seconds), medians."""
        steps = sorted(self.one_step() for _ in range(reps))
        heads = sorted(self.lm_head_time() for _ in range(max(3, reps)))
        t1, tl = steps[len(steps) // 2], heads[len(heads) // 2]
        layer = max(t1 - tl, 0.0)
        return tl + self.num_layers * layer, t1, tl
