"""Greedy-token agreement between the B200 decode engine and the CPU oracle decoder.
Used by tests/test_gpu_decode.py and __graft_entry__.smoke().

Teacher-forced: every decoder consumes the exact oracle's token each step, so one disagreement
does not cascade.  Three decoders run on the same weights and inputs:
  * ours       -- the engine (all hot-path kernels, one CUDA graph per step);
  * exact      -- the oracle with fp32 dequantised weights and an fp64 softmax (W4A16);
  * reference  -- the oracle with the reference's own kernel arithmetic (fp16 NVFP4 GEMM,
                  fp16 probabilities in the decode attention; oracle.decode "reference").
Raw greedy agreement of ours and of the reference emulation with the exact oracle, and the
relative L2 of each one's logits against the exact oracle's, are returned.

Why the reference emulation is measured beside the engine: random-init models have near-tied
logits (the top-2 gap of 151,936 Gaussian logits is ~0.2 standard deviations, and bf16 logits
near 6 have a 1/32 spacing), and the e4m3 KV cache turns last-bit bf16 differences of k/v into
one-e4m3-step (6-12%) jumps of single cache elements.  Any implementation whose arithmetic is
not bit-identical to the exact oracle therefore flips some near-ties -- the reference itself
included.  The pass criterion compares the engine with what the reference's own numerics reach
on the same inputs."""
from __future__ import annotations

import math
from dataclasses import dataclass
from types import SimpleNamespace

import numpy as np
import torch

from oracle.decode import OracleDecoder
from adallm_b200.decode_step import DecodeConfig, Qwen3DecodeEngine, DecodeSession


def small_config(layers: int) -> DecodeConfig:
    return DecodeConfig(num_layers=layers, hidden=1024, num_heads=8, num_kv_heads=2, head_dim=128,
                        intermediate=3072, vocab=4096, max_position=4096, page_size=16)


def qwen3_8b_config(layers: int) -> DecodeConfig:
    """BASELINE config 3 widths (hidden 4096, 32/8 heads of 128, SwiGLU 12288, vocab 151936,
    theta 1e6, page 16) with `layers` decoder layers."""
    return DecodeConfig(num_layers=layers, max_position=4096)


@dataclass
class Agreement:
    raw: float                 # ours vs exact, greedy tokens
    raw_reference: float       # reference emulation vs exact (nan when not run)
    logits_rel_l2_max: float   # ours vs exact, worst step
    logits_rel_l2_mean: float
    ref_logits_rel_l2_mean: float
    tokens: int
    ref_logits_rel_l2_max: float = float("nan")

    def margin(self, z: float = 2.5) -> float:
        """z standard errors of the difference of two agreement rates measured on `tokens` tokens."""
        p = min(max(self.raw_reference, 0.5), 1.0)
        return z * math.sqrt(2.0 * max(p * (1.0 - p), 1.0 / self.tokens) / self.tokens)


def run_agreement(cfg: DecodeConfig | None = None, layers=2, steps=8, batch=4, prompt=4, graph=True,
                  emulate=False, seed=1) -> Agreement:
    d = torch.device("cuda:0")
    cfg = cfg or small_config(layers)
    eng = Qwen3DecodeEngine(cfg, d, batch, max_ctx=prompt + steps + 8, seed=seed)
    ocfg = SimpleNamespace(num_layers=cfg.num_layers, hidden=cfg.hidden, num_heads=cfg.num_heads,
                           num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, intermediate=cfg.intermediate,
                           rms_eps=cfg.rms_eps, page_size=cfg.page_size)
    w = eng.export_cpu_weights()
    exact = OracleDecoder(ocfg, w, numerics="exact")
    emul = OracleDecoder(ocfg, w, numerics="reference") if emulate else None
    return agreement_loop(eng, exact, emul, steps, batch, prompt, graph, seed)


def gemma3_test_config(layers: int, window: int = 64):
    """BASELINE config 2 widths (hidden 5376, 32/16 heads of 128, GeGLU 21504, vocab 262208,
    5:1 local/global) with `layers` layers and a window short enough for the test's contexts
    to cross it (the kernels take any window; the bench runs the 1024 of config 2)."""
    from adallm_b200.gemma3_step import Gemma3Config
    return Gemma3Config(num_layers=layers, sliding_window=window, max_position=4096)


def run_agreement_gemma3(cfg, steps=8, batch=4, prompt=4, graph=True, emulate=False, seed=1) -> Agreement:
    from adallm_b200.gemma3_step import Gemma3DecodeEngine
    from oracle.decode import Gemma3OracleDecoder
    d = torch.device("cuda:0")
    eng = Gemma3DecodeEngine(cfg, d, batch, max_ctx=prompt + steps + 8, seed=seed)
    w = eng.export_cpu_weights()
    exact = Gemma3OracleDecoder(cfg, w, numerics="exact")
    emul = Gemma3OracleDecoder(cfg, w, numerics="reference") if emulate else None
    return agreement_loop(eng, exact, emul, steps, batch, prompt, graph, seed)


def moe_test_config(layers: int):
    """BASELINE config 4 widths (hidden 2048, 32/4 heads of 128, 128 experts top-8 of
    intermediate 768, vocab 151936) with `layers` layers."""
    from adallm_b200.moe_step import MoEConfig
    return MoEConfig(num_layers=layers, max_position=4096)


def run_agreement_moe(cfg, steps=8, batch=16, prompt=4, graph=True, emulate=False, seed=1) -> Agreement:
    from adallm_b200.moe_step import Qwen3MoeDecodeEngine
    from oracle.decode import MoEOracleDecoder
    d = torch.device("cuda:0")
    eng = Qwen3MoeDecodeEngine(cfg, d, batch, max_ctx=prompt + steps + 8, seed=seed)
    w = eng.export_cpu_weights()
    exact = MoEOracleDecoder(cfg, w, numerics="exact")
    emul = MoEOracleDecoder(cfg, w, numerics="reference") if emulate else None
    return agreement_loop(eng, exact, emul, steps, batch, prompt, graph, seed)


def agreement_loop(eng, exact, emul, steps, batch, prompt, graph, seed) -> Agreement:
    """Teacher-forced greedy decode of `prompt` random tokens then `steps` more through the engine
    (one captured graph per step, or eager launches) and the oracle decoders."""
    cfg = eng.cfg
    layers = cfg.num_layers
    emulate = emul is not None
    sess = DecodeSession(eng, seed=seed)

    def caches():
        kc = [np.zeros((eng.num_pages, cfg.page_size, cfg.num_kv_heads, cfg.head_dim), np.uint8) for _ in range(layers)]
        return kc, [np.zeros_like(kc[0]) for _ in range(layers)]
    kc, vc = caches()
    kr, vr = caches() if emulate else (None, None)
    g = eng.capture() if graph else None
    gen = torch.Generator().manual_seed(seed + 2)
    tokens = torch.randint(0, cfg.vocab, (batch, prompt), generator=gen)
    agree = agree_ref = total = 0
    errs, ref_errs = [], []
    cur = tokens[:, 0]
    for i in range(prompt + steps):
        sess.prepare(cur)
        sess.upload()
        if g is not None:
            g.replay()
        else:
            eng.forward()
        ours = sess.download()
        meta = (sess.h_ids.clone(), sess.h_pos.clone(), sess.h_slot.numpy().copy(), sess.h_ctx.numpy().copy(),
                sess.block_tables.numpy())
        logits = exact.step(*meta, kc, vc)
        theirs = logits.argmax(dim=1)
        ref_logits = emul.step(*meta, kr, vr) if emulate else None
        sess.commit()
        if i >= prompt - 1:  # the tokens generated after the prompt
            agree += int((ours == theirs).sum())
            total += batch
            errs.append(float((eng.logits.float().cpu() - logits).norm() / logits.norm()))
            if emulate:
                agree_ref += int((ref_logits.argmax(dim=1) == theirs).sum())
                ref_errs.append(float((ref_logits - logits).norm() / logits.norm()))
        cur = tokens[:, i + 1] if i + 1 < prompt else theirs
    eng.check_errors()
    return Agreement(raw=agree / max(total, 1), raw_reference=agree_ref / max(total, 1) if emulate else float("nan"),
                     logits_rel_l2_max=max(errs), logits_rel_l2_mean=float(np.mean(errs)),
                     ref_logits_rel_l2_mean=float(np.mean(ref_errs)) if emulate else float("nan"), tokens=total,
                     ref_logits_rel_l2_max=max(ref_errs) if emulate else float("nan"))
