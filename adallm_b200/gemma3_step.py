"""Gemma3-shape decode step built from the adallm_b200 kernels (tensor-parallel size 1).

The reference's Gemma3 decoder (adallm/architectures/gemma3.py) differs from Qwen3 in what
surrounds the same hot-path ops:

    embedding x bf16(sqrt(hidden))                      (gemma3.py:198-205)
    per layer (gemma3.py:156-181):
      x, residual = input_layernorm(h, residual)         GemmaRMSNorm: x * rs * (1 + w)
      qkv_proj; q_norm / k_norm (GemmaRMSNorm over head_dim); RoPE -- local layers use
        rope_local_base_freq without scaling, global layers rope_theta with rope_scaling
        (gemma3.py:58-69); FP8 KV store + paged decode attention with
        scale = query_pre_attn_scalar^-0.5 (:42) and the sliding window on
        "sliding_attention" layers only (:136-139)
      h = post_attention_layernorm(o_proj(attn))
      x, residual = pre_feedforward_layernorm(h, residual)
      h = post_feedforward_layernorm(down(GELU_tanh(gate) * up))    (:97-125)
    final: norm(h, residual); lm_head tied to the embedding (:223-225); greedy argmax

Fused here into nine launches per layer (ten with split-K attention): the projection's partial
planes are summed by the next kernel, and each "post-norm, residual add, pre-norm, quantise"
pair is one kernel (ada_gemma_norm2_quant_parts).  Weights are random-init NVFP4 as in
decode_step.py; norm weights are small random offsets around GemmaRMSNorm's zero init.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as N
from .decode_step import ATTN_META_EARLY, Qwen3DecodeEngine, stable_seed


@dataclass
class Gemma3Config:
    """Gemma3-27B text widths: hidden 5376, 32 query / 16 KV heads of 128,
    GeGLU 21504, local:global 5:1 with window 1024."""
    num_layers: int = 62
    hidden: int = 5376
    num_heads: int = 32
    num_kv_heads: int = 16
    head_dim: int = 128
    intermediate: int = 21504
    vocab: int = 262208
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    rope_scaling_factor: float = 8.0
    rope_local_theta: float = 1e4
    sliding_window: int = 1024
    global_every: int = 6          # layer i is global when (i + 1) % global_every == 0
    query_pre_attn_scalar: float = 168.0
    max_position: int = 32768
    page_size: int = 16
    terms: int = 4
    tp_size: int = 1
    tp_rank: int = 0

    hq = property(lambda self: self.num_heads)
    hkv = property(lambda self: self.num_kv_heads)
    inter = property(lambda self: self.intermediate)
    vocab_shard = property(lambda self: self.vocab)

    def is_sliding(self, layer: int) -> bool:
        return (layer + 1) % self.global_every != 0

    def window(self, layer: int) -> int:
        return self.sliding_window if self.is_sliding(layer) else 0


GEMMA3_27B = Gemma3Config()


class Gemma3DecodeEngine(Qwen3DecodeEngine):
    """Static-shape Gemma3 decode engine for batch ``max_batch`` (graph-capturable, TP = 1)."""

    def __init__(self, cfg: Gemma3Config, device, max_batch: int, max_ctx: int, seed: int = 0):
        if cfg.tp_size != 1:
            raise ValueError("the Gemma3 decode engine runs at tensor-parallel size 1")
        super().__init__(cfg, device, max_batch, max_ctx, seed=seed, group=None, fused=True)
        if not self.use_parts:
            raise ValueError("Gemma3 engine: a projection has no partial-plane split at this batch")

    def _init_weights(self):
        c = self.cfg
        d = self.device
        D = c.head_dim
        self.layers = []
        g = torch.Generator(device=d)

        def norm_w(n, name, li):  # GemmaRMSNorm weights: offsets around zero
            g.manual_seed(stable_seed(self.seed, "norm", name, li))
            return (torch.randn(n, generator=g, device=d) * 0.1).to(torch.bfloat16)

        for li in range(c.num_layers):
            L = {}
            L["qkv"] = self._sharded("qkv", li, [("q", c.num_heads * D), ("k", c.num_kv_heads * D),
                                                 ("v", c.num_kv_heads * D)], c.hidden, False)
            L["o"] = self._sharded("o", li, [("o", c.hidden)], c.num_heads * D, True)
            L["gate_up"] = self._sharded("gu", li, [("gate", c.intermediate), ("up", c.intermediate)], c.hidden,
                                         False)
            L["down"] = self._sharded("down", li, [("down", c.hidden)], c.intermediate, True)
            for name in ("in_norm", "post_attn_norm", "pre_ff_norm", "post_ff_norm"):
                L[name] = norm_w(c.hidden, name, li)
            L["q_norm"] = norm_w(D, "q_norm", li)
            L["k_norm"] = norm_w(D, "k_norm", li)
            self.layers.append(L)
        self.final_norm = norm_w(c.hidden, "final", 0)
        emb = torch.empty((c.vocab, c.hidden), dtype=torch.bfloat16, device=d)
        self._fill_rows(emb, "embed", 0)
        self.embed = emb
        self.lm_head = emb  # tie_word_embeddings (gemma3.py:223-225)
        # the reference registers sqrt(hidden) as a buffer in the model dtype (bf16)
        self.normalizer = torch.tensor(c.hidden ** 0.5, dtype=torch.bfloat16, device=d)
        from .rotary_embedding import build_cos_sin_cache
        self.cos_sin_global = build_cos_sin_cache(D, c.max_position, c.rope_theta,
                                                  {"rope_type": "linear", "factor": c.rope_scaling_factor},
                                                  d).contiguous()
        self.cos_sin_local = build_cos_sin_cache(D, c.max_position, c.rope_local_theta, None, d).contiguous()
        self.cos_sin = self.cos_sin_global

    # ------------------------------------------------------------------ step
    def _norm2(self, planes, post_w, w, qb, stream, y=None):
        """h = GemmaRMSNorm(post_w)(sum of planes); residual += h; GemmaRMSNorm(w) of the sum,
        quantised into qb (or written to y when qb is None)."""
        c = self.cfg
        _, ns, ld = planes
        H = c.hidden
        rp = self.residual.data_ptr()
        xq, sfx, gx = qb if qb is not None else (None, None, None)
        st = N.lib().ada_gemma_norm2_quant_parts(self.parts.data_ptr(), ns, self.B * ld, ld, post_w.data_ptr(), rp, H,
                                                 rp, H, w.data_ptr(), N.ptr(y), H, self.B, H, c.rms_eps, 0, c.terms,
                                                 self.bn, N.ptr(xq), N.ptr(sfx), N.ptr(gx), stream)
        N.check(st, "gemma post-norm + add + norm + quant")

    def forward(self):
        c = self.cfg
        B, D = self.B, c.head_dim
        lib = N.lib()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        N.check(lib.ada_embedding(self.input_ids.data_ptr(), B, self.embed.data_ptr(), 0, c.vocab, c.hidden,
                                  self.hidden.data_ptr(), 0, stream), "embedding")
        self.hidden.mul_(self.normalizer)  # gemma3.py:203, bf16 x bf16
        qn = c.hq * D
        scale = c.query_pre_attn_scalar ** -0.5
        planes = None
        for li, L in enumerate(self.layers):
            if li == 0:
                self.residual.copy_(self.hidden)
                xq, sfx, gx = self.q_hidden
                N.check(lib.ada_rmsnorm_quant(self.hidden.data_ptr(), c.hidden, None, 0, None, 0,
                                              L["in_norm"].data_ptr(), None, 0, B, c.hidden, c.rms_eps, 1, 0, c.terms,
                                              self.bn, xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), stream),
                        "gemma norm + quant")
            else:
                self._norm2(planes, self.layers[li - 1]["post_ff_norm"], L["in_norm"], self.q_hidden, stream)
            ns, ld = self._gemm_parts(self.q_hidden, L["qkv"], "qkv", stream)
            kc, vc = self.kv_cache[0, li], self.kv_cache[1, li]
            cs = self.cos_sin_local if c.is_sliding(li) else self.cos_sin_global
            N.check(lib.ada_qk_norm_rope_store_parts_ex(self.parts.data_ptr(), ns, B * ld, ld, B, c.hq, c.hkv, D,
                                                        L["q_norm"].data_ptr(), L["k_norm"].data_ptr(), c.rms_eps, 1,
                                                        self.positions.data_ptr(), cs.data_ptr(), cs.shape[0],
                                                        self.slot_mapping.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                                        1.0, 1.0, self.q_rot.data_ptr(), None, 0, stream),
                    "gemma qk_norm_rope_store")
            xq, sfx, gx = self.q_attn
            N.check(lib.ada_fp8_paged_decode_quant_ex(
                self.q_rot.data_ptr(), 0, qn, D, kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1),
                kc.stride(2), self.num_pages, self.block_tables.data_ptr(), self.block_tables.stride(0),
                self.max_pages_per_seq, self.context_lens.data_ptr(), B, c.hq, c.hkv, D, c.page_size,
                scale, 1.0, 1.0, c.window(li), None, 0, c.terms, self.bn, xq.data_ptr(), sfx.data_ptr(),
                gx.data_ptr(), self.attn_ws.data_ptr(), self.attn_ws_bytes, ATTN_META_EARLY, stream), "attention")
            planes = ("local",) + self._gemm_parts(self.q_attn, L["o"], "o", stream)
            self._norm2(planes, L["post_attn_norm"], L["pre_ff_norm"], self.q_hidden, stream)
            ns, ld = self._gemm_parts(self.q_hidden, L["gate_up"], "gate_up", stream)
            xq, sfx, gx = self.q_inter
            N.check(lib.ada_gated_act_quant_parts(self.parts.data_ptr(), ns, B * ld, ld, None, 0, B, c.inter, 1, 0,
                                                  c.terms, self.bn, xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(),
                                                  stream), "gelu_and_mul+quant")
            planes = ("local",) + self._gemm_parts(self.q_inter, L["down"], "down", stream)
        self._norm2(planes, self.layers[-1]["post_ff_norm"], self.final_norm, None, stream, y=self.xnorm)
        self._lm_head(stream)

    def kernels_per_step(self) -> int:
        """Embedding; per layer: norm(+quant), qkv GEMM, q/k-norm+RoPE+store, attention (split +
        merge+quant, or one kernel for short caches with <= 8 KV heads), o GEMM, norm pair, gate_up
        GEMM, GELU*up+quant, down GEMM; final norm pair; argmax x2."""
        short = self.max_pages_per_seq * self.cfg.page_size <= 1024 and self.cfg.hkv <= 8
        return 1 + self.cfg.num_layers * (9 + (1 if short else 2)) + 3

    def export_cpu_weights(self) -> dict:
        layers = []
        for L in self.layers:
            d = {}
            for name in ("qkv", "o", "gate_up", "down"):
                w = L[name]
                d[name] = (w.packed.cpu(), w.scale.cpu(), float(w.scale_2.item()))
            for name in ("in_norm", "post_attn_norm", "pre_ff_norm", "post_ff_norm", "q_norm", "k_norm"):
                d[name] = L[name].cpu()
            layers.append(d)
        return dict(layers=layers, embed=self.embed.cpu(), lm_head=self.lm_head.cpu(),
                    final_norm=self.final_norm.cpu(), cos_sin_global=self.cos_sin_global.cpu(),
                    cos_sin_local=self.cos_sin_local.cpu())
