"""CPU oracle of one Qwen3-shape decode step, composed from the oracle ops and
run in eager CPU torch with the reference's dtype flow.  Test infrastructure only
(token-agreement tests and the timed CPU baseline of bench.py).

Reference anchors (paths inside the reference project):
  * decoder layer     adallm/architectures/qwen3.py:1358-1371
  * attention block   adallm/architectures/qwen3.py:471-487 (q/k norm :481-483, rope :484)
  * MLP               adallm/architectures/qwen3.py:512-516
  * dequant mode      adallm/infra/loader.py:92-102 then F.linear (adallm/ops/linear.py:74)
  * KV store / decode adallm/ops/attention.py:236-251, :126-233
  * logits            adallm/ops/embed_head.py:56-66 (F.linear with the bf16 lm_head)

Numerics (``numerics=``):
  * "exact" (``exact=True``): fp32 dequantised weights, fp32 products, fp64 softmax -- the
    W4A16 oracle the GPU path is compared with;
  * "bf16" (``exact=False``): the reference's dequant mode, weights dequantised once to bf16 and
    bf16 F.linear (the timed CPU baseline);
  * "reference": the reference's own GPU kernels' arithmetic -- the fp16 NVFP4 GEMM
    (adallm/ops/nvfp4_gemm.py:58-136: x rounded to fp16, the weight tile formed in fp16, fp32
    accumulation, fp16 output cast back) and the fp16 decode attention (attention.py:165-233,
    probabilities rounded to fp16 before P.V) -- used to measure how far the reference itself
    sits from "exact" on the same inputs.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import layers as ol
from .attention import paged_decode, paged_decode_fp16_kernel
from .moe import route_topk
from .nvfp4 import dequant_nvfp4_kernel_fp16, dequant_nvfp4_torch, e4m3_encode


class OracleDecoder:
    def __init__(self, cfg, weights: dict, exact: bool = True, numerics: str | None = None):
        """cfg: an object with num_layers, hidden, num_heads, num_kv_heads, head_dim,
        intermediate, rms_eps, page_size; weights: CPU tensors
          layers[i][name] = (packed u8 [N,K/2], scale fp16 [N,K/16], scale_2 float) for
          qkv / o / gate_up / down, plus in_norm, post_norm, q_norm, k_norm (bf16)
          embed, lm_head (bf16 [V, H]), final_norm (bf16), cos_sin (fp32 [P, 1, D])."""
        self.cfg = cfg
        self.numerics = numerics or ("exact" if exact else "bf16")
        if self.numerics not in ("exact", "bf16", "reference"):
            raise ValueError(f"unknown numerics {self.numerics!r}")
        self.exact = self.numerics == "exact"
        self.layers = []
        for L in weights["layers"]:
            d = {}
            for name in ("qkv", "o", "gate_up", "down"):
                if name not in L:
                    continue
                packed, scale, s2 = L[name]
                if self.numerics == "reference":  # fp16 weight tile values, kept as fp32 for the matmul
                    d[name] = dequant_nvfp4_kernel_fp16(packed, scale, s2).float()
                    continue
                w = dequant_nvfp4_torch(packed, scale.float(), np.float32(s2))
                d[name] = w if self.exact else w.to(torch.bfloat16)
            for name in ("in_norm", "post_norm", "q_norm", "k_norm"):
                if name in L:
                    d[name] = L[name]
            self.layers.append(d)
        self.embed = weights["embed"]
        self.lm_head = weights["lm_head"]
        self.final_norm = weights["final_norm"]
        self.cos_sin = weights["cos_sin"]

    def _linear(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        if self.numerics == "exact":
            return (x.float() @ w.t()).to(x.dtype)
        if self.numerics == "reference":
            # nvfp4_gemm.py:101 a.to(fp16); :129 tl.dot fp16 x fp16 -> fp32; :131 acc.to(fp16);
            # :564 c.to(out_dtype).  fp16 x fp16 products are exact in fp32.
            return (x.to(torch.float16).float() @ w.t()).to(torch.float16).to(x.dtype)
        return F.linear(x, w)

    def step(self, ids, positions, slot_mapping, context_lens, block_tables, k_caches, v_caches):
        """One decode step.  ids/positions int64 [B]; slot_mapping/context_lens int32 [B];
        block_tables int32 [B, P]; k_caches/v_caches: per layer uint8 numpy arrays
        [pages, page, Hkv, D] (updated in place).  Returns fp32 logits [B, V]."""
        c = self.cfg
        B, D = ids.shape[0], c.head_dim
        hq, hkv = c.num_heads, c.num_kv_heads
        h = self.embed[torch.as_tensor(ids)]
        residual = None
        pos = torch.as_tensor(positions)
        for li, L in enumerate(self.layers):
            if residual is None:
                residual = h
                x = ol.rms_norm(h, L["in_norm"], c.rms_eps)
            else:
                x, residual = ol.add_rms_norm(h, residual, L["in_norm"], c.rms_eps)
            qkv = self._linear(x, L["qkv"])
            q, k, v = qkv.split([hq * D, hkv * D, hkv * D], dim=-1)
            q = ol.rms_norm(q.reshape(B, hq, D), L["q_norm"], c.rms_eps)
            k = ol.rms_norm(k.reshape(B, hkv, D), L["k_norm"], c.rms_eps)
            q, k = ol.apply_rope(pos, q, k, self.cos_sin)
            kc, vc = k_caches[li], v_caches[li]
            kflat = kc.reshape(-1, hkv * D)
            vflat = vc.reshape(-1, hkv * D)
            for b in range(B):
                s = int(slot_mapping[b])
                if s >= 0:
                    kflat[s] = e4m3_encode(k[b].float().numpy().reshape(-1))
                    vflat[s] = e4m3_encode(v[b].float().numpy().reshape(-1))
            attend = paged_decode_fp16_kernel if self.numerics == "reference" else paged_decode
            o = attend(q.float().numpy(), kc, vc, np.asarray(block_tables), np.asarray(context_lens), D ** -0.5)
            o = torch.from_numpy(o).to(torch.float16).to(torch.bfloat16)  # reference: fp16 out -> orig dtype
            h = self._linear(o.reshape(B, hq * D), L["o"])
            x, residual = ol.add_rms_norm(h, residual, L["post_norm"], c.rms_eps)
            gu = self._linear(x, L["gate_up"])
            h = self._linear(ol.silu_and_mul(gu), L["down"])
        x, _ = ol.add_rms_norm(h, residual, self.final_norm, c.rms_eps)
        return F.linear(x, self.lm_head).float()


class Gemma3OracleDecoder(OracleDecoder):
    """One Gemma3 decode step (adallm/architectures/gemma3.py) with the same numerics modes.

    Reference anchors (paths inside the reference project):
      * embedding x bf16(sqrt(hidden))        gemma3.py:198-205
      * decoder layer (4 GemmaRMSNorms)       gemma3.py:156-181
      * attention (q/k GemmaRMSNorm, local / global RoPE, scale, window)   gemma3.py:32-93, :136-139
      * MLP GELU(tanh) * up                   gemma3.py:97-125, adallm/ops/activation.py:17-26
      * final norm, tied lm_head              gemma3.py:205-206, :223-225
    cfg additionally carries query_pre_attn_scalar, sliding_window and is_sliding(layer);
    weights carry per layer in_norm / post_attn_norm / pre_ff_norm / post_ff_norm / q_norm /
    k_norm and the two rope caches cos_sin_local / cos_sin_global."""

    def __init__(self, cfg, weights: dict, numerics: str = "exact"):
        w = dict(weights)
        w["cos_sin"] = weights["cos_sin_global"]
        super().__init__(cfg, w, numerics=numerics)
        for L, src in zip(self.layers, weights["layers"]):
            for name in ("post_attn_norm", "pre_ff_norm", "post_ff_norm"):
                L[name] = src[name]
        self.cos_sin_local = weights["cos_sin_local"]
        self.normalizer = torch.tensor(cfg.hidden ** 0.5, dtype=torch.bfloat16)

    def step(self, ids, positions, slot_mapping, context_lens, block_tables, k_caches, v_caches):
        c = self.cfg
        B, D = ids.shape[0], c.head_dim
        hq, hkv = c.num_heads, c.num_kv_heads
        h = self.embed[torch.as_tensor(ids)] * self.normalizer
        residual = None
        pos = torch.as_tensor(positions)
        attend = paged_decode_fp16_kernel if self.numerics == "reference" else paged_decode
        for li, L in enumerate(self.layers):
            if residual is None:
                residual = h
                x = ol.gemma_rms_norm(h, L["in_norm"], c.rms_eps)
            else:
                x, residual = ol.gemma_add_rms_norm(h, residual, L["in_norm"], c.rms_eps)
            qkv = self._linear(x, L["qkv"])
            q, k, v = qkv.split([hq * D, hkv * D, hkv * D], dim=-1)
            q = ol.gemma_rms_norm(q.reshape(B, hq, D), L["q_norm"], c.rms_eps)
            k = ol.gemma_rms_norm(k.reshape(B, hkv, D), L["k_norm"], c.rms_eps)
            sliding = c.is_sliding(li)
            q, k = ol.apply_rope(pos, q, k, self.cos_sin_local if sliding else self.cos_sin)
            _store(k_caches[li], v_caches[li], k, v, slot_mapping, hkv * D)
            o = attend(q.float().numpy(), k_caches[li], v_caches[li], np.asarray(block_tables),
                       np.asarray(context_lens), c.query_pre_attn_scalar ** -0.5,
                       window=c.sliding_window if sliding else 0)
            o = torch.from_numpy(o).to(torch.float16).to(torch.bfloat16)
            h = ol.gemma_rms_norm(self._linear(o.reshape(B, hq * D), L["o"]), L["post_attn_norm"], c.rms_eps)
            x, residual = ol.gemma_add_rms_norm(h, residual, L["pre_ff_norm"], c.rms_eps)
            gu = self._linear(x, L["gate_up"])
            h = ol.gemma_rms_norm(self._linear(ol.gelu_and_mul(gu), L["down"]), L["post_ff_norm"], c.rms_eps)
        x, _ = ol.gemma_add_rms_norm(h, residual, self.final_norm, c.rms_eps)
        return F.linear(x, self.lm_head).float()


def _store(kc, vc, k, v, slot_mapping, width):
    """The e4m3 KV store of one step (attention.py:245-251): rows with slot -1 are skipped."""
    kflat = kc.reshape(-1, width)
    vflat = vc.reshape(-1, width)
    for b in range(k.shape[0]):
        s = int(slot_mapping[b])
        if s >= 0:
            kflat[s] = e4m3_encode(k[b].float().numpy().reshape(-1))
            vflat[s] = e4m3_encode(v[b].float().numpy().reshape(-1))


class MoEOracleDecoder(OracleDecoder):
    """One Qwen3-MoE decode step (adallm/architectures/qwen3.py, Qwen3MoeDecoderLayer) with the
    same numerics modes.  The attention half is OracleDecoder's; the MLP restates
    Qwen3MoeSparseMoeBlock.forward's TP = 1 path (qwen3.py:1010-1032, :1263-1290):
      router_logits = F.linear(x, gate)  (bf16);  softmax fp32, top-k, renormalise, to bf16;
      for each slot k: gate / up / down of expert ids[:, k] (nvfp4_linear_gather, bf16 out),
      act = SiLU(gate) * up, final += out * w[:, k]  (bf16 arithmetic, slot order).
    numerics "reference" forms the expert weights as the gather kernel does (fp16 tile,
    nvfp4_gemm.py:403-449) with fp32 accumulation; the kernel also rounds each product a * b to
    fp16 before its sum (:452), which is not restated.
    weights: per layer qkv / o as OracleDecoder, experts_gate_up = (packed [E, 2I, H/2],
    scale [E, 2I, H/16], scale_2 [E]) with gate rows first, experts_down likewise, router bf16
    [E, H]; cfg adds num_experts, top_k, moe_intermediate, norm_topk_prob."""

    def __init__(self, cfg, weights: dict, numerics: str = "exact"):
        super().__init__(cfg, weights, numerics=numerics)
        for L, src in zip(self.layers, weights["layers"]):
            L["router"] = src["router"]
            for name in ("experts_gate_up", "experts_down"):
                packed, scale, s2 = src[name]
                mats = []
                for e in range(packed.shape[0]):
                    if self.numerics == "reference":
                        mats.append(dequant_nvfp4_kernel_fp16(packed[e], scale[e], float(s2[e])).float())
                    else:
                        mats.append(dequant_nvfp4_torch(packed[e], scale[e].float(), np.float32(s2[e])))
                L[name] = torch.stack(mats)

    def _moe(self, x: torch.Tensor, L) -> torch.Tensor:
        c = self.cfg
        ids, w = route_topk(F.linear(x, L["router"]), c.top_k, c.norm_topk_prob, x.dtype)
        final = torch.zeros_like(x)
        inter = c.moe_intermediate
        for k in range(c.top_k):
            gu = torch.empty((x.shape[0], 2 * inter), dtype=x.dtype)
            out = torch.empty_like(x)
            experts = ids[:, k].unique().tolist()
            for e in experts:
                rows = (ids[:, k] == e).nonzero().view(-1)
                gu[rows] = self._linear(x[rows], L["experts_gate_up"][e])
            act = ol.silu_and_mul(gu)
            for e in experts:
                rows = (ids[:, k] == e).nonzero().view(-1)
                out[rows] = self._linear(act[rows], L["experts_down"][e])
            final = final + out * w[:, k:k + 1]
        return final

    def step(self, ids, positions, slot_mapping, context_lens, block_tables, k_caches, v_caches):
        c = self.cfg
        B, D = ids.shape[0], c.head_dim
        hq, hkv = c.num_heads, c.num_kv_heads
        h = self.embed[torch.as_tensor(ids)]
        residual = None
        pos = torch.as_tensor(positions)
        attend = paged_decode_fp16_kernel if self.numerics == "reference" else paged_decode
        for li, L in enumerate(self.layers):
            if residual is None:
                residual = h
                x = ol.rms_norm(h, L["in_norm"], c.rms_eps)
            else:
                x, residual = ol.add_rms_norm(h, residual, L["in_norm"], c.rms_eps)
            qkv = self._linear(x, L["qkv"])
            q, k, v = qkv.split([hq * D, hkv * D, hkv * D], dim=-1)
            q = ol.rms_norm(q.reshape(B, hq, D), L["q_norm"], c.rms_eps)
            k = ol.rms_norm(k.reshape(B, hkv, D), L["k_norm"], c.rms_eps)
            q, k = ol.apply_rope(pos, q, k, self.cos_sin)
            _store(k_caches[li], v_caches[li], k, v, slot_mapping, hkv * D)
            o = attend(q.float().numpy(), k_caches[li], v_caches[li], np.asarray(block_tables),
                       np.asarray(context_lens), D ** -0.5)
            o = torch.from_numpy(o).to(torch.float16).to(torch.bfloat16)
            h = self._linear(o.reshape(B, hq * D), L["o"])
            x, residual = ol.add_rms_norm(h, residual, L["post_norm"], c.rms_eps)
            h = self._moe(x, L)
        x, _ = ol.add_rms_norm(h, residual, self.final_norm, c.rms_eps)
        return F.linear(x, self.lm_head).float()
