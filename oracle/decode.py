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
                packed, scale, s2 = L[name]
                if self.numerics == "reference":  # fp16 weight tile values, kept as fp32 for the matmul
                    d[name] = dequant_nvfp4_kernel_fp16(packed, scale, s2).float()
                    continue
                w = dequant_nvfp4_torch(packed, scale.float(), np.float32(s2))
                d[name] = w if self.exact else w.to(torch.bfloat16)
            for name in ("in_norm", "post_norm", "q_norm", "k_norm"):
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
