"""RMSNorm / GemmaRMSNorm / rotary embedding / gated activations oracle, run
eagerly in CPU torch with the reference's rounding order.  Test
infrastructure only.

Reference anchors (paths inside the reference project):
  * RMSNorm.rms_forward / add_rms_forward         adallm/ops/layernorm.py:16-40
  * GemmaRMSNorm.rms_forward / add_rms_forward    adallm/ops/layernorm.py:64-92
  * RotaryEmbedding cache + forward               adallm/ops/rotary_embedding.py:17-56
  * apply_rotary_emb (NeoX rotate-half)           adallm/ops/rotary_embedding.py:6-14
  * SiluAndMul / GeluAndMul(tanh)                 adallm/ops/activation.py:6-26
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """layernorm.py:16-26: fp32 normalise, cast to x.dtype, THEN multiply by w."""
    dt = x.dtype
    xf = x.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    xf = xf * torch.rsqrt(var + eps)
    return xf.to(dt) * w.to(dt)


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
    """layernorm.py:28-40: fp32 add; the new residual is the rounded sum; the
    norm uses the unrounded fp32 sum."""
    dt = x.dtype
    xf = x.float() + residual.float()
    res = xf.to(dt)
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    xf = xf * torch.rsqrt(var + eps)
    return xf.to(dt) * w.to(dt), res


def gemma_rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """layernorm.py:64-74: y = (x * rsqrt(mean(x^2)+eps) * (1 + w)) in fp32, then cast."""
    dt = x.dtype
    xf = x.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    xf = xf * torch.rsqrt(var + eps)
    return (xf * (1.0 + w.float())).to(dt)


def gemma_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
    """layernorm.py:76-92: fp16 adds in fp32; bf16 adds natively (rounded)."""
    dt = x.dtype
    if dt == torch.float16:
        s = x.float() + residual.float()
    else:
        s = x + residual
    res = s.to(dt)
    xf = s.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    xf = xf * torch.rsqrt(var + eps)
    return (xf * (1.0 + w.float())).to(dt), res


def rope_cache(head_size: int, max_position: int, base: float, rope_scaling: dict | None = None) -> torch.Tensor:
    """rotary_embedding.py:26-43: fp32 [max_position, 1, head_size] = [cos | sin]."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_size, 2, dtype=torch.float) / head_size))
    t = torch.arange(max_position, dtype=torch.float)
    if rope_scaling is not None:
        rope_type = rope_scaling.get("rope_type", rope_scaling.get("type", "linear"))
        if rope_type != "linear":
            raise ValueError(f"Unsupported rope_scaling type: {rope_type}")
        t = t / float(rope_scaling.get("factor", 1.0))
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1)


def apply_rope(positions: torch.Tensor, q: torch.Tensor, k: torch.Tensor, cache: torch.Tensor):
    """rotary_embedding.py:6-14, :45-56 (NeoX half split, fp32 math, cast back)."""
    cs = cache[positions]
    cos, sin = cs.chunk(2, dim=-1)

    def rot(x):
        x1, x2 = torch.chunk(x.float(), 2, dim=-1)
        return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)

    return rot(q), rot(k)


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """activation.py:11-14."""
    a, b = x.chunk(2, -1)
    return F.silu(a) * b


def gelu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """activation.py:22-26 (tanh approximation)."""
    a, b = x.chunk(2, -1)
    return F.gelu(a, approximate="tanh") * b
