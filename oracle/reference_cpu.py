"""The reference's own CPU-runnable decode path, run from the reference package itself, for the
timed CPU baseline (bench.py's cpu_baseline leg and ``bench.py --impl reference``).  Test and
benchmark infrastructure only; never part of the product path.

The reference (package ``adallm``, installed next to this repository with
``pip install --target baseline/_ref``, or found through ADALLM_REF) is built as its model
runner builds it, minus the GPU:
  * model: ``adallm.architectures.qwen3.Qwen3ForCausalLM`` (qwen3.py:1588-1618, decoder layer
    :1340-1371, attention :414-487, MLP :490-516) with its own RMSNorm, rotary, SiluAndMul
    modules (run eagerly: TORCHDYNAMO_DISABLE) and LinearBase's ``F.linear`` (linear.py:74);
  * weights: random NVFP4 codes and e4m3 block scales dequantised to bf16 once by the
    reference's ``adallm.infra.nvfp4.dequant_nvfp4`` (nvfp4.py:36-77), the loader's "dequant"
    mode (loader.py:92-102);
  * attention: the reference has no CPU decode kernel (its FP8 decode is a Triton kernel,
    attention.py:126-233).  The FP8 KV store uses the statements of store_kvcache's torch
    branch (attention.py:245-251); the cache is gathered with the reference's own
    ``_gather_kv_from_blocks`` (attention.py:254-286) and attended with torch's SDPA (GQA);
  * per step: ``set_context`` as ``ModelRunner.prepare_decode`` does (model_runner.py:278-298),
    ``model(input_ids, positions)``, ``compute_logits`` (embed_head.py:56-66) and a greedy
    argmax.
If the reference package cannot be imported, ``available()`` says why.
"""
from __future__ import annotations

import os
import sys
import time
from types import SimpleNamespace

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.environ.get("ADALLM_REF", os.path.join(ROOT, "baseline", "_ref"))


def _import_reference():
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import torch
    try:
        import torch._dynamo
        torch._dynamo.config.disable = True  # the reference's @torch.compile ops run eagerly here
    except Exception:
        pass
    import adallm.architectures.qwen3 as rq
    import adallm.infra.context as rctx
    import adallm.infra.nvfp4 as rnv
    import adallm.ops.attention as rattn
    return rq, rctx, rnv, rattn


def available() -> tuple[bool, str]:
    try:
        _import_reference()
        return True, REF_DIR
    except Exception as exc:  # pragma: no cover - depends on the install
        return False, f"reference package not importable from {REF_DIR}: {exc}"


class ReferenceCpuDecode:
    """A Qwen3-shape model of the reference package on the host cores, decode steps at a fixed
    batch and context length (every step attends `ctx` cached tokens per sequence)."""

    def __init__(self, layers=36, hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=12288, vocab=151936,
                 batch=16, ctx=64, page=16, threads=None, seed=0):
        import torch
        import torch.distributed as dist
        import torch.nn.functional as F
        rq, rctx, rnv, rattn = _import_reference()
        self.threads = threads or os.cpu_count()
        torch.set_num_threads(self.threads)
        if not dist.is_initialized():  # LinearBase reads the TP rank / size (world 1, no rendezvous)
            dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
        cfg = SimpleNamespace(hidden_size=hidden, num_attention_heads=heads, num_key_value_heads=kv_heads,
                              max_position_embeddings=max(4096, ctx + 16), rms_norm_eps=1e-6, attention_bias=False,
                              head_dim=head_dim, rope_theta=1e6, rope_scaling=None, intermediate_size=inter,
                              hidden_act="silu", vocab_size=vocab, num_hidden_layers=layers,
                              tie_word_embeddings=False)
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            t0 = time.perf_counter()
            self.model = rq.Qwen3ForCausalLM(cfg)
        finally:
            torch.set_default_dtype(prev)
        g = torch.Generator().manual_seed(seed)

        def nvfp4_bf16(n, k):
            packed = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.uint8)
            sbits = torch.randint(0x30, 0x41, (n, k // 16), generator=g, dtype=torch.uint8)
            scale = sbits.view(torch.float8_e4m3fn).to(torch.float16)
            s2 = torch.tensor(1.0 / (k ** 0.5 * 3.2), dtype=torch.float32)
            return rnv.dequant_nvfp4(packed, scale, s2, group_size=16, dtype=torch.bfloat16)

        with torch.no_grad():
            for layer in self.model.model.layers:
                at, mlp = layer.self_attn, layer.mlp
                at.qkv_proj.weight.data.copy_(nvfp4_bf16((heads + 2 * kv_heads) * head_dim, hidden))
                at.o_proj.weight.data.copy_(nvfp4_bf16(hidden, heads * head_dim))
                mlp.gate_up_proj.weight.data.copy_(nvfp4_bf16(2 * inter, hidden))
                mlp.down_proj.weight.data.copy_(nvfp4_bf16(hidden, inter))
                for norm in (layer.input_layernorm, layer.post_attention_layernorm, at.q_norm, at.k_norm):
                    norm.weight.data.fill_(1.0)
            self.model.model.norm.weight.data.fill_(1.0)
            self.model.model.embed_tokens.weight.data.copy_(torch.randn((vocab, hidden), generator=g) * 0.02)
            self.model.lm_head.weight.data.copy_(torch.randn((vocab, hidden), generator=g) * 0.02)
        self.setup_s = time.perf_counter() - t0

        # paged FP8 KV cache [2, L, pages, page, Hkv, D] as ModelRunner.allocate_kv_cache lays it out
        # (model_runner.py:153-169), holding `ctx` random cached tokens per sequence
        pages_per_seq = -(-(ctx + 1) // page)
        pages = batch * pages_per_seq
        kv = (torch.randn((2, layers, pages, page, kv_heads, head_dim), generator=g)).to(torch.float8_e4m3fn)
        perm = torch.randperm(pages, generator=g).to(torch.int32)
        self.block_tables = perm.view(batch, pages_per_seq).contiguous()
        scale = head_dim ** -0.5
        gather = rattn._gather_kv_from_blocks
        get_context = rctx.get_context

        def cpu_decode_attention(mod, q, k, v):
            """Attention.forward's decode branch on the host: the FP8 store (store_kvcache's torch
            statements, attention.py:245-251), the reference's page gather and SDPA per sequence."""
            c = get_context()
            D = mod.num_kv_heads * mod.head_dim
            slots = c.slot_mapping.to(torch.int64)
            mod.k_cache.view(-1, D)[slots] = k.to(mod.k_cache.dtype).view(-1, D)
            mod.v_cache.view(-1, D)[slots] = v.to(mod.v_cache.dtype).view(-1, D)
            kk, vv, cu = gather(mod.k_cache, mod.v_cache, c.block_tables, c.context_lens)
            out = torch.empty((q.shape[0], mod.num_heads, mod.head_dim), dtype=torch.float32)
            for b in range(q.shape[0]):
                s, e = int(cu[b]), int(cu[b + 1])
                qb = q[b].to(torch.float16).float().unsqueeze(1)           # [Hq, 1, D]
                kb = kk[s:e].float().transpose(0, 1)                       # [Hkv, n, D]
                vb = vv[s:e].float().transpose(0, 1)
                out[b] = F.scaled_dot_product_attention(qb, kb, vb, scale=scale, enable_gqa=True).squeeze(1)
            return out.to(torch.float16).to(q.dtype)

        for li, layer in enumerate(self.model.model.layers):
            attn = layer.self_attn.attn
            attn.k_cache, attn.v_cache = kv[0, li], kv[1, li]
            attn.forward = (lambda m: (lambda q, k, v: cpu_decode_attention(m, q, k, v)))(attn)
        self.kv = kv
        self.rctx = rctx
        self.batch, self.ctx, self.page, self.vocab = batch, ctx, page, vocab

    def step(self) -> float:
        """One decode step of the batch at context length ctx (the new token at position ctx - 1);
        returns its wall time in seconds."""
        import torch
        B, page = self.batch, self.page
        pos = torch.full((B,), self.ctx - 1, dtype=torch.int64)
        blk = self.block_tables[torch.arange(B), pos // page].to(torch.int64)
        slot = (blk * page + pos % page).to(torch.int32)
        ids = torch.randint(0, self.vocab, (B,))
        t0 = time.perf_counter()
        with torch.inference_mode():
            self.rctx.set_context(False, slot_mapping=slot, context_lens=torch.full((B,), self.ctx, dtype=torch.int32),
                                  block_tables=self.block_tables, max_seqlen_k=self.ctx)
            h = self.model(ids, pos)
            logits = self.model.compute_logits(h)
            tokens = logits.argmax(dim=-1)
            self.rctx.reset_context()
        dt = time.perf_counter() - t0
        self.last_tokens = tokens
        return dt
