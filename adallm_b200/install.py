"""Install the B200 kernels into the reference runtime (package ``adallm``).

    import adallm_b200
    adallm_b200.install()          # before adallm.LLMEngine(...) builds the model

Replaces, by the same names and signatures:
  adallm.ops.nvfp4_gemm.nvfp4_linear / nvfp4_linear_dual / nvfp4_linear_gather   (nvfp4_gemm.py:460, :567, :657)
  adallm.ops.linear.nvfp4_linear (the name LinearBase._linear calls, linear.py:6, :61-74)
  adallm.ops.attention.store_kvcache                                            (attention.py:236)
  adallm.ops.attention.Attention.forward -- decode branch, and the prefix-cache prefill branch
      (attention.py:335-358: gather + flash-attn varlen -> one kernel over the e4m3 pages); a
      prefill without a block table keeps the reference's flash-attn (fresh_prefill="reference",
      the default when flash-attn is importable) or runs the same kernel over the pages
      store_kvcache just wrote (fresh_prefill="kernel")
  adallm.ops.layernorm.RMSNorm.forward / GemmaRMSNorm.forward                    (layernorm.py:42-50, :94-102)
  adallm.ops.rotary_embedding.RotaryEmbedding.forward                            (rotary_embedding.py:45-56)
  adallm.ops.activation.SiluAndMul.forward / GeluAndMul.forward                   (activation.py:11-26)
  adallm.runtime.model_runner.ModelRunner.fp8_decode_selftest (model_runner.py:171-232 imports the
      Triton kernel by name; the replacement runs the same zero-input smoke on this kernel)
  adallm.architectures.qwen3.Qwen3DecoderLayer.forward at decode time (qwen3.py:1358-1371): the
      layer as nine fused kernels (adallm_b200.fused_layer), the reference's forward otherwise
  adallm.infra.loader's post-load step (loader.py:129-162, called at the end of load_model): runs
      the reference's step, then prepack_model() derives every NVFP4 weight's tensor-core
      scale layout once at load
and points this package's forward context at adallm.infra.context.get_context.

Weight layout, loader and engine are untouched: NVFP4 parameters keep their
uint8 [N, K/2] / fp16 [N, K/16] / fp32 [] layout (linear.py:31-43); the tensor-core
scale layout is derived from weight_scale on first use and cached on the tensor.
"""
from __future__ import annotations

import os

import torch

_INSTALLED = False


def _fresh_prefill_default() -> str:
    """"reference" (keep the reference's flash-attn over the fresh bf16 K/V) when flash-attn is
    importable -- flash-attn 2.8.3 runs on the B200 (recorded by tests/test_gpu_dropin.py) --
    else "kernel"."""
    try:
        import flash_attn  # noqa: F401
    except Exception:
        return "kernel"
    return "reference"


def block_tables_from_slots(slot_mapping: torch.Tensor, cu_seqlens_q: torch.Tensor, max_seqlen_q: int,
                            page_size: int) -> torch.Tensor:
    """Block table [B, ceil(max_seqlen_q / page)] of a prefill with no cached prefix, read off its
    slot mapping (slot = page_id * page + offset, model_runner.py:262-267): sequence b's j-th page
    holds its token j * page, whose slot is slot_mapping[cu_seqlens_q[b] + j * page]; -1 past the
    sequence.  Device ops only, no host synchronisation."""
    pages = -(-int(max_seqlen_q) // page_size)
    j = torch.arange(pages, device=slot_mapping.device, dtype=torch.int64) * page_size
    start = cu_seqlens_q[:-1].to(torch.int64).unsqueeze(1) + j.unsqueeze(0)
    valid = start < cu_seqlens_q[1:].to(torch.int64).unsqueeze(1)
    idx = torch.where(valid, start, torch.zeros_like(start))
    pid = torch.div(slot_mapping.to(torch.int64)[idx], page_size, rounding_mode="floor")
    return torch.where(valid, pid, torch.full_like(pid, -1)).to(torch.int32)


def install(terms: int | None = None, fresh_prefill: str | None = None, fused_layers: bool = True) -> None:
    """Rebind the reference's hot-path ops to this package's kernels.

    terms: activation e2m1 terms of the NVFP4 linear below prefill size (default 4); calls of
      256 tokens or more run the reference's own W4A16 arithmetic (nvfp4_gemm.nvfp4_linear_w4a16).
    fused_layers: decode steps of the reference's Qwen3DecoderLayer (qwen3.py:1358-1371) run as
      nine fused kernels (adallm_b200.fused_layer: RMSNorm+quantiser producers, split-K partial
      planes summed by the next kernel, attention with the o_proj quantiser) on the layer's own
      parameters, KV cache and forward context; every call the fused path does not cover
      (prefill, TP > 1, ...) runs the reference's forward over the replaced ops.
    fresh_prefill: the prefill without a cached prefix (no block table; the reference runs
      flash-attn varlen over the fresh bf16 K/V, attention.py:346-358): "reference" keeps that,
      "kernel" stores K/V first (as the reference does) and runs this package's prefill kernel
      over the e4m3 pages just written, with the block table read off the slot mapping.  Default:
      "reference" when flash-attn is importable, else "kernel"."""
    global _INSTALLED
    import adallm.infra.context as ref_ctx
    import adallm.ops.activation as ref_act
    import adallm.ops.attention as ref_attn
    import adallm.ops.layernorm as ref_ln
    import adallm.ops.linear as ref_linear
    import adallm.ops.nvfp4_gemm as ref_gemm
    import adallm.ops.rotary_embedding as ref_rope

    from . import activation, attention, context, layernorm, nvfp4_gemm, rotary_embedding
    from . import _native as N

    N.lib()  # fail loudly now if the CUDA library is missing: there is no fallback
    if terms is not None:
        nvfp4_gemm.DEFAULT_TERMS = int(terms)
    # NVFP4_FP8=1 selects the reference's W4A8 kernel (e4m3 activations per 64-wide K chunk and
    # e4m3 weights, nvfp4_gemm.py:23-40, :496-535).  The replacement computes the same under both
    # settings: the multi-term activation (DEFAULT_TERMS) below prefill size and the W4A16 product
    # from 256 tokens, both closer to the exact W4A16 product than the W4A8 kernel is (measured by
    # tests/test_gpu_reference_triton.py).  The setting is recorded, not acted on.
    nvfp4_gemm.REFERENCE_FP8_REQUESTED = os.getenv("NVFP4_FP8", "0").strip().lower() not in ("0", "false", "off")

    ref_gemm.nvfp4_linear = nvfp4_gemm.nvfp4_linear
    ref_gemm.nvfp4_linear_dual = nvfp4_gemm.nvfp4_linear_dual
    ref_gemm.nvfp4_linear_gather = nvfp4_gemm.nvfp4_linear_gather
    ref_linear.nvfp4_linear = nvfp4_gemm.nvfp4_linear
    try:  # the MoE blocks import the functional ops by name
        import adallm.architectures.qwen3 as ref_qwen3
        for name in ("nvfp4_linear", "nvfp4_linear_dual", "nvfp4_linear_gather"):
            if hasattr(ref_qwen3, name):
                setattr(ref_qwen3, name, getattr(nvfp4_gemm, name))
    except Exception:
        pass

    def store_kvcache(key, value, k_cache, v_cache, slot_mapping):
        attention.store_kvcache(key, value, k_cache, v_cache, slot_mapping)

    ref_attn.store_kvcache = store_kvcache

    orig_forward = getattr(ref_attn.Attention, "_adallm_ref_forward", ref_attn.Attention.forward)
    ref_attn.Attention._adallm_ref_forward = orig_forward

    mode = fresh_prefill or _fresh_prefill_default()
    if mode not in ("kernel", "reference"):
        raise ValueError(f"fresh_prefill must be 'kernel' or 'reference', not {mode!r}")

    def attn_forward(self, q, k, v):
        ctx = ref_ctx.get_context()
        has_cache = self.k_cache.numel() > 0 and self.v_cache.numel() > 0
        if self.k_cache.dtype != torch.float8_e4m3fn:
            return orig_forward(self, q, k, v)
        fresh = ctx.is_prefill and ctx.block_tables is None
        if fresh and (mode == "reference" or not has_cache or ctx.slot_mapping is None
                      or ctx.slot_mapping.numel() != q.shape[0]):
            return orig_forward(self, q, k, v)  # warm-up prefill (no cache yet) or the flash-attn route
        orig_dtype = q.dtype
        if has_cache:
            attention.store_kvcache(k, v, self.k_cache, self.v_cache, ctx.slot_mapping)
        window = self.sliding_window if (self.sliding_window is not None and self.sliding_window > 0) else 0
        if ctx.is_prefill:
            tables = ctx.block_tables if not fresh else block_tables_from_slots(
                ctx.slot_mapping, ctx.cu_seqlens_q, ctx.max_seqlen_q, self.k_cache.shape[1])
            try:
                o = attention.paged_prefill(q.view(-1, self.num_heads, self.head_dim), self.k_cache, self.v_cache,
                                            tables, ctx.cu_seqlens_q, ctx.cu_seqlens_k, ctx.max_seqlen_q,
                                            self.scale, window)
            except Exception as exc:
                if torch.cuda.is_current_stream_capturing() or isinstance(exc, ValueError):
                    raise
                raise RuntimeError("FP8 paged prefill kernel failed; no fallback is allowed in this runtime.") from exc
            return o if o.dtype == orig_dtype else o.to(orig_dtype)
        try:
            o = attention.paged_decode(q.view(-1, self.num_heads, self.head_dim), self.k_cache, self.v_cache,
                                       ctx.block_tables, ctx.context_lens, self.scale, window)
        except Exception as exc:
            if torch.cuda.is_current_stream_capturing() or isinstance(exc, ValueError):
                raise
            raise RuntimeError("FP8 KV decode kernel failed; no fallback is allowed in this runtime.") from exc
        return o if o.dtype == orig_dtype else o.to(orig_dtype)

    ref_attn.Attention.forward = attn_forward

    ref_ln.RMSNorm.forward = lambda self, x, residual=None: layernorm.rms_norm(x, self.weight, self.eps, residual)
    ref_ln.GemmaRMSNorm.forward = lambda self, x, residual=None: layernorm.rms_norm(x, self.weight, self.eps,
                                                                                   residual, gemma=True)
    ref_rope.RotaryEmbedding.forward = lambda self, positions, query, key: rotary_embedding.apply_rope(
        positions, query, key, self.cos_sin_cache)
    ref_act.SiluAndMul.forward = lambda self, x: activation.gated_act(x, 0)
    ref_act.GeluAndMul.forward = lambda self, x: activation.gated_act(x, 1)

    try:
        import adallm.runtime.model_runner as ref_runner

        def selftest(self):
            # zero-input compile/run check of the replacement decode kernel (model_runner.py:171-232)
            dev = torch.device("cuda", torch.cuda.current_device())
            q = torch.zeros((1, 8, 128), dtype=torch.bfloat16, device=dev)
            kc = torch.zeros((1, 16, 8, 128), dtype=torch.float8_e4m3fn, device=dev)
            attention.paged_decode(q, kc, kc, torch.zeros((1, 1), dtype=torch.int32, device=dev),
                                   torch.ones(1, dtype=torch.int32, device=dev), 1.0)
            torch.cuda.synchronize()

        ref_runner.ModelRunner.fp8_decode_selftest = selftest
    except Exception:
        pass

    try:  # load-time scale prepack, after the reference's own post-load step (loader.py:129-162)
        import adallm.infra.loader as ref_loader
        orig_post = getattr(ref_loader, "_adallm_ref_post_load", ref_loader._init_nvfp4_bcol_scales)
        ref_loader._adallm_ref_post_load = orig_post

        def post_load(model):
            orig_post(model)
            nvfp4_gemm.prepack_model(model)

        ref_loader._init_nvfp4_bcol_scales = post_load
    except Exception:
        pass

    try:  # the decode step of the Qwen3 decoder layer on the fused kernels
        import adallm.architectures.qwen3 as ref_qwen3
        from . import fused_layer

        layer_cls = ref_qwen3.Qwen3DecoderLayer
        orig_layer = getattr(layer_cls, "_adallm_ref_forward", layer_cls.forward)
        layer_cls._adallm_ref_forward = orig_layer
        if fused_layers:
            def layer_forward(self, positions, hidden_states, residual):
                out = fused_layer.decode_forward(self, positions, hidden_states, residual, ref_ctx.get_context())
                return out if out is not None else orig_layer(self, positions, hidden_states, residual)

            layer_cls.forward = layer_forward
        else:
            layer_cls.forward = orig_layer
    except Exception:
        pass

    context.use_context_provider(ref_ctx.get_context)
    _INSTALLED = True


def installed() -> bool:
    return _INSTALLED
