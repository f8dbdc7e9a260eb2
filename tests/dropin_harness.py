"""The drop-in check: this package's kernels inside the reference runtime itself.

Runs in its own process (``python -m tests.dropin_harness ...``): ``adallm_b200.install()``
rebinds the reference package's ops (installed beside the repository in baseline/_ref, or
ADALLM_REF), then the reference's own code does the rest --

  --check  a synthetic ModelOpt-style NVFP4 checkpoint of the Qwen3-8B widths (hidden 4096,
           32/8 heads of 128, SwiGLU 12288, vocab 151936; `--layers` decoder layers) is written
           to disk; ``adallm.runtime.model_runner.ModelRunner`` (model_runner.py:17-79) builds the
           model, loads it through ``adallm.infra.loader.load_model`` (the install()-hooked
           post-load prepack included), allocates the FP8 paged KV cache, runs the decode
           self-test and captures its decode CUDA graphs (model_runner.py:333-368).  Sequences
           are scheduled by the reference's ``BlockManager`` (page 256, prefix hashing): a fresh
           prefill of two prompts, then a prompt sharing a full 256-token page with the first
           (a prefix-cache hit: the paged-prefill branch), then teacher-forced decode steps of
           all three through ``ModelRunner.prepare_decode`` + ``run_model`` (graph replay).
           Every logits row is compared with the CPU oracle decoder (exact numerics) and with the
           emulation of the reference's own kernel arithmetic on the same inputs; one JSON line
           with the figures is printed.
  --bench  the decode-step time of the reference's Qwen3ForCausalLM (36 layers, Qwen3-8B
           widths, random NVFP4 weights filled on the device) under install(), through the
           reference's KV allocation and graph capture (ModelRunner.allocate_kv_cache /
           capture_cudagraph / prepare_decode / run_model, called on a runner built without the
           NCCL set-up and checkpoint load of its __init__); one JSON line.
  --flash-attn  whether flash-attn (the reference's prefill without a prefix cache) runs on
           this GPU; one JSON line.

Test and benchmark infrastructure only (tests/test_gpu_dropin.py, bench.py's kernel lines)."""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.environ.get("ADALLM_REF", os.path.join(ROOT, "baseline", "_ref"))
PAGE = 256  # the reference runtime requires kvcache_block_size % 256 == 0 (settings.py:152)

QWEN3 = dict(hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=12288, vocab=151936)


def reference_available() -> tuple[bool, str]:
    if not os.path.isdir(os.path.join(REF_DIR, "adallm")):
        return False, f"reference package not found in {REF_DIR}"
    return True, REF_DIR


def _setup(fresh_prefill: str | None = None, fused_layers: bool = True):
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    os.environ.setdefault("ADALLM_DISABLE_PROGRESS", "1")
    os.environ.setdefault("ADALLM_QUIET", "1")
    for p in (ROOT, REF_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    import adallm_b200
    adallm_b200.install(fresh_prefill=fresh_prefill, fused_layers=fused_layers)


def _hf_config_dict(layers: int, vocab: int) -> dict:
    q = QWEN3
    return {"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": q["hidden"],
            "intermediate_size": q["inter"], "num_hidden_layers": layers, "num_attention_heads": q["heads"],
            "num_key_value_heads": q["kv_heads"], "head_dim": q["head_dim"], "vocab_size": vocab,
            "max_position_embeddings": 40960, "rms_norm_eps": 1e-6, "rope_theta": 1000000,
            "attention_bias": False, "hidden_act": "silu", "tie_word_embeddings": False, "torch_dtype": "bfloat16",
            "quantization_config": {"quant_method": "modelopt", "quant_algo": "NVFP4",
                                    "config_groups": {"group_0": {"weights": {"group_size": 16}}},
                                    "kv_cache_scheme": {"num_bits": 8}}}


def _config(model_dir: str, **kw):
    """The reference's Config for a model directory.  With transformers 5 the Qwen3 config keeps
    rope_theta inside rope_parameters (and reports rope_scaling {"rope_type": "default"}), which
    the reference's get_rope (rotary_embedding.py:77-90) does not read: the two attributes the
    reference reads are set back to their transformers 4 meaning."""
    from adallm.settings import Config
    cfg = Config(model_dir, **kw)
    cfg.hf_config.rope_theta = 1000000.0
    cfg.hf_config.rope_scaling = None
    return cfg


def random_weights(layers: int, vocab: int, seed: int):
    """CPU weights in the reference parameter layout (packed e2m1 uint8 [N, K/2], fp16-held e4m3
    block scales [N, K/16], fp32 global scale per fused linear), as the oracle decoder takes them,
    plus the per-projection tensors a ModelOpt checkpoint stores."""
    import torch
    from adallm_b200.decode_step import random_nvfp4
    q = QWEN3
    H, D = q["hidden"], q["head_dim"]
    g = torch.Generator().manual_seed(seed)
    ckpt, layers_w = {}, []
    for li in range(layers):
        parts = {"q": (q["heads"] * D, H), "k": (q["kv_heads"] * D, H), "v": (q["kv_heads"] * D, H),
                 "o": (H, q["heads"] * D), "gate": (q["inter"], H), "up": (q["inter"], H), "down": (H, q["inter"])}
        mats = {}
        for name, (n, k) in parts.items():
            packed, scale, s2 = random_nvfp4(n, k, seed * 1000 + li * 16 + len(mats), torch.device("cpu"))
            mats[name] = (packed, scale, s2)
        # one global scale per fused linear (the loader keeps the last shard's, loader.py:103-115)
        s_qkv, s_gu = mats["q"][2], mats["gate"][2]
        pre = f"model.layers.{li}."
        for name, mod, s2 in (("q", "self_attn.q_proj", s_qkv), ("k", "self_attn.k_proj", s_qkv),
                              ("v", "self_attn.v_proj", s_qkv), ("o", "self_attn.o_proj", mats["o"][2]),
                              ("gate", "mlp.gate_proj", s_gu), ("up", "mlp.up_proj", s_gu),
                              ("down", "mlp.down_proj", mats["down"][2])):
            packed, scale, _ = mats[name]
            ckpt[pre + mod + ".weight"] = packed
            ckpt[pre + mod + ".weight_scale"] = scale.to(torch.float8_e4m3fn)
            ckpt[pre + mod + ".weight_scale_2"] = torch.tensor(s2, dtype=torch.float32)
            ckpt[pre + mod + ".input_scale"] = torch.tensor(1.0, dtype=torch.float32)
        norms = {n: (1.0 + 0.1 * torch.randn(size, generator=g)).to(torch.bfloat16)
                 for n, size in (("in_norm", H), ("post_norm", H), ("q_norm", D), ("k_norm", D))}
        ckpt[pre + "input_layernorm.weight"] = norms["in_norm"]
        ckpt[pre + "post_attention_layernorm.weight"] = norms["post_norm"]
        ckpt[pre + "self_attn.q_norm.weight"] = norms["q_norm"]
        ckpt[pre + "self_attn.k_norm.weight"] = norms["k_norm"]
        cat = lambda names, s2: (torch.cat([mats[n][0] for n in names]), torch.cat([mats[n][1] for n in names]), s2)
        L = dict(qkv=cat("qkv", s_qkv), o=mats["o"], gate_up=cat(["gate", "up"], s_gu), down=mats["down"])
        L.update(norms)
        layers_w.append(L)
    embed = (torch.randn((vocab, H), generator=g) * 0.02).to(torch.bfloat16)
    lm_head = (torch.randn((vocab, H), generator=g) * 0.02).to(torch.bfloat16)
    final_norm = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    ckpt["model.embed_tokens.weight"] = embed
    ckpt["lm_head.weight"] = lm_head
    ckpt["model.norm.weight"] = final_norm
    from oracle.layers import rope_cache
    oracle_w = dict(layers=layers_w, embed=embed, lm_head=lm_head, final_norm=final_norm,
                    cos_sin=rope_cache(D, 4096, 1e6))
    return ckpt, oracle_w


def check(layers: int, decode_steps: int, seed: int, fresh_prefill: str = "kernel", fused_layers: bool = True) -> dict:
    """fresh_prefill "kernel" (default here): the fresh prefill also runs this package's paged
    prefill kernel, so every attention of the check is ours; "reference" keeps flash-attn.
    fused_layers: install()'s fused decode layers (default) or the per-op path."""
    _setup(fresh_prefill, fused_layers)
    import numpy as np
    import torch
    from safetensors.torch import save_file
    from adallm.infra.context import reset_context
    from adallm.runtime.block_manager import BlockManager
    from adallm.runtime.model_runner import ModelRunner
    from adallm.runtime.sequence import Sequence
    from types import SimpleNamespace
    from oracle.decode import OracleDecoder

    vocab = QWEN3["vocab"]
    ckpt, ow = random_weights(layers, vocab, seed)
    tmp = tempfile.mkdtemp(prefix="adallm_dropin_")
    with open(os.path.join(tmp, "config.json"), "w") as f:
        json.dump(_hf_config_dict(layers, vocab), f)
    with open(os.path.join(tmp, "hf_quant_config.json"), "w") as f:
        json.dump({"quantization": {"quant_algo": "NVFP4", "group_size": 16}}, f)
    save_file(ckpt, os.path.join(tmp, "model.safetensors"))
    del ckpt
    config = _config(tmp, max_num_seqs=8, max_model_len=1024, max_num_batched_tokens=4096,
                     gpu_memory_utilization=0.9, kvcache_block_size=PAGE)
    t0 = time.perf_counter()
    runner = ModelRunner(config, 0, [])
    setup_s = time.perf_counter() - t0
    from adallm_b200 import nvfp4_gemm
    prepacked = sum(1 for m in runner.model.modules()
                    if getattr(getattr(m, "weight_scale", None), "_ada_sf", None) is not None)

    ocfg = SimpleNamespace(num_layers=layers, hidden=QWEN3["hidden"], num_heads=QWEN3["heads"],
                           num_kv_heads=QWEN3["kv_heads"], head_dim=QWEN3["head_dim"],
                           intermediate=QWEN3["inter"], rms_eps=1e-6, page_size=PAGE)
    decoders = {"exact": OracleDecoder(ocfg, ow, numerics="exact"),
                "reference": OracleDecoder(ocfg, ow, numerics="reference")}
    nblk = config.num_kvcache_blocks
    caches = {k: ([np.zeros((nblk, PAGE, QWEN3["kv_heads"], QWEN3["head_dim"]), np.uint8) for _ in range(layers)],
                  [np.zeros((nblk, PAGE, QWEN3["kv_heads"], QWEN3["head_dim"]), np.uint8) for _ in range(layers)])
              for k in decoders}
    bm = BlockManager(nblk, PAGE)
    Sequence.block_size = PAGE
    gen = torch.Generator().manual_seed(seed + 7)
    rand = lambda n: torch.randint(0, vocab, (n,), generator=gen).tolist()
    shared = rand(PAGE)
    seqs = [Sequence(shared + rand(16)), Sequence(rand(40))]
    later = Sequence(shared + rand(20))  # a full shared page: prefix-cache hit

    def oracle_rows(batch, new_only=True):
        """Rows of the oracle step for the tokens the runtime computes: the uncached prompt tokens
        (prefill) -- every row attends its own prefix, which the oracle's step stores first."""
        ids, pos, slots, ctxl, tabs = [], [], [], [], []
        width = max(len(s.block_table) for s in batch)
        for s in batch:
            start = s.num_cached_tokens if new_only else len(s) - 1
            for p in range(start, len(s)):
                ids.append(s.token_ids[p])
                pos.append(p)
                slots.append(s.block_table[p // PAGE] * PAGE + p % PAGE)
                ctxl.append(p + 1)
                tabs.append(s.block_table + [-1] * (width - len(s.block_table)))
        return (torch.tensor(ids), torch.tensor(pos), np.asarray(slots, np.int32), np.asarray(ctxl, np.int32),
                np.asarray(tabs, np.int32))

    def oracle_step(batch, prefill):
        rows = oracle_rows(batch, new_only=prefill)
        last = np.cumsum([len(s) - (s.num_cached_tokens if prefill else len(s) - 1) for s in batch]) - 1
        return {k: d.step(*rows, *caches[k])[torch.from_numpy(last)] for k, d in decoders.items()}

    errs, ref_errs, agree, agree_ref, total = [], [], 0, 0, 0
    phases = []

    def compare(name, ours, theirs):
        ex, rf = theirs["exact"], theirs["reference"]
        e = float((ours - ex).norm() / ex.norm())
        re = float((rf - ex).norm() / ex.norm())
        errs.append(e)
        ref_errs.append(re)
        phases.append({"phase": name, "rows": int(ex.shape[0]), "rel_l2": round(e, 5), "ref_rel_l2": round(re, 5)})
        return ex.argmax(dim=1)

    # 1. fresh prefill of two prompts (no block tables in the context)
    for s in seqs:
        bm.allocate(s)
    ids, pos = runner.prepare_prefill(seqs)
    ours = runner.run_model(ids, pos, True).float().cpu()
    reset_context()
    toks = compare("prefill_fresh", ours, oracle_step(seqs, True))
    # 2. a prompt sharing the first full page: prefix-cache prefill (block tables in the context)
    bm.allocate(later)
    assert later.num_cached_tokens == PAGE, later.num_cached_tokens
    ids, pos = runner.prepare_prefill([later])
    ours_l = runner.run_model(ids, pos, True).float().cpu()
    reset_context()
    tok_l = compare("prefill_prefix_cache", ours_l, oracle_step([later], True))
    allseqs = seqs + [later]
    nxt = torch.cat([toks, tok_l]).tolist()
    # 3. teacher-forced decode steps of all three (graph replay)
    for step in range(decode_steps):
        for s, t in zip(allseqs, nxt):
            s.append_token(int(t))
            bm.may_append(s)
        ids, pos = runner.prepare_decode(allseqs)
        ours = runner.run_model(ids, pos, False).float().cpu()
        reset_context()
        theirs = oracle_step(allseqs, False)
        ref_tok = compare(f"decode_{step}", ours, theirs)
        agree += int((ours.argmax(dim=1) == ref_tok).sum())
        agree_ref += int((theirs["reference"].argmax(dim=1) == ref_tok).sum())
        total += len(allseqs)
        nxt = ref_tok.tolist()
    nvfp4_gemm.check_device_errors()
    out = {"layers": layers, "decode_steps": decode_steps, "page": PAGE, "fresh_prefill": fresh_prefill,
           "setup_s": round(setup_s, 1),
           "prepacked_weights": prepacked, "graphs": sorted(runner.graphs.keys()),
           "raw": agree / total, "raw_reference": agree_ref / total, "tokens": total,
           "rel_l2_max": max(errs), "rel_l2_mean": float(np.mean(errs)),
           "ref_rel_l2_mean": float(np.mean(ref_errs)), "phases": phases[:2],
           "fused_layers": fused_layers, "fused_layer_calls": _fused_calls()}
    runner.exit()
    return out


def _fused_calls() -> int:
    from adallm_b200 import fused_layer
    return int(fused_layer.CALLS)


def bench(layers: int, batch: int, ctx: int, reps: int, fused_layers: bool = True) -> dict:
    """Decode-step time of the reference runtime's captured graph with this package installed."""
    _setup(None, fused_layers)
    import torch
    import torch.distributed as dist
    from adallm.architectures.registry import build_model
    from adallm.infra.context import reset_context
    from adallm.infra.quant import set_quant_config
    from adallm.runtime.model_runner import ModelRunner
    from adallm.runtime.sequence import Sequence
    from adallm_b200 import nvfp4_gemm
    from adallm_b200.decode_step import random_nvfp4

    tmp = tempfile.mkdtemp(prefix="adallm_dropin_bench_")
    with open(os.path.join(tmp, "config.json"), "w") as f:
        json.dump(_hf_config_dict(layers, QWEN3["vocab"]), f)
    config = _config(tmp, max_num_seqs=batch, max_model_len=max(1024, ctx + 64), max_num_batched_tokens=16384,
                     gpu_memory_utilization=0.9, kvcache_block_size=PAGE)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if not dist.is_initialized():  # the model's parallel layers read the TP rank and size (world 1)
        dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    hf = config.hf_config
    set_quant_config(hf, config)
    torch.set_default_dtype(torch.bfloat16)
    torch.set_default_device("cuda")
    model, _ = build_model(hf)
    with torch.no_grad():
        for i, m in enumerate(model.modules()):
            w, s = getattr(m, "weight", None), getattr(m, "weight_scale", None)
            if w is not None and w.dtype == torch.uint8 and s is not None:
                n, k = w.shape[0], w.shape[1] * 2
                packed, scale, s2 = random_nvfp4(n, k, 100 + i, dev)
                w.copy_(packed)
                s.copy_(scale)
                m.weight_scale_2.fill_(s2)
            elif w is not None and w.dtype == torch.bfloat16:
                if w.dim() == 1:
                    w.fill_(1.0)
                else:
                    w.normal_(0.0, 0.02)
    nvfp4_gemm.prepack_model(model)
    runner = ModelRunner.__new__(ModelRunner)
    runner.config, runner.block_size, runner.enforce_eager = config, PAGE, False
    runner.world_size, runner.rank, runner.model = 1, 0, model
    runner.allocate_kv_cache()
    runner.capture_cudagraph()
    torch.set_default_device("cpu")
    seqs = []
    Sequence.block_size = PAGE
    next_block = 0
    for b in range(batch):
        s = Sequence(list(range(ctx)))
        nb = -(-ctx // PAGE)
        s.block_table = list(range(next_block, next_block + nb))
        next_block += nb
        seqs.append(s)
    ids, pos = runner.prepare_decode(seqs)
    for _ in range(3):
        runner.run_model(ids, pos, False)
    graph = runner.graphs[next(x for x in runner.graph_bs if x >= batch)]
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    e1.synchronize()
    step_ms = e0.elapsed_time(e1) / reps
    # the same through run_model, with the host work of a step (static-buffer copies, lm_head)
    t0 = time.perf_counter()
    for _ in range(reps):
        runner.run_model(ids, pos, False)
    torch.cuda.synchronize()
    run_ms = (time.perf_counter() - t0) * 1e3 / reps
    reset_context()
    nvfp4_gemm.check_device_errors()
    return {"layers": layers, "batch": batch, "ctx": ctx, "page": PAGE, "graph_ms": round(step_ms, 4),
            "run_model_ms": round(run_ms, 4), "tok_s": round(batch / (run_ms / 1e3), 1),
            "graph_tok_s": round(batch / (step_ms / 1e3), 1), "fused_layers": fused_layers,
            "fused_layer_calls": _fused_calls()}


def flash_attn_probe() -> dict:
    import torch
    try:
        from flash_attn import flash_attn_varlen_func
    except Exception as exc:
        return {"flash_attn": "not importable", "error": str(exc)[:200]}
    d = torch.device("cuda", 0)
    q = torch.randn((32, 4, 128), device=d, dtype=torch.float16)
    cu = torch.tensor([0, 32], dtype=torch.int32, device=d)
    try:
        o = flash_attn_varlen_func(q, q, q, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=32, max_seqlen_k=32,
                                   causal=True)
        torch.cuda.synchronize()
        return {"flash_attn": "runs", "finite": bool(torch.isfinite(o).all())}
    except Exception as exc:
        return {"flash_attn": "fails", "error": str(exc).splitlines()[0][:200],
                "capability": list(torch.cuda.get_device_capability())}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=["check", "bench", "flash-attn"])
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--steps", type=int, default=24)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--ctx", type=int, default=512)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--seed", type=int, default=5)
    ap.add_argument("--fresh-prefill", default="kernel", choices=["kernel", "reference"])
    ap.add_argument("--per-op", action="store_true", help="install(fused_layers=False): the per-op decode path")
    a = ap.parse_args()
    ok, why = reference_available()
    if not ok:
        print(json.dumps({"unavailable": why}))
        return
    if a.mode == "check":
        r = check(a.layers, a.steps, a.seed, a.fresh_prefill, not a.per_op)
    elif a.mode == "bench":
        r = bench(a.layers, a.batch, a.ctx, a.reps, not a.per_op)
    else:
        r = flash_attn_probe()
    print("DROPIN " + json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
