"""The drop-in shim against the real reference package (CPU: import and patch only;
no kernel runs).  Skipped where the reference checkout is absent (the GPU box)."""
import inspect
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# the reference package installed next to the repository (pip --target baseline/_ref), or ADALLM_REF
REF = os.environ.get("ADALLM_REF", os.path.join(ROOT, "baseline", "_ref"))


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "adallm")):
        pytest.skip("reference checkout not available")
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    sys.path.insert(0, REF)
    try:
        import adallm.ops.nvfp4_gemm as g  # noqa: F401
    except Exception as exc:  # pragma: no cover
        pytest.skip(f"reference not importable here: {exc}")
    import adallm
    return adallm


def test_signatures_match_reference(ref):
    import adallm.ops.nvfp4_gemm as rg
    import adallm.ops.attention as ra
    from adallm_b200 import nvfp4_gemm, attention
    for name in ("nvfp4_linear", "nvfp4_linear_dual", "nvfp4_linear_gather"):
        rp = list(inspect.signature(getattr(rg, name)).parameters)
        op = list(inspect.signature(getattr(nvfp4_gemm, name)).parameters)
        assert op[:len(rp)] == rp, (name, rp, op)
    rp = list(inspect.signature(ra.store_kvcache).parameters)
    op = list(inspect.signature(attention.store_kvcache).parameters)
    assert op[:len(rp)] == rp


def test_install_patches_reference_ops(ref):
    import adallm.ops.nvfp4_gemm as rg
    import adallm.ops.linear as rl
    import adallm.ops.attention as ra
    import adallm.ops.layernorm as rln
    import adallm.ops.rotary_embedding as rr
    import adallm_b200
    from adallm_b200 import nvfp4_gemm, context
    ref_fwd = ra.Attention.forward
    adallm_b200.install()
    assert rg.nvfp4_linear is nvfp4_gemm.nvfp4_linear
    assert rl.nvfp4_linear is nvfp4_gemm.nvfp4_linear
    assert ra.Attention._adallm_ref_forward is ref_fwd or ra.Attention._adallm_ref_forward.__name__ == "forward"
    assert ra.Attention.forward.__name__ == "attn_forward"
    assert "rms_norm" in rln.RMSNorm.forward.__code__.co_names
    assert "apply_rope" in rr.RotaryEmbedding.forward.__code__.co_names
    # our context now reads the reference's
    import adallm.infra.context as rc
    rc.set_context(False, slot_mapping="s")
    assert context.get_context().slot_mapping == "s"
    rc.reset_context()
    context.use_context_provider(None)
    assert adallm_b200.install is not None


def test_ops_raise_without_cuda(ref):
    import torch
    from adallm_b200.nvfp4_gemm import nvfp4_linear
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        nvfp4_linear(x, torch.zeros(128, 128, dtype=torch.uint8), torch.zeros(128, 16, dtype=torch.float16),
                     torch.tensor(1.0), None, None, 16)


def test_prefill_routing(ref, monkeypatch):
    """After install(): a prefill with a block table (prefix cache) and an e4m3 cache goes to
    the paged prefill kernel with the context's metadata; a prefill without one stays on the
    reference branch.  The kernels are replaced by recorders (no CUDA here)."""
    import torch
    import adallm.ops.attention as ra
    import adallm.infra.context as rc
    import adallm_b200
    from adallm_b200 import attention, context
    adallm_b200.install()
    calls = []
    monkeypatch.setattr(attention, "store_kvcache", lambda *a, **k: calls.append("store"))

    def fake_prefill(q, kc, vc, bt, cu_q, cu_k, max_q, scale, window=0, *a, **k):
        calls.append(("prefill", bt, cu_q, cu_k, max_q, window))
        return torch.ones_like(q, dtype=torch.float16)

    monkeypatch.setattr(attention, "paged_prefill", fake_prefill)
    m = ra.Attention(8, 128, 0.088, 2, sliding_window=64)
    m.k_cache = torch.zeros((4, 16, 2, 128), dtype=torch.float8_e4m3fn)
    m.v_cache = torch.zeros((4, 16, 2, 128), dtype=torch.float8_e4m3fn)
    q = torch.zeros((5, 8 * 128), dtype=torch.bfloat16)
    kv = torch.zeros((5, 2, 128), dtype=torch.bfloat16)
    cu_q = torch.tensor([0, 5], dtype=torch.int32)
    cu_k = torch.tensor([0, 20], dtype=torch.int32)
    bt = torch.tensor([[2, 0]], dtype=torch.int32)
    try:
        rc.set_context(True, cu_q, cu_k, 5, 20, torch.arange(5, dtype=torch.int32), None, bt)
        o = m.forward(q, kv, kv)
        assert calls[0] == "store" and calls[1][0] == "prefill"
        assert calls[1][1] is bt and calls[1][2] is cu_q and calls[1][3] is cu_k
        assert calls[1][4] == 5 and calls[1][5] == 64
        assert o.dtype == torch.bfloat16 and o.shape == (5, 8, 128)
        # a prefill without a block table: fresh_prefill="kernel" stores, then attends the pages
        # just written with the block table read off the slot mapping
        calls.clear()
        adallm_b200.install(fresh_prefill="kernel")
        slots = torch.tensor([3 * 16 + i for i in range(5)], dtype=torch.int32)
        rc.set_context(True, cu_q, cu_q, 5, 5, slots, None, None)
        m.forward(q, kv, kv)
        assert calls[0] == "store" and calls[1][0] == "prefill"
        assert calls[1][1].tolist() == [[3]] and calls[1][2] is cu_q and calls[1][3] is cu_q
        # fresh_prefill="reference" keeps the reference branch (flash-attn, which cannot run here)
        calls.clear()
        adallm_b200.install(fresh_prefill="reference")
        with pytest.raises(Exception):
            m.forward(q, kv, kv)
        assert all(c == "store" for c in calls)
        with pytest.raises(ValueError):
            adallm_b200.install(fresh_prefill="nope")
    finally:
        rc.reset_context()
        context.use_context_provider(None)


def test_block_tables_from_slots():
    """Fresh-prefill block tables from the slot mapping: ragged sequences (1, 16, 17 and 40 tokens,
    page 16) on scattered pages, -1 past each sequence."""
    import torch
    from adallm_b200.install import block_tables_from_slots
    page = 16
    pages = [[7], [2], [9, 4], [11, 0, 5]]
    lens = [1, 16, 17, 40]
    slots, cu = [], [0]
    for pg, n in zip(pages, lens):
        slots += [pg[t // page] * page + t % page for t in range(n)]
        cu.append(cu[-1] + n)
    bt = block_tables_from_slots(torch.tensor(slots, dtype=torch.int32), torch.tensor(cu, dtype=torch.int32),
                                 max(lens), page)
    assert bt.dtype == torch.int32
    assert bt.tolist() == [[7, -1, -1], [2, -1, -1], [9, 4, -1], [11, 0, 5]]


def test_synthetic_checkpoint_loads_through_reference_loader(ref):
    """The drop-in harness's synthetic ModelOpt-style checkpoint (one layer of the Qwen3-8B
    widths, small vocabulary) goes through the reference's own loader into its Qwen3ForCausalLM
    (CPU, NVFP4 kernel-mode parameters): every packed weight, fp16-held e4m3 block scale, fused
    global scale and norm lands where the oracle decoder expects it."""
    import tempfile
    import torch
    import torch.distributed as dist
    from safetensors.torch import save_file
    from tests import dropin_harness as h
    from adallm.architectures.registry import build_model
    from adallm.infra.loader import load_model
    from adallm.infra.quant import set_quant_config
    ckpt, ow = h.random_weights(1, 512, seed=3)
    tmp = tempfile.mkdtemp()
    import json
    with open(os.path.join(tmp, "config.json"), "w") as f:
        json.dump(h._hf_config_dict(1, 512), f)
    save_file(ckpt, os.path.join(tmp, "model.safetensors"))
    cfg = h._config(tmp, max_num_seqs=8, max_model_len=1024, max_num_batched_tokens=4096, kvcache_block_size=256)
    if not dist.is_initialized():
        dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    set_quant_config(cfg.hf_config, cfg)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        model, _ = build_model(cfg.hf_config)
    finally:
        torch.set_default_dtype(prev)
    load_model(model, tmp)
    L = model.model.layers[0]
    w = ow["layers"][0]
    for mod, name in ((L.self_attn.qkv_proj, "qkv"), (L.self_attn.o_proj, "o"), (L.mlp.gate_up_proj, "gate_up"),
                      (L.mlp.down_proj, "down")):
        packed, scale, s2 = w[name]
        assert torch.equal(mod.weight.data, packed), name
        assert torch.equal(mod.weight_scale.data, scale), name
        assert float(mod.weight_scale_2) == float(torch.tensor(s2, dtype=torch.float32)), name
    assert torch.equal(L.input_layernorm.weight.data, w["in_norm"])
    assert torch.equal(L.self_attn.q_norm.weight.data, w["q_norm"])
    assert torch.equal(model.lm_head.weight.data, ow["lm_head"])
    assert cfg.hf_config.rope_theta == 1e6 and cfg.hf_config.rope_scaling is None


def test_load_time_prepack_hook(ref, monkeypatch):
    """After install(): the loader's post-load step runs the reference's step, then
    prepack_model on the loaded model (recorded here; no CUDA)."""
    import adallm.infra.loader as rl
    import adallm_b200
    from adallm_b200 import nvfp4_gemm, context
    adallm_b200.install()
    calls = []
    monkeypatch.setattr(nvfp4_gemm, "prepack_model", lambda m: calls.append(m) or 0)
    try:
        rl._init_nvfp4_bcol_scales(type("M", (), {"modules": lambda self: iter(())})())
        assert len(calls) == 1
    finally:
        context.use_context_provider(None)


def test_nvfp4_fp8_setting_is_recorded_and_keeps_the_terms(ref, monkeypatch):
    """NVFP4_FP8=1 (the reference's W4A8 mode) under install(): recorded, and the linear keeps its
    multi-term activation arithmetic below 256 tokens and the W4A16 route from there (both more
    accurate than W4A8; measured on the GPU)."""
    import adallm_b200
    from adallm_b200 import nvfp4_gemm, context
    terms, min_m = nvfp4_gemm.DEFAULT_TERMS, nvfp4_gemm.W4A16_MIN_M
    try:
        monkeypatch.setenv("NVFP4_FP8", "1")
        adallm_b200.install()
        assert nvfp4_gemm.REFERENCE_FP8_REQUESTED is True and nvfp4_gemm.DEFAULT_TERMS == terms
        assert nvfp4_gemm.W4A16_MIN_M == min_m
        monkeypatch.setenv("NVFP4_FP8", "0")
        adallm_b200.install()
        assert nvfp4_gemm.REFERENCE_FP8_REQUESTED is False and nvfp4_gemm.DEFAULT_TERMS == terms
    finally:
        context.use_context_provider(None)


def test_install_routes_the_qwen3_decoder_layer(ref):
    """install() routes Qwen3DecoderLayer.forward through the fused decode layer (fused_layers,
    the default) and keeps the reference's forward for every call it does not cover: a prefill
    context, no context, tensors off the GPU.  fused_layers=False restores the reference's."""
    import torch
    import adallm.architectures.qwen3 as rq
    import adallm_b200
    from adallm_b200 import fused_layer
    from types import SimpleNamespace
    layer_cls = rq.Qwen3DecoderLayer
    adallm_b200.install()
    orig = layer_cls._adallm_ref_forward
    assert layer_cls.forward.__name__ == "layer_forward"
    x = torch.zeros(4, 4096, dtype=torch.bfloat16)
    pos = torch.zeros(4, dtype=torch.int64)
    prefill = SimpleNamespace(is_prefill=True, block_tables=None, context_lens=None, slot_mapping=None)
    decode = SimpleNamespace(is_prefill=False, block_tables=torch.zeros((4, 1), dtype=torch.int32),
                             context_lens=torch.ones(4, dtype=torch.int32), slot_mapping=torch.zeros(4, dtype=torch.int32))
    fake_layer = SimpleNamespace()
    assert fused_layer.decode_forward(fake_layer, pos, x, None, prefill) is None
    assert fused_layer.decode_forward(fake_layer, pos, x, None, None) is None
    assert fused_layer.decode_forward(fake_layer, pos, x, None, decode) is None  # CPU tensors
    adallm_b200.install(fused_layers=False)
    assert layer_cls.forward is orig
    adallm_b200.install()
    assert layer_cls.forward.__name__ == "layer_forward" and layer_cls._adallm_ref_forward is orig
    from adallm_b200 import context
    context.use_context_provider(None)
