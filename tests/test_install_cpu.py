"""The drop-in shim against the real reference package (CPU: import and patch only;
no kernel runs).  Skipped where the reference checkout is absent (the GPU box)."""
import inspect
import os
import sys

import pytest

REF = os.environ.get("ADALLM_REF", "/root/reference")


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
        calls.clear()
        rc.set_context(True, cu_q, cu_q, 5, 5, torch.arange(5, dtype=torch.int32), None, None)
        with pytest.raises(Exception):  # the reference branch (flash-attn) cannot run on CPU
            m.forward(q, kv, kv)
        assert all(c == "store" for c in calls)
    finally:
        rc.reset_context()
        context.use_context_provider(None)


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
