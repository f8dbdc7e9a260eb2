"""KV store / RMSNorm / RoPE / gated activation / embedding / argmax kernels vs
the CPU oracle.  KV store is bit-exact; the floating-point ops are compared in
bf16 ulps (the reference's eager rounding order is reproduced; only reduction
order and transcendental implementations may differ)."""
import numpy as np
import pytest
import torch

from oracle import attention as oa
from oracle import layers as ol
from oracle import nvfp4 as nv
from adallm_b200.attention import store_kvcache
from adallm_b200.layernorm import rms_norm, RMSNorm, GemmaRMSNorm
from adallm_b200.rotary_embedding import RotaryEmbedding, build_cos_sin_cache, apply_rope
from adallm_b200.activation import gated_act
from adallm_b200 import _native as N
from tests.gpu_util import dev, rel_l2, u8, bf16_ulp_mismatch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("k_scale,v_scale", [(1.0, 1.0), (0.5, 3.0)])
def test_store_kvcache_bit_exact(dtype, k_scale, v_scale):
    d = dev()
    g = torch.Generator().manual_seed(0)
    t, hkv, hd, pages, page = 37, 8, 128, 12, 16
    key = (torch.randn((t, hkv, hd), generator=g) * 100).to(dtype)  # exercises saturation at 448
    val = torch.randn((t, hkv, hd), generator=g).to(dtype)
    slots = torch.randperm(pages * page, generator=g)[:t].to(torch.int32)
    slots[3] = -1
    slots[20] = -1
    kc = torch.zeros((pages, page, hkv, hd), dtype=torch.uint8)
    vc = torch.zeros_like(kc)
    kc_d, vc_d = kc.to(d).view(torch.float8_e4m3fn), vc.to(d).view(torch.float8_e4m3fn)
    store_kvcache(key.to(d), val.to(d), kc_d, vc_d, slots.to(d), k_scale, v_scale)
    torch.cuda.synchronize()
    kref, vref = kc.numpy().copy(), vc.numpy().copy()
    oa.store_kvcache(key.float().numpy(), val.float().numpy(), kref, vref, slots.numpy(), k_scale, v_scale)
    np.testing.assert_array_equal(u8(kc_d), kref)
    np.testing.assert_array_equal(u8(vc_d), vref)


@pytest.mark.parametrize("hidden", [128, 4096, 5376])
@pytest.mark.parametrize("gemma", [False, True])
@pytest.mark.parametrize("with_res", [False, True])
def test_rmsnorm(hidden, gemma, with_res):
    d = dev()
    g = torch.Generator().manual_seed(hidden)
    x = (torch.randn((19, hidden), generator=g) * 2).to(torch.bfloat16)
    r = torch.randn((19, hidden), generator=g).to(torch.bfloat16)
    w = ((0.1 if gemma else 1.0) * torch.randn((hidden,), generator=g) + (0 if gemma else 1)).to(torch.bfloat16)
    if with_res:
        y, res = rms_norm(x.to(d), w.to(d), 1e-6, r.to(d), gemma=gemma)
        fn = ol.gemma_add_rms_norm if gemma else ol.add_rms_norm
        y_ref, res_ref = fn(x, r, w, 1e-6)
        assert torch.equal(res.cpu(), res_ref)
    else:
        y = rms_norm(x.to(d), w.to(d), 1e-6, gemma=gemma)
        y_ref = (ol.gemma_rms_norm if gemma else ol.rms_norm)(x, w, 1e-6)
    # a 1-ulp difference of the normalised value (rsqrt / reduction order) can become
    # 2 ulps after the bf16 weight multiply of the Qwen variant
    frac, mx = bf16_ulp_mismatch(y.cpu(), y_ref)
    assert mx <= 2 and frac < 0.01, (frac, mx)
    assert rel_l2(y.float().cpu(), y_ref.float()) < 1e-3


def test_norm_modules_per_head():
    d = dev()
    m = RMSNorm(128).to(d).to(torch.bfloat16)
    x = torch.randn(16, 32, 128, device=d, dtype=torch.bfloat16)
    y = m(x)
    assert y.shape == x.shape
    frac, mx = bf16_ulp_mismatch(y.cpu(), ol.rms_norm(x.cpu(), m.weight.cpu(), 1e-6))
    assert mx <= 2 and frac < 0.01
    gm = GemmaRMSNorm(256).to(d).to(torch.bfloat16)
    x2 = torch.randn(3, 256, device=d, dtype=torch.bfloat16)
    y2, r2 = gm(x2, x2)
    assert torch.equal(r2.cpu(), (x2 + x2).cpu())


@pytest.mark.parametrize("scaling", [None, {"rope_type": "linear", "factor": 8.0}])
def test_rope_exact(scaling):
    d = dev()
    rope = RotaryEmbedding(128, 128, 4096, 1e6, scaling).to(d)
    cache_cpu = ol.rope_cache(128, 4096, 1e6, scaling)
    assert torch.equal(rope.cos_sin_cache.cpu(), cache_cpu)
    pos = torch.tensor([0, 1, 5, 77, 4095, 1000, 3], dtype=torch.long)
    q = torch.randn(7, 32, 128).to(torch.bfloat16)
    k = torch.randn(7, 8, 128).to(torch.bfloat16)
    qo, ko = rope(pos.to(d), q.to(d), k.to(d))
    qr, kr = ol.apply_rope(pos, q, k, cache_cpu)
    assert torch.equal(qo.cpu(), qr) and torch.equal(ko.cpu(), kr)


def test_rope_strided_qkv_views():
    d = dev()
    cache = build_cos_sin_cache(128, 512, 1e6, None, d)
    qkv = torch.randn(5, (32 + 16) * 128, device=d, dtype=torch.bfloat16)
    q = qkv[:, :32 * 128].view(5, 32, 128)
    k = qkv[:, 32 * 128:40 * 128].view(5, 8, 128)
    pos = torch.arange(5, device=d)
    qo, ko = apply_rope(pos, q, k, cache)
    qr, kr = ol.apply_rope(pos.cpu(), q.cpu(), k.cpu(), cache.cpu())
    assert torch.equal(qo.cpu(), qr) and torch.equal(ko.cpu(), kr)


@pytest.mark.parametrize("act", [0, 1])
def test_gated_act(act):
    d = dev()
    x = (torch.randn(17, 2 * 1536) * 3).to(torch.bfloat16)
    y = gated_act(x.to(d), act)
    y_ref = (ol.silu_and_mul if act == 0 else ol.gelu_and_mul)(x)
    # the activation's transcendental differs by ~1 fp32 ulp, which can move the bf16 activation by
    # one ulp before the product rounds again (<= 2 bf16 ulps); GELU's far tail is ~0 either side of zero
    assert torch.allclose(y.float().cpu(), y_ref.float(), rtol=2 ** -6, atol=1e-5)
    assert rel_l2(y.float().cpu(), y_ref.float()) < 2e-3


def test_embedding_and_argmax():
    d = dev()
    table = torch.randn(1000, 256, device=d, dtype=torch.bfloat16)
    ids = torch.tensor([0, 999, 5, 5, 400], device=d, dtype=torch.long)
    y = torch.empty(5, 256, device=d, dtype=torch.bfloat16)
    s = torch.cuda.current_stream().cuda_stream
    N.check(N.lib().ada_embedding(ids.data_ptr(), 5, table.data_ptr(), 0, 1000, 256, y.data_ptr(), 0, s), "emb")
    assert torch.equal(y, table[ids])
    # vocab shard [500, 1000): rows outside are zero (adallm/ops/embed_head.py:35-40)
    N.check(N.lib().ada_embedding(ids.data_ptr(), 5, table[500:].data_ptr(), 500, 1000, 256, y.data_ptr(), 0, s),
            "emb")
    assert torch.equal(y[1], table[999]) and torch.all(y[0] == 0)
    logits = torch.randn(6, 151936, device=d, dtype=torch.bfloat16)
    logits[2, 17] = 100.0
    logits[2, 99] = 100.0  # first maximum wins
    out = torch.empty(6, device=d, dtype=torch.long)
    ws = torch.empty(N.lib().ada_argmax_workspace_size(6, 151936), dtype=torch.uint8, device=d)
    N.check(N.lib().ada_argmax(logits.data_ptr(), 151936, 6, 151936, 0, out.data_ptr(), ws.data_ptr(), ws.numel(), s),
            "argmax")
    ref = logits.float().argmax(dim=1)
    assert out[2].item() == 17
    assert torch.equal(out.cpu(), ref.cpu())
    # odd widths / strides take the scalar path
    odd = torch.randn(3, 1001, device=d, dtype=torch.float16)[:, :999]
    N.check(N.lib().ada_argmax(odd.data_ptr(), 1001, 3, 999, 1, out.data_ptr(), ws.data_ptr(), ws.numel(), s),
            "argmax")
    assert torch.equal(out[:3].cpu(), odd.float().argmax(dim=1).cpu())
