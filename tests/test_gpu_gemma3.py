"""Gemma3 on the B200.

* ada_gemma_norm2_quant_parts -- post-norm of the projection's partial planes, residual add,
  pre-norm and quantisation in one kernel -- is bit-identical to the composition of the plain
  kernels (GemmaRMSNorm without residual, then GemmaRMSNorm with residual, then act-quant).
* ada_qk_norm_rope_store[_parts]_ex with the Gemma per-head norm: the planes form equals the
  bf16 form bit for bit, and both match the CPU oracle (GemmaRMSNorm then RoPE) within 2 bf16
  ulps, with the same K/V bytes in the cache wherever the rotated k agrees.
* The whole Gemma3 decode step (engine, CUDA graph) against the CPU oracle decoder, teacher-forced:
  full widths (hidden 5376, 32/16 heads, GeGLU 21504, vocab 262208), 6 layers (5 local + 1
  global, window 64 so the 144-token contexts cross it), batch 4, 128 generated tokens; the same
  criteria as the Qwen3 agreement test (tests/test_gpu_decode.py)."""
import numpy as np
import pytest
import torch

from adallm_b200 import _native as N
from adallm_b200.layernorm import rms_norm
from tests.gpu_util import dev
from tests.test_gpu_fused import qbufs, same_with_bound

pytestmark = pytest.mark.gpu


def _plane_sum(parts):
    s = parts[0].clone()
    for i in range(1, parts.shape[0]):
        s = s + parts[i]
    return s.to(torch.bfloat16)


@pytest.mark.parametrize("rows,hidden,terms,quant", [(4, 5376, 4, True), (16, 4096, 1, True), (3, 5376, 4, False)])
def test_gemma_norm2_matches_composition(rows, hidden, terms, quant):
    d = dev()
    g = torch.Generator(device="cpu").manual_seed(rows + hidden)
    ns = 3
    parts = (torch.randn((ns, rows, hidden), generator=g) * 2).to(d)
    res = torch.randn((rows, hidden), generator=g).to(torch.bfloat16).to(d)
    wpost = (torch.randn(hidden, generator=g) * 0.1).to(torch.bfloat16).to(d)
    w = (torch.randn(hidden, generator=g) * 0.1).to(torch.bfloat16).to(d)
    h = rms_norm(_plane_sum(parts), wpost, 1e-6, gemma=True)
    y_ref, r_ref = rms_norm(h, w, 1e-6, res.clone(), gemma=True)
    r2 = res.clone()
    y = torch.empty_like(res)
    got = qbufs(rows, hidden, terms, 16, d) if quant else (None, None, None)
    st = N.lib().ada_gemma_norm2_quant_parts(parts.data_ptr(), ns, rows * hidden, hidden, wpost.data_ptr(),
                                             r2.data_ptr(), hidden, r2.data_ptr(), hidden, w.data_ptr(), y.data_ptr(),
                                             hidden, rows, hidden, 1e-6, 0, terms, 16, N.ptr(got[0]), N.ptr(got[1]),
                                             N.ptr(got[2]), torch.cuda.current_stream().cuda_stream)
    N.check(st, "gemma norm2")
    torch.cuda.synchronize()
    assert torch.equal(r2, r_ref)
    assert torch.equal(y, y_ref)
    if quant:
        same_with_bound(got, y_ref, terms, 16)


def test_qk_norm_gemma_planes_and_oracle():
    from adallm_b200.rotary_embedding import build_cos_sin_cache
    from oracle import layers as ol
    from oracle.nvfp4 import e4m3_encode
    d = dev()
    s = torch.cuda.current_stream().cuda_stream
    T, hq, hkv, D = 5, 32, 16, 128
    width = (hq + 2 * hkv) * D
    g = torch.Generator(device="cpu").manual_seed(9)
    parts = torch.randn((2, T, width), generator=g).to(d)
    qkv = _plane_sum(parts)
    qw = (torch.randn(D, generator=g) * 0.1).to(torch.bfloat16).to(d)
    kw = (torch.randn(D, generator=g) * 0.1).to(torch.bfloat16).to(d)
    pos = torch.randint(0, 1000, (T,), generator=g).to(d)
    cs = build_cos_sin_cache(D, 1024, 1e4, None, d).contiguous()
    slots = torch.arange(T, dtype=torch.int32, device=d) * 2
    out = []
    for use_parts in (False, True):
        kc = torch.zeros((16, 1, hkv, D), dtype=torch.uint8, device=d)
        vc = torch.zeros_like(kc)
        q = torch.empty((T, hq, D), dtype=torch.bfloat16, device=d)
        k = torch.empty((T, hkv, D), dtype=torch.bfloat16, device=d)
        if use_parts:
            st = N.lib().ada_qk_norm_rope_store_parts_ex(parts.data_ptr(), 2, T * width, width, T, hq, hkv, D,
                                                         qw.data_ptr(), kw.data_ptr(), 1e-6, 1, pos.data_ptr(),
                                                         cs.data_ptr(), cs.shape[0], slots.data_ptr(), kc.data_ptr(),
                                                         vc.data_ptr(), 1.0, 1.0, q.data_ptr(), k.data_ptr(), 0, s)
        else:
            st = N.lib().ada_qk_norm_rope_store_ex(qkv.data_ptr(), width, T, hq, hkv, D, qw.data_ptr(), kw.data_ptr(),
                                                   1e-6, 1, pos.data_ptr(), cs.data_ptr(), cs.shape[0],
                                                   slots.data_ptr(), kc.data_ptr(), vc.data_ptr(), 1.0, 1.0,
                                                   q.data_ptr(), k.data_ptr(), 0, s)
        N.check(st, "qk gemma")
        out.append((q, k, kc, vc))
    torch.cuda.synchronize()
    for a, b in zip(out[0], out[1]):
        assert torch.equal(a, b)
    # CPU oracle: GemmaRMSNorm per head (layernorm.py:64-74), then RoPE (rotary_embedding.py:6-14)
    x = qkv.cpu()
    qr = ol.gemma_rms_norm(x[:, :hq * D].reshape(T, hq, D), qw.cpu(), 1e-6)
    kr = ol.gemma_rms_norm(x[:, hq * D:(hq + hkv) * D].reshape(T, hkv, D), kw.cpu(), 1e-6)
    qr, kr = ol.apply_rope(pos.cpu(), qr, kr, cs.cpu())
    q, k, kc, vc = out[0]
    # 2 bf16 ulps of the value, plus 2 ulps at the head's unit scale for rotated pairs that cancel
    ulp = lambda t: torch.clamp(t.float().abs(), min=1e-30).log2().floor().exp2() * 2.0 ** -7
    tol = lambda t: 2 * ulp(t) + 2.0 ** -7
    assert bool(((q.cpu().float() - qr.float()).abs() <= tol(qr)).all())
    assert bool(((k.cpu().float() - kr.float()).abs() <= tol(kr)).all())
    same_k = (k.cpu() == kr)
    want = e4m3_encode(kr.float().numpy().reshape(T, -1))
    got = kc.cpu().numpy().reshape(16, -1)[slots.cpu().numpy()]
    assert np.array_equal(got.reshape(T, hkv, D)[same_k.numpy()], want.reshape(T, hkv, D)[same_k.numpy()])
    v_want = e4m3_encode(x[:, (hq + hkv) * D:].float().numpy())
    assert np.array_equal(vc.cpu().numpy().reshape(16, -1)[slots.cpu().numpy()], v_want)


def test_gemma3_decode_agreement_128_steps():
    from tests.decode_check import gemma3_test_config, run_agreement_gemma3
    from tests.test_gpu_decode import _report
    r = run_agreement_gemma3(gemma3_test_config(6, window=64), steps=127, batch=4, prompt=16, graph=True,
                             emulate=True)
    _report("gemma3_full_width_bs4", r)
    assert r.raw >= min(0.99, r.raw_reference - r.margin()), r
    assert r.logits_rel_l2_mean <= 1.25 * max(r.ref_logits_rel_l2_mean, 1e-3), r
    assert r.logits_rel_l2_max < 5e-2, r
