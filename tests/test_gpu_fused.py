"""Fused producers of the NVFP4 GEMM operand are bit-identical to running the op and
then ada_nvfp4_act_quant on its (rounded) output; the fused decode engine matches the
unfused one."""
import numpy as np
import pytest
import torch

from oracle import attention as oa
from adallm_b200 import _native as N
from adallm_b200.attention import paged_decode
from adallm_b200.layernorm import rms_norm
from adallm_b200.activation import gated_act
from tests.gpu_util import dev

pytestmark = pytest.mark.gpu


def qbufs(m, k, terms, bn, d):
    m_pad = -(-m // bn) * bn
    return (torch.zeros(m_pad * terms * k // 2, dtype=torch.uint8, device=d),
            torch.zeros((m_pad // bn) * (k // 64) * 512, dtype=torch.uint8, device=d),
            torch.zeros(m_pad, dtype=torch.float32, device=d))


def act_quant(x, terms, bn):
    d = x.device
    m, k = x.shape
    xq, sfx, gx = qbufs(m, k, terms, bn, d)
    N.check(N.lib().ada_nvfp4_act_quant(x.data_ptr(), N.DT[x.dtype], x.stride(0), m, k, terms, bn, xq.data_ptr(),
                                        sfx.data_ptr(), gx.data_ptr(), torch.cuda.current_stream().cuda_stream), "aq")
    return xq, sfx, gx


def same(a, b):
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def same_with_bound(got, y_ref, terms, bn):
    """The RMSNorm producers' quantised operand: the row scale comes from a bound on the
    normalised row's amax (rs * max|x w| * (1 + 2^-6)), never below amax / 6 (amax / 2688 for
    one term) and at most ~2.4% above it (the margin over the two bf16 roundings); given that scale, the codes (and block scales) are
    exactly the quantiser's (oracle.nvfp4.quantize_act_terms with the scale as given)."""
    from oracle import nvfp4 as nv
    from tests.test_gpu_nvfp4 import unpack_sf, unpack_xq
    rows, k = y_ref.shape
    m_tiles = -(-rows // bn)
    yf = y_ref.float().cpu().numpy()
    amax = np.abs(yf).max(axis=1)
    div = 2688.0 if terms == 1 else 6.0
    gx = got[2].cpu().numpy()[:rows]
    min_amax = np.float32(2.0 ** -64)  # rows whose (bound on the) amax is below it quantise to zero, scale 1
    live = amax >= min_amax
    dead = amax * 1.025 < min_amax
    assert np.all(gx[live] >= amax[live] / div * (1 - 2.0 ** -20))
    assert np.all(gx[live] <= amax[live] / div * 1.025)
    assert np.all(gx[dead] == 1.0)
    codes, sbits, _ = nv.quantize_act_terms(yf, terms, row_scale=gx)
    got_codes = unpack_xq(got[0].cpu().numpy(), terms, m_tiles, bn, k)
    norm = lambda c: np.where((c & 7) == 0, 0, c)  # +0 / -0 codes decode identically
    np.testing.assert_array_equal(norm(got_codes[:, :rows]), norm(codes))
    if terms == 1:
        np.testing.assert_array_equal(unpack_sf(got[1].cpu().numpy(), m_tiles, bn, k)[:rows], sbits)


@pytest.mark.parametrize("hidden,gemma,with_res", [(4096, False, True), (4096, False, False), (5376, True, True),
                                                   (512, False, True)])
@pytest.mark.parametrize("rows,terms,bn", [(16, 4, 16), (5, 1, 16), (40, 2, 64), (16, 8, 16)])
def test_rmsnorm_quant_matches_unfused(hidden, gemma, with_res, rows, terms, bn):
    d = dev()
    g = torch.Generator(device="cpu").manual_seed(hidden + rows)
    x = (torch.randn((rows, hidden), generator=g) * 3).to(torch.bfloat16).to(d)
    r = torch.randn((rows, hidden), generator=g).to(torch.bfloat16).to(d)
    w = (torch.randn(hidden, generator=g) * 0.1 + (0 if gemma else 1)).to(torch.bfloat16).to(d)
    s = torch.cuda.current_stream().cuda_stream
    if with_res:
        y_ref, r_ref = rms_norm(x, w, 1e-6, r.clone(), gemma=gemma)
    else:
        y_ref = rms_norm(x, w, 1e-6, gemma=gemma)
    got = qbufs(rows, hidden, terms, bn, d)
    y = torch.empty_like(x)
    r2 = r.clone()
    N.check(N.lib().ada_rmsnorm_quant(x.data_ptr(), hidden, r2.data_ptr() if with_res else None, hidden,
                                      r2.data_ptr() if with_res else None, hidden, w.data_ptr(), y.data_ptr(), hidden,
                                      rows, hidden, 1e-6, int(gemma), 0, terms, bn, got[0].data_ptr(),
                                      got[1].data_ptr(), got[2].data_ptr(), s), "rmsnorm_quant")
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    if with_res:
        assert torch.equal(r2, r_ref)
    same_with_bound(got, y_ref, terms, bn)


@pytest.mark.parametrize("gemma", [False, True])
def test_rmsnorm_quant_amax_edge_rows(gemma):
    """The bound on the normalised row amax travels with the sum of squares (one exchange): a
    constant row, ties of the maximum across CTAs, an all-zero row, rows near the bottom and the
    top of the range, one huge outlier, zero norm weights, and ordinary rows all get a row scale
    within the bound's margin and exactly the quantiser's codes for it."""
    d = dev()
    H, rows, terms, bn = 4096, 16, 4, 16
    g = torch.Generator(device="cpu").manual_seed(21)
    x = torch.randn((rows, H), generator=g)
    x[0] = 1.5
    x[1] = 0.0
    x[2, ::512] = 9.0  # the same maximum in every CTA's slice
    x[3] *= 1e-30
    x[4] *= 1e30
    x[5, 1234] = 3.0e4
    x[6] = torch.where(torch.arange(H) % 2 == 0, 2.0, -2.0)
    x = x.to(torch.bfloat16).to(d)
    w = (torch.randn(H, generator=g) * 0.1 + (0 if gemma else 1)).to(torch.bfloat16)
    w[:8] = 0.0
    w = w.to(d)
    s = torch.cuda.current_stream().cuda_stream
    y_ref = rms_norm(x, w, 1e-6, gemma=gemma)
    got = qbufs(rows, H, terms, bn, d)
    y = torch.empty_like(x)
    N.check(N.lib().ada_rmsnorm_quant(x.data_ptr(), H, None, H, None, H, w.data_ptr(), y.data_ptr(), H, rows, H,
                                      1e-6, int(gemma), 0, terms, bn, got[0].data_ptr(), got[1].data_ptr(),
                                      got[2].data_ptr(), s), "rmsnorm_quant")
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    same_with_bound(got, y_ref, terms, bn)


@pytest.mark.parametrize("inter,act,terms", [(12288, 0, 4), (1536, 0, 1), (3072, 1, 4), (21504, 1, 6)])
def test_gated_act_quant_matches_unfused(inter, act, terms):
    d = dev()
    x = (torch.randn((16, 2 * inter), device=d) * 2).to(torch.bfloat16)
    y_ref = gated_act(x, act)
    ref = act_quant(y_ref, terms, 16)
    got = qbufs(16, inter, terms, 16, d)
    y = torch.empty_like(y_ref)
    N.check(N.lib().ada_gated_act_quant(x.data_ptr(), 2 * inter, y.data_ptr(), inter, 16, inter, act, 0, terms, 16,
                                        got[0].data_ptr(), got[1].data_ptr(), got[2].data_ptr(),
                                        torch.cuda.current_stream().cuda_stream), "gated_act_quant")
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    same(got, ref)


@pytest.mark.parametrize("flags", [0, 1])
@pytest.mark.parametrize("batch,hq,hkv,terms,ctx_hi", [(16, 32, 8, 4, 900), (7, 16, 2, 1, 900), (16, 64, 8, 5, 900),
                                                       (16, 32, 8, 4, 5000), (3, 16, 2, 4, 3000)])
def test_paged_decode_quant_matches_unfused(batch, hq, hkv, terms, ctx_hi, flags):
    """Short caches (one fused kernel) and long ones (split kernel, whose split length is worked
    out before the launch wait under ADA_ATTN_META_EARLY, then merge + quantise)."""
    d = dev()
    case = oa.make_paged_case(5, batch=batch, hq=hq, hkv=hkv, d=128, page=16, ctx_lo=1, ctx_hi=ctx_hi)
    q = torch.from_numpy(case["q"]).to(torch.bfloat16).to(d)
    k = torch.from_numpy(case["k"]).to(d).view(torch.float8_e4m3fn)
    v = torch.from_numpy(case["v"]).to(d).view(torch.float8_e4m3fn)
    bt = torch.from_numpy(case["block_tables"]).to(d)
    ctx = torch.from_numpy(case["context_lens"]).to(d)
    out_ref = paged_decode(q, k, v, bt, ctx, case["scale"])
    ref = act_quant(out_ref.view(batch, hq * 128), terms, 16)
    got = qbufs(batch, hq * 128, terms, 16, d)
    out = torch.empty_like(out_ref)
    wsb = int(N.lib().ada_fp8_paged_decode_workspace_size(batch, hq, bt.shape[1], 16, 128))
    ws = torch.empty(wsb, dtype=torch.uint8, device=d)
    # flags 1 (ADA_ATTN_META_EARLY): metadata read before the programmatic-launch wait, same result
    N.check(N.lib().ada_fp8_paged_decode_quant_ex(
        q.data_ptr(), 0, q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
        k.shape[0], bt.data_ptr(), bt.stride(0), bt.shape[1], ctx.data_ptr(), batch, hq, hkv, 128, 16,
        case["scale"], 1.0, 1.0, 0, out.data_ptr(), 0, terms, 16, got[0].data_ptr(), got[1].data_ptr(),
        got[2].data_ptr(), ws.data_ptr(), wsb, flags, torch.cuda.current_stream().cuda_stream), "decode_quant")
    torch.cuda.synchronize()
    assert torch.equal(out, out_ref)
    same(got, ref)


def test_fused_engine_matches_unfused():
    """The fused engine (quantisers inside the producers) against the unfused one (plain op, then
    ada_nvfp4_act_quant) on the same weights and tokens."""
    from tests.decode_check import small_config
    from adallm_b200.decode_step import Qwen3DecodeEngine, DecodeSession
    d = dev()
    logits = []
    for fused in (True, False):
        eng = Qwen3DecodeEngine(small_config(3), d, 4, max_ctx=32, seed=7, fused=fused)
        sess = DecodeSession(eng, seed=7)
        outs = []
        for step in range(5):  # teacher-forced: both engines see the same tokens every step
            sess.prepare(torch.tensor([(7 * step + 3 * i + 1) % 1000 for i in range(4)]))
            sess.upload()
            eng.forward()
            sess.download()
            sess.commit()
            outs.append(eng.logits.clone())
        logits.append(torch.stack(outs))
    # the fused RMSNorm producers take their row scale from a bound on the amax (<= 2.4% above
    # it), the unfused path from the exact amax: the operands differ at the quantiser's noise,
    # which the e4m3 KV cache amplifies to the level the engine shows against the exact oracle
    # (~0.03 logits rel-L2 in the agreement tests)
    a, b = logits[0].float(), logits[1].float()
    rel = [float((a[i] - b[i]).norm() / b[i].norm()) for i in range(a.shape[0])]
    print("fused vs unfused logits rel-L2 per step", rel)
    assert max(rel) < 5e-2 and sum(rel) / len(rel) < 3e-2, rel


def test_pdl_toggle_gives_identical_results():
    from tests.decode_check import small_config
    from adallm_b200.decode_step import Qwen3DecodeEngine, DecodeSession
    d = dev()
    res = []
    for pdl in (1, 0):
        prev = N.lib().ada_set_pdl(pdl)
        try:
            eng = Qwen3DecodeEngine(small_config(2), d, 4, max_ctx=32, seed=3)
            sess = DecodeSession(eng, seed=3)
            g = eng.capture()
            sess.prepare(torch.tensor([5, 6, 7, 8]))
            sess.upload()
            g.replay()
            torch.cuda.synchronize()
            res.append(eng.logits.clone())
            del g
        finally:
            N.lib().ada_set_pdl(prev)
    assert torch.equal(res[0], res[1])


# ---- split-K partial planes: GEMM leaves fp32 planes, the next kernel sums them ------------------
def _rand_weight(n, k, d, seed):
    from adallm_b200.decode_step import random_nvfp4
    from adallm_b200.nvfp4_gemm import prepack_scales
    packed, scale, s2 = random_nvfp4(n, k, seed, d)
    return packed, prepack_scales(scale, n, k), torch.tensor(s2, dtype=torch.float32, device=d)


def _gemm_partials(xq, sfx, gx, m, terms, bn, w, n, k, d):
    ns = int(N.lib().ada_nvfp4_gemm_splits(m, n, k, terms))
    assert 1 <= ns <= 8
    parts = torch.full((ns, m, n), float("nan"), dtype=torch.float32, device=d)
    ws = torch.zeros(256, dtype=torch.uint8, device=d)
    N.check(N.lib().ada_nvfp4_gemm_partials(xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), m, terms, bn,
                                            w[0].data_ptr(), w[0].stride(0), w[1].data_ptr(), w[2].data_ptr(), n, k,
                                            parts.data_ptr(), n, m * n, ns, ws.data_ptr(), 256,
                                            torch.cuda.current_stream().cuda_stream), "gemm_partials")
    return parts, ns


def _gemm_reduced(xq, sfx, gx, m, terms, bn, w, n, k, ns, d):
    y = torch.empty((m, n), dtype=torch.bfloat16, device=d)
    ws = torch.zeros(256, dtype=torch.uint8, device=d)
    N.check(N.lib().ada_nvfp4_gemm(xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), m, terms, bn, w[0].data_ptr(),
                                   w[0].stride(0), w[1].data_ptr(), w[2].data_ptr(), n, k, None, y.data_ptr(), 0, n,
                                   ns, ws.data_ptr(), 256, torch.cuda.current_stream().cuda_stream), "gemm")
    return y


def _plane_sum(parts):
    acc = parts[0].clone()
    for p in parts[1:]:
        acc = acc + p  # fp32, plane order
    return acc.to(torch.bfloat16)


@pytest.mark.parametrize("m,n,k", [(16, 6144, 4096), (16, 4096, 12288), (16, 24576, 4096), (5, 512, 1024)])
def test_gemm_partials_sum_to_reduced_gemm(m, n, k):
    d = dev()
    terms, bn = 4, int(N.lib().ada_nvfp4_block_n(m, 4))
    x = torch.randn((m, k), device=d, dtype=torch.bfloat16)
    xq, sfx, gx = act_quant(x, terms, bn)
    w = _rand_weight(n, k, d, n + k)
    parts, ns = _gemm_partials(xq, sfx, gx, m, terms, bn, w, n, k, d)
    torch.cuda.synchronize()
    assert not torch.isnan(parts).any()
    y = _gemm_reduced(xq, sfx, gx, m, terms, bn, w, n, k, ns, d)
    assert torch.equal(_plane_sum(parts), y)


def test_parts_consumers_match_plain_ops():
    d = dev()
    s = torch.cuda.current_stream().cuda_stream
    m, H, I, terms, bn = 16, 4096, 12288, 4, 16
    g = torch.Generator(device="cpu").manual_seed(11)
    # RMSNorm + residual from planes
    parts = (torch.randn((3, m, H), generator=g) * 2).to(d)
    x = _plane_sum(parts)
    res = torch.randn((m, H), generator=g).to(torch.bfloat16).to(d)
    w = (torch.randn(H, generator=g) * 0.1 + 1).to(torch.bfloat16).to(d)
    r1, r2 = res.clone(), res.clone()
    ref = qbufs(m, H, terms, bn, d)
    got = qbufs(m, H, terms, bn, d)
    N.check(N.lib().ada_rmsnorm_quant(x.data_ptr(), H, r1.data_ptr(), H, r1.data_ptr(), H, w.data_ptr(), None, 0, m,
                                      H, 1e-6, 0, 0, terms, bn, ref[0].data_ptr(), ref[1].data_ptr(),
                                      ref[2].data_ptr(), s), "rmsq")
    N.check(N.lib().ada_rmsnorm_quant_parts(parts.data_ptr(), 3, m * H, H, r2.data_ptr(), H, r2.data_ptr(), H,
                                            w.data_ptr(), None, 0, m, H, 1e-6, 0, 0, terms, bn, got[0].data_ptr(),
                                            got[1].data_ptr(), got[2].data_ptr(), s), "rmsq_parts")
    y1, y2 = torch.empty_like(x), torch.empty_like(x)
    r3, r4 = res.clone(), res.clone()
    N.check(N.lib().ada_rmsnorm(x.data_ptr(), H, r3.data_ptr(), H, r3.data_ptr(), H, w.data_ptr(), y1.data_ptr(), H,
                                m, H, 1e-6, 0, 0, s), "rms")
    N.check(N.lib().ada_rmsnorm_quant_parts(parts.data_ptr(), 3, m * H, H, r4.data_ptr(), H, r4.data_ptr(), H,
                                            w.data_ptr(), y2.data_ptr(), H, m, H, 1e-6, 0, 0, terms, bn, None, None,
                                            None, s), "rms_parts_plain")
    torch.cuda.synchronize()
    same(got, ref)
    assert torch.equal(r1, r2) and torch.equal(y1, y2) and torch.equal(r3, r4)
    # SiLU * up from planes
    parts = (torch.randn((1, m, 2 * I), generator=g) * 2).to(d)
    x = _plane_sum(parts)
    ref = act_quant(gated_act(x, 0), terms, bn)
    got = qbufs(m, I, terms, bn, d)
    N.check(N.lib().ada_gated_act_quant_parts(parts.data_ptr(), 1, m * 2 * I, 2 * I, None, 0, m, I, 0, 0, terms, bn,
                                              got[0].data_ptr(), got[1].data_ptr(), got[2].data_ptr(), s), "act_parts")
    torch.cuda.synchronize()
    same(got, ref)


def test_qk_norm_rope_store_from_planes():
    from adallm_b200.rotary_embedding import build_cos_sin_cache
    d = dev()
    s = torch.cuda.current_stream().cuda_stream
    T, hq, hkv, D = 7, 32, 8, 128
    width = (hq + 2 * hkv) * D
    g = torch.Generator(device="cpu").manual_seed(5)
    parts = torch.randn((4, T, width), generator=g).to(d)
    qkv = _plane_sum(parts)
    qw = (torch.randn(D, generator=g) * 0.1 + 1).to(torch.bfloat16).to(d)
    kw = (torch.randn(D, generator=g) * 0.1 + 1).to(torch.bfloat16).to(d)
    pos = torch.randint(0, 100, (T,), generator=g).to(d)
    cs = build_cos_sin_cache(D, 128, 1e6, None, d).contiguous()
    slots = torch.arange(T, dtype=torch.int32, device=d) * 3
    out = []
    for use_parts in (False, True):
        kc = torch.zeros((64, 1, hkv, D), dtype=torch.uint8, device=d)
        vc = torch.zeros_like(kc)
        q = torch.empty((T, hq, D), dtype=torch.bfloat16, device=d)
        if use_parts:
            st = N.lib().ada_qk_norm_rope_store_parts(parts.data_ptr(), 4, T * width, width, T, hq, hkv, D,
                                                      qw.data_ptr(), kw.data_ptr(), 1e-6, pos.data_ptr(),
                                                      cs.data_ptr(), cs.shape[0], slots.data_ptr(), kc.data_ptr(),
                                                      vc.data_ptr(), 1.0, 1.0, q.data_ptr(), None, 0, s)
        else:
            st = N.lib().ada_qk_norm_rope_store(qkv.data_ptr(), width, T, hq, hkv, D, qw.data_ptr(), kw.data_ptr(),
                                                1e-6, pos.data_ptr(), cs.data_ptr(), cs.shape[0], slots.data_ptr(),
                                                kc.data_ptr(), vc.data_ptr(), 1.0, 1.0, q.data_ptr(), None, 0, s)
        N.check(st, "qk")
        out.append((q, kc, vc))
    torch.cuda.synchronize()
    for a, b in zip(out[0], out[1]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("m,with_res", [(16, True), (5, True), (16, False)])
def test_rmsnorm_quant_combine_matches_combine_then_rmsnorm(m, with_res):
    """The MoE block's weighted combine folded into the next RMSNorm (ada_rmsnorm_quant_combine)
    equals ada_moe_combine followed by ada_rmsnorm_quant bit for bit (quantised operand, new
    residual) and, without a quantised output, ada_moe_combine + ada_rmsnorm (config-4 widths)."""
    d = dev()
    s = torch.cuda.current_stream().cuda_stream
    H, k, terms, bn = 2048, 8, 4, 16
    g = torch.Generator(device="cpu").manual_seed(12)
    y_rows = torch.randn((m * k, H), generator=g).to(torch.bfloat16).to(d)
    rw = torch.rand((m, k), generator=g).to(torch.bfloat16).to(d)
    res = torch.randn((m, H), generator=g).to(torch.bfloat16).to(d)
    w = (torch.randn(H, generator=g) * 0.1 + 1).to(torch.bfloat16).to(d)
    hidden = torch.empty((m, H), dtype=torch.bfloat16, device=d)
    N.check(N.lib().ada_moe_combine(y_rows.data_ptr(), 0, H, rw.data_ptr(), m, k, H, hidden.data_ptr(), H, s),
            "combine")
    r1, r2 = res.clone(), res.clone()
    rp1 = r1.data_ptr() if with_res else None
    rp2 = r2.data_ptr() if with_res else None
    ref, got = qbufs(m, H, terms, bn, d), qbufs(m, H, terms, bn, d)
    N.check(N.lib().ada_rmsnorm_quant(hidden.data_ptr(), H, rp1, H, rp1, H, w.data_ptr(), None, 0, m, H, 1e-6, 0, 0,
                                      terms, bn, ref[0].data_ptr(), ref[1].data_ptr(), ref[2].data_ptr(), s), "rmsq")
    N.check(N.lib().ada_rmsnorm_quant_combine(y_rows.data_ptr(), H, rw.data_ptr(), k, rp2, H, rp2, H, w.data_ptr(),
                                              None, 0, m, H, 1e-6, 0, 0, terms, bn, got[0].data_ptr(),
                                              got[1].data_ptr(), got[2].data_ptr(), s), "rmsq_combine")
    y1, y2 = torch.empty_like(hidden), torch.empty_like(hidden)
    r3, r4 = res.clone(), res.clone()
    N.check(N.lib().ada_rmsnorm(hidden.data_ptr(), H, r3.data_ptr(), H, r3.data_ptr(), H, w.data_ptr(), y1.data_ptr(),
                                H, m, H, 1e-6, 0, 0, s), "rms")
    N.check(N.lib().ada_rmsnorm_quant_combine(y_rows.data_ptr(), H, rw.data_ptr(), k, r4.data_ptr(), H, r4.data_ptr(),
                                              H, w.data_ptr(), y2.data_ptr(), H, m, H, 1e-6, 0, 0, terms, bn, None,
                                              None, None, s), "rms_combine_plain")
    torch.cuda.synchronize()
    same(got, ref)
    assert torch.equal(r1, r2) and torch.equal(y1, y2) and torch.equal(r3, r4)
