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
    ref = act_quant(y_ref, terms, bn)
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
    same(got, ref)


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


@pytest.mark.parametrize("batch,hq,hkv,terms", [(16, 32, 8, 4), (7, 16, 2, 1), (16, 64, 8, 5)])
def test_paged_decode_quant_matches_unfused(batch, hq, hkv, terms):
    d = dev()
    case = oa.make_paged_case(5, batch=batch, hq=hq, hkv=hkv, d=128, page=16, ctx_lo=1, ctx_hi=900)
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
    N.check(N.lib().ada_fp8_paged_decode_quant(
        q.data_ptr(), 0, q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
        k.shape[0], bt.data_ptr(), bt.stride(0), bt.shape[1], ctx.data_ptr(), batch, hq, hkv, 128, 16,
        case["scale"], 1.0, 1.0, 0, out.data_ptr(), 0, terms, 16, got[0].data_ptr(), got[1].data_ptr(),
        got[2].data_ptr(), ws.data_ptr(), wsb, torch.cuda.current_stream().cuda_stream), "decode_quant")
    torch.cuda.synchronize()
    assert torch.equal(out, out_ref)
    same(got, ref)


def test_fused_engine_matches_unfused():
    from tests.decode_check import small_config
    from adallm_b200.decode_step import Qwen3DecodeEngine, DecodeSession
    d = dev()
    logits = []
    for fused in (True, False):
        eng = Qwen3DecodeEngine(small_config(3), d, 4, max_ctx=32, seed=7, fused=fused)
        sess = DecodeSession(eng, seed=7)
        toks = torch.tensor([1, 2, 3, 4])
        outs = []
        for _ in range(5):
            sess.prepare(toks)
            sess.upload()
            eng.forward()
            toks = sess.download()
            sess.commit()
            outs.append(eng.logits.clone())
        logits.append(torch.stack(outs))
    assert torch.equal(logits[0], logits[1])


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
