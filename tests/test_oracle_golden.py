"""Pin the CPU oracle against golden vectors produced by the reference's own
Python code (tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest
import torch

from oracle import nvfp4 as nv
from oracle import attention as oa
from oracle import layers as ol
from tests.conftest import bf16_from_bits


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_e2m1_lut_matches_reference(golden_dir):
    g = _load(golden_dir, "golden_nvfp4.npz")
    np.testing.assert_array_equal(nv.E2M1_LUT, g["lut"])


def test_dequant_matches_reference(golden_dir):
    g = _load(golden_dir, "golden_nvfp4.npz")
    out = nv.dequant_nvfp4(g["packed"], g["scale_fp16"].astype(np.float32), g["scale_2"])
    np.testing.assert_array_equal(out, g["dequant"])
    # e4m3 scale bits decode to exactly the fp16 values the loader stores
    np.testing.assert_array_equal(nv.e4m3_decode(g["scale_bits"]), g["scale_fp16"].astype(np.float32))


def test_dequant_linear_matches_reference(golden_dir):
    g = _load(golden_dir, "golden_nvfp4.npz")
    x = bf16_from_bits(g["x_bf16"]).float().numpy()
    y = nv.linear_ref(x, g["packed"], g["scale_fp16"].astype(np.float32), g["scale_2"])
    y_ref = bf16_from_bits(g["y_bf16"]).float().numpy()
    # the reference rounds the dequantised weight to bf16 before F.linear
    assert nv.rel_l2(y, y_ref) < 1e-2


def test_e4m3_cast_matches_reference(golden_dir):
    g = _load(golden_dir, "golden_kv.npz")
    vals = bf16_from_bits(g["cast_in_bf16"]).float().numpy()
    np.testing.assert_array_equal(nv.e4m3_encode(vals), g["cast_out_e4m3"])


def test_gather_kv_matches_reference(golden_dir):
    g = _load(golden_dir, "golden_kv.npz")
    kf = nv.e4m3_decode(g["k_cache"]).astype(np.float16)
    vf = nv.e4m3_decode(g["v_cache"]).astype(np.float16)
    k_out, v_out, cu = oa.gather_kv_from_blocks(kf, vf, g["block_tables"], g["context_lens"])
    np.testing.assert_array_equal(k_out, g["k_out"])
    np.testing.assert_array_equal(v_out, g["v_out"])
    np.testing.assert_array_equal(cu, g["cu"])


def test_norms_match_reference(golden_dir):
    g = _load(golden_dir, "golden_layers.npz")
    x, r = bf16_from_bits(g["x"]), bf16_from_bits(g["r"])
    w, wg = bf16_from_bits(g["w"]), bf16_from_bits(g["wg"])
    assert torch.equal(ol.rms_norm(x, w, 1e-6), bf16_from_bits(g["y_rms"]))
    y, res = ol.add_rms_norm(x, r, w, 1e-6)
    assert torch.equal(y, bf16_from_bits(g["y_add"]))
    assert torch.equal(res, bf16_from_bits(g["r_add"]))
    assert torch.equal(ol.gemma_rms_norm(x, wg, 1e-6), bf16_from_bits(g["y_g"]))
    y, res = ol.gemma_add_rms_norm(x, r, wg, 1e-6)
    assert torch.equal(y, bf16_from_bits(g["y_gadd"]))
    assert torch.equal(res, bf16_from_bits(g["r_gadd"]))


def test_rope_matches_reference(golden_dir):
    g = _load(golden_dir, "golden_layers.npz")
    cache = ol.rope_cache(64, 512, 1e6)
    np.testing.assert_array_equal(cache.numpy(), g["cache"])
    cache_lin = ol.rope_cache(64, 512, 1e4, {"rope_type": "linear", "factor": 8.0})
    np.testing.assert_array_equal(cache_lin.numpy(), g["cache_lin"])
    pos = torch.from_numpy(g["pos"])
    q, k = bf16_from_bits(g["q"]), bf16_from_bits(g["k"])
    q1, k1 = ol.apply_rope(pos, q, k, cache)
    assert torch.equal(q1, bf16_from_bits(g["q1"])) and torch.equal(k1, bf16_from_bits(g["k1"]))
    q2, k2 = ol.apply_rope(pos, q, k, cache_lin)
    assert torch.equal(q2, bf16_from_bits(g["q2"])) and torch.equal(k2, bf16_from_bits(g["k2"]))


def test_activations_match_reference(golden_dir):
    g = _load(golden_dir, "golden_layers.npz")
    a = bf16_from_bits(g["a"])
    assert torch.equal(ol.silu_and_mul(a), bf16_from_bits(g["y_silu"]))
    assert torch.equal(ol.gelu_and_mul(a), bf16_from_bits(g["y_gelu"]))


def test_e2m1_round_to_nearest_even():
    v = np.array([0.0, 0.24, 0.25, 0.26, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.1, 7.0, 1e9,
                  -0.75, -5.0, -100.0], np.float32)
    want = np.array([0, 0, 0, 1, 2, 2, 4, 4, 6, 6, 7, 7, 7, 8 | 2, 8 | 6, 8 | 7], np.uint8)
    np.testing.assert_array_equal(nv.e2m1_encode(v), want)


def test_e4m3_saturates_and_rounds():
    v = np.array([448.0, 464.0, 470.0, 1e6, -1e6, 2.0 ** -9, 2.0 ** -10, 1.5 * 2.0 ** -10, 1.0625, 1.1875], np.float32)
    bits = nv.e4m3_encode(v)
    dec = nv.e4m3_decode(bits)
    np.testing.assert_array_equal(dec, np.array([448, 448, 448, 448, -448, 2.0 ** -9, 0.0, 2.0 ** -9, 1.0, 1.25], np.float32))


def test_paged_decode_oracle_matches_gather_softmax():
    case = oa.make_paged_case(3, batch=4, hq=8, hkv=2, d=32, page=16, ctx_lo=1, ctx_hi=70, extra_cols=2)
    out = oa.paged_decode(case["q"], case["k"], case["v"], case["block_tables"], case["context_lens"], case["scale"])
    kf = nv.e4m3_decode(case["k"]).astype(np.float16)
    vf = nv.e4m3_decode(case["v"]).astype(np.float16)
    k_out, v_out, cu = oa.gather_kv_from_blocks(kf, vf, case["block_tables"], case["context_lens"])
    q16 = case["q"].astype(np.float16).astype(np.float64)
    for b in range(4):
        ks = k_out[cu[b]:cu[b + 1]].astype(np.float64)
        vs = v_out[cu[b]:cu[b + 1]].astype(np.float64)
        for h in range(8):
            s = ks[:, h // 4] @ q16[b, h] * case["scale"]
            p = np.exp(s - s.max())
            p /= p.sum()
            np.testing.assert_allclose(out[b, h], p @ vs[:, h // 4], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("window", [0, 9])
def test_paged_prefill_oracle_matches_gather_causal_softmax(window):
    """The prefill oracle is the reference's gather (pinned above by golden_kv.npz) followed by
    flash-attn's varlen causal attention as published: bottom-right aligned mask, window (W, 0).
    Restated here with explicit loops over sequences, heads and query rows."""
    case = oa.make_prefill_case(4, [0, 13, 40], [21, 1, 18], 8, 2, 32, 16)
    out = oa.paged_prefill(case["q"], case["k"], case["v"], case["block_tables"], case["cu_q"], case["cu_k"],
                           case["scale"], window)
    kf = nv.e4m3_decode(case["k"]).astype(np.float16)
    vf = nv.e4m3_decode(case["v"]).astype(np.float16)
    len_k = np.diff(case["cu_k"])
    k_out, v_out, cu = oa.gather_kv_from_blocks(kf, vf, case["block_tables"], len_k)
    q16 = case["q"].astype(np.float16).astype(np.float64)
    for b in range(3):
        q0, lq = int(case["cu_q"][b]), int(case["cu_q"][b + 1] - case["cu_q"][b])
        ks = k_out[cu[b]:cu[b + 1]].astype(np.float64)
        vs = v_out[cu[b]:cu[b + 1]].astype(np.float64)
        off = ks.shape[0] - lq
        for h in range(8):
            for i in range(lq):
                lo = max(0, i + off - window) if window else 0
                s = ks[lo:i + off + 1, h // 4] @ q16[q0 + i, h] * case["scale"]
                p = np.exp(s - s.max())
                p /= p.sum()
                np.testing.assert_allclose(out[q0 + i, h], p @ vs[lo:i + off + 1, h // 4], rtol=1e-5, atol=1e-5)


def test_act_terms_reconstruct():
    rng = np.random.default_rng(0)
    x = torch.from_numpy(rng.standard_normal((4, 512)).astype(np.float32)).to(torch.bfloat16).float().numpy()
    errs = {}
    for t in (1, 2, 3, 4, 6, 8):
        c, s, g = nv.quantize_act_terms(x, t)
        errs[t] = nv.rel_l2(nv.dequant_act_terms(c, s, g), x)
    assert errs[1] < 0.12 and errs[2] < 0.03 and errs[4] < 1e-3 and errs[6] < 5e-5 and errs[8] < 2e-6
    assert errs[2] > errs[3] > errs[4] > errs[6] > errs[8]


def test_act_terms_known_answer():
    # row amax 6 -> g_0 = 1: term 0 holds the e2m1-representable values exactly, term 1
    # (g_1 = 1/6) the remainder of 5 = 4 + 1, term 2 what 1 * 6 = 6 leaves (nothing)
    x = np.zeros((2, 256), np.float32)
    x[0, :4] = [6.0, -3.0, 0.5, 5.0]
    x[1, :] = 2.0 ** -70  # below 2^-64: quantises to zero with scale 1
    c, s, g = nv.quantize_act_terms(x, 3)
    assert s is None and g[0] == 1.0 and g[1] == 1.0
    vals = nv.e2m1_decode(c)
    assert list(vals[0, 0, :4]) == [6.0, -3.0, 0.5, 4.0]
    assert list(vals[1, 0, :4]) == [0.0, 0.0, 0.0, 6.0]
    assert np.all(vals[2, 0] == 0) and np.all(vals[:, 1] == 0)
    np.testing.assert_array_equal(nv.dequant_act_terms(c, s, g)[0, :4], x[0, :4])
    np.testing.assert_array_equal(nv.term_scales(np.float32([6.0]), 3)[:, 0], np.float32([6.0, 1.0, 1.0 / 6.0]))


def test_store_kvcache_oracle_skips_minus_one():
    kc = np.zeros((3, 4, 2, 8), np.uint8)
    vc = np.zeros_like(kc)
    key = np.ones((3, 2, 8), np.float32)
    val = -np.ones((3, 2, 8), np.float32)
    oa.store_kvcache(key, val, kc, vc, np.array([5, -1, 0]))
    assert (nv.e4m3_decode(kc.reshape(-1, 16)[5]) == 1).all() and (nv.e4m3_decode(vc.reshape(-1, 16)[0]) == -1).all()
    assert (kc.reshape(-1, 16)[[1, 2, 3, 4, 6]] == 0).all()


def test_torch_dequant_matches_numpy(golden_dir):
    g = _load(golden_dir, "golden_nvfp4.npz")
    a = nv.dequant_nvfp4(g["packed"], g["scale_fp16"].astype(np.float32), g["scale_2"])
    b = nv.dequant_nvfp4_torch(torch.from_numpy(g["packed"]), torch.from_numpy(g["scale_fp16"]).float(),
                               float(g["scale_2"]))
    np.testing.assert_array_equal(a, b.numpy())


def test_w4a16_oracle_matches_reference_golden_and_fp16_kernel_emulation(golden_dir):
    """oracle.nvfp4.linear_w4a16_ref (the W4A16 product: fp16 x, exact fp16 code x block scale,
    scale_2 after the sum) against the reference's golden linear output (bf16 weights in its
    dequant mode: within 1e-2 as linear_ref) and against the emulation of the reference's fp16
    Triton kernel, which folds scale_2 into fp16 weights and rounds its output to fp16 (within
    those roundings, < 2e-3); on exactly representable inputs the oracle is exact."""
    g = _load(golden_dir, "golden_nvfp4.npz")
    x = bf16_from_bits(g["x_bf16"]).float()
    y = nv.linear_w4a16_ref(x, g["packed"], g["scale_fp16"].astype(np.float32), g["scale_2"])
    y_ref = bf16_from_bits(g["y_bf16"]).float().numpy()
    assert nv.rel_l2(y.numpy(), y_ref) < 1e-2
    w16 = nv.dequant_nvfp4_kernel_fp16(g["packed"], g["scale_fp16"], g["scale_2"]).float()
    emu = (x.half().float() @ w16.t()).half().double()
    assert nv.rel_l2(y.numpy(), emu.numpy()) < 2e-3
    # one code per row, a unit scale, scale_2 = 1: the product is exact
    packed = np.zeros((4, 8), np.uint8)
    packed[:, 0] = [0x01, 0x07, 0x0F, 0x19]        # (K 0, K 1): (0.5, 0) | (6, 0) | (-6, 0) | (-0.5, 0.5)
    xk = torch.zeros((1, 16), dtype=torch.float16)
    xk[0, 0], xk[0, 1] = 2.0, 3.0
    out = nv.linear_w4a16_ref(xk, packed, np.ones((4, 1), np.float32), np.float32(1.0))
    np.testing.assert_array_equal(out.numpy(), [[1.0, 12.0, -12.0, -1.0 + 1.5]])
