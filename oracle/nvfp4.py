"""NVFP4 oracle: e2m1/e4m3 codecs, the reference dequantiser, fixture
quantisers and the dequantise-then-matmul linear.  Test infrastructure only.

Reference anchors (paths inside the reference project):
  * e2m1 lookup table          adallm/infra/nvfp4.py:7-18 (same table at
                               adallm/ops/nvfp4_gemm.py:7-18)
  * dequant_nvfp4              adallm/infra/nvfp4.py:36-77
  * nvfp4_linear semantics     adallm/ops/nvfp4_gemm.py:460-564 (kernel :58-136)
  * its fp16 (W4A16) product  adallm/ops/nvfp4_gemm.py:100-128 (linear_w4a16_ref)
  * weight / scale layout      adallm/ops/linear.py:31-43 (uint8 [N, K/2],
                               fp16 [N, K/16] holding e4m3 values, fp32 [])

The reference ships no quantiser (checkpoints come from NVIDIA ModelOpt), so
``quantize_weight`` follows the synthetic-config text: one e4m3 scale per 16
contiguous K elements (block amax / 6) relative to one fp32 per-tensor global
scale (amax / (6 * 448)), nearest-e2m1 codes, two codes per byte with the even
K index in the low nibble.

``quantize_act_terms`` is the bit-exact specification of the activation
quantiser that feeds the tcgen05 ``kind::mxf4nvf4`` GEMM of adallm_b200 (it
has no reference counterpart): the bf16 activation row is written as a sum of
T NVFP4 terms that share one fp32 per-row global scale, each term quantising
the residual left by the previous ones.
"""
from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0
E2M1_MAX = 6.0
GLOBAL_DIV = 6.0 * 448.0  # 2688


def _e2m1_magnitudes() -> np.ndarray:
    # code bits: s e1 e0 m  (adallm/infra/nvfp4.py:7-18)
    out = []
    for code in range(8):
        exp = (code >> 1) & 0x3
        mant = code & 0x1
        if exp == 0:
            out.append(0.5 * mant)
        else:
            out.append((1.0 + 0.5 * mant) * 2.0 ** (exp - 1))
    return np.asarray(out, dtype=np.float64)


def _e4m3_magnitudes() -> np.ndarray:
    # e4m3fn: bias 7, no inf, 0x7f / 0xff are NaN; codes 0..126 are finite
    out = []
    for code in range(127):
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0:
            out.append(m / 8.0 * 2.0 ** -6)
        else:
            out.append((1.0 + m / 8.0) * 2.0 ** (e - 7))
    return np.asarray(out, dtype=np.float64)


E2M1_MAG = _e2m1_magnitudes()
E4M3_MAG = _e4m3_magnitudes()
E2M1_LUT = np.concatenate([E2M1_MAG, -E2M1_MAG]).astype(np.float32)  # 16 entries


def _round_to_table(mag: np.ndarray, table: np.ndarray) -> np.ndarray:
    """Round non-negative float magnitudes to the nearest entry of a sorted
    table, ties to the even code, saturating at the last entry.  Returns codes."""
    x = np.asarray(mag, dtype=np.float64)
    n = table.shape[0]
    hi = np.searchsorted(table, x, side="left")
    hi = np.clip(hi, 1, n - 1)
    lo = hi - 1
    d_lo = x - table[lo]
    d_hi = table[hi] - x
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & ((hi & 1) == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(x >= table[-1], n - 1, code)
    code = np.where(x <= 0, 0, code)
    return code.astype(np.uint8)


def e2m1_encode(v: np.ndarray) -> np.ndarray:
    """fp32 -> e2m1 code (round-to-nearest-even, saturate to +-6)."""
    v = np.asarray(v, dtype=np.float32)
    code = _round_to_table(np.abs(v), E2M1_MAG)
    return (code | (np.signbit(v).astype(np.uint8) << 3)).astype(np.uint8)


def e2m1_decode(code: np.ndarray) -> np.ndarray:
    return E2M1_LUT[np.asarray(code, dtype=np.int64) & 0xF]


def e4m3_encode(v: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn bits, round-to-nearest-even, saturating to +-448 (the
    ``cvt.rn.satfinite`` behaviour; the reference's Triton store at
    adallm/ops/attention.py:11-31 casts the same way)."""
    v = np.asarray(v, dtype=np.float32)
    code = _round_to_table(np.abs(v), E4M3_MAG)
    code = code | (np.signbit(v).astype(np.uint8) << 7)
    code = np.where(np.isnan(v), np.uint8(0x7F), code)
    return code.astype(np.uint8)


def e4m3_decode(bits: np.ndarray) -> np.ndarray:
    b = np.asarray(bits, dtype=np.uint8)
    mag = E4M3_MAG[np.minimum(b & 0x7F, 126)].astype(np.float32)
    mag = np.where((b & 0x7F) == 0x7F, np.float32(np.nan), mag)
    return np.where(b & 0x80, -mag, mag).astype(np.float32)


def pack_codes(codes: np.ndarray) -> np.ndarray:
    """[..., K] e2m1 codes -> [..., K/2] bytes, even K in the low nibble
    (adallm/infra/nvfp4.py:54-61)."""
    c = np.asarray(codes, dtype=np.uint8)
    return (c[..., 0::2] & 0xF) | ((c[..., 1::2] & 0xF) << 4)


def unpack_codes(packed: np.ndarray) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = p & 0xF
    out[..., 1::2] = p >> 4
    return out


def dequant_nvfp4(packed: np.ndarray, scale: np.ndarray, scale_2, group_size: int = 16) -> np.ndarray:
    """Restates adallm/infra/nvfp4.py:36-77: W = lut[nibble] * scale[n, k//g] * scale_2 in fp32."""
    packed = np.asarray(packed)
    if packed.dtype != np.uint8:
        raise ValueError("packed_weight must be uint8 for NVFP4 dequantization")
    if packed.ndim != 2:
        raise ValueError("packed_weight must be 2D [out, in/2]")
    n, khalf = packed.shape
    k = khalf * 2
    if k % group_size != 0:
        raise ValueError("in_features must be divisible by group_size")
    vals = e2m1_decode(unpack_codes(packed))  # [n, k] fp32
    s = np.asarray(scale, dtype=np.float32)
    if scale_2 is not None:
        s = s * np.float32(np.asarray(scale_2, dtype=np.float32))
    if s.ndim == 1:
        s = s.reshape(n, 1)
    groups = k // group_size
    if s.shape[1] not in (1, groups):
        raise ValueError("weight_scale shape does not match packed_weight")
    v = vals.reshape(n, groups, group_size)
    if s.shape[1] == 1:
        v = v * s.reshape(n, 1, 1)
    else:
        v = v * s.reshape(n, groups, 1)
    return v.reshape(n, k).astype(np.float32)


def dequant_nvfp4_torch(packed, scale, scale_2, group_size: int = 16, dtype=None):
    """Same arithmetic as dequant_nvfp4 (adallm/infra/nvfp4.py:36-77) in multi-threaded CPU
    torch, for the large one-time dequantisation of the timed CPU baseline."""
    import torch
    p = torch.as_tensor(packed)
    n, khalf = p.shape
    lut = torch.from_numpy(E2M1_LUT)
    vals = torch.empty((n, khalf * 2), dtype=torch.float32)
    vals[:, 0::2] = lut[(p & 0x0F).long()]
    vals[:, 1::2] = lut[(p >> 4).long()]
    s = torch.as_tensor(scale).float()
    if scale_2 is not None:
        s = s * float(scale_2)
    out = (vals.view(n, -1, group_size) * s.view(n, -1, 1)).view(n, khalf * 2)
    return out if dtype is None else out.to(dtype)


def dequant_nvfp4_kernel_fp16(packed, scale, scale_2, group_size: int = 16):
    """The weight tile as the reference's fp16 NVFP4 GEMM kernel forms it
    (adallm/ops/nvfp4_gemm.py:107-126, launched by nvfp4_linear :460-564 with NVFP4_FP8 unset):
    base = fp16 LUT[nibble], scale loaded as fp16, scale2 = fp16(scale_2), and
    b = base * scale * scale2 evaluated left to right in fp16 (each product rounded to
    nearest fp16).  A product of two fp16 values is exact in fp32, so rounding the fp32
    product to fp16 reproduces the fp16 multiply.  Returns torch fp16 [N, K]."""
    import torch
    p = torch.as_tensor(packed)
    n, khalf = p.shape
    lut = torch.from_numpy(E2M1_LUT).to(torch.float16)
    base = torch.empty((n, khalf * 2), dtype=torch.float16)
    base[:, 0::2] = lut[(p & 0x0F).long()]
    base[:, 1::2] = lut[(p >> 4).long()]
    s = torch.as_tensor(scale).to(torch.float16).float().repeat_interleave(group_size, dim=1)
    s2 = torch.tensor(float(scale_2), dtype=torch.float32).to(torch.float16).float()
    t = (base.float() * s).to(torch.float16)
    return (t.float() * s2).to(torch.float16)


def linear_w4a8_ref(x, packed, scale, scale_2, block_k: int = 64):
    """The reference's W4A8 linear (nvfp4_gemm_kernel_fp8, adallm/ops/nvfp4_gemm.py:252-360, taken
    when NVFP4_FP8=1 with its defaults NVFP4_FP8_A_SCALE=1, NVFP4_FP8_B_SCALE=0,
    NVFP4_FP8_BCOL=0, NVFP4_FP8_FORMAT=e4nv; BLOCK_K = 64 for M <= 16 or K < 8192, :480-490).
    Per BLOCK_K chunk: a = fp16(x); amax = row max |a| over the chunk (0 -> 1);
    a8 = e4m3(a / amax); b8 = e4m3(b) of the fp16 weight tile b = LUT * scale * scale2 (unscaled);
    acc += (a8 . b8) * amax in fp32; output fp16.  Returns torch fp16 [M, N]."""
    import torch
    a = torch.as_tensor(x).to(torch.float16).float()
    w16 = dequant_nvfp4_kernel_fp16(packed, scale, scale_2).float()
    b8 = torch.from_numpy(e4m3_decode(e4m3_encode(w16.numpy())))
    m, k = a.shape
    acc = torch.zeros((m, w16.shape[0]), dtype=torch.float32)
    for k0 in range(0, k, block_k):
        ac = a[:, k0:k0 + block_k]
        amax = ac.abs().amax(dim=1, keepdim=True)
        amax = torch.where(amax == 0, torch.ones_like(amax), amax)
        a8 = torch.from_numpy(e4m3_decode(e4m3_encode((ac / amax).numpy())))
        acc += (a8.double() @ b8[:, k0:k0 + block_k].double().t()).float() * amax
    return acc.to(torch.float16)


def quantize_weight(w: np.ndarray, group_size: int = 16):
    """Fixture quantiser for synthetic NVFP4 weights (no reference counterpart).

    Returns (packed uint8 [N, K/2], scale_bits uint8 [N, K/16] (e4m3),
    scale_2 float32 scalar)."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    amax = np.float32(np.max(np.abs(w))) if w.size else np.float32(0)
    g = np.float32(amax / np.float32(GLOBAL_DIV)) if amax > 0 else np.float32(1.0)
    blocks = w.reshape(n, k // group_size, group_size)
    bamax = np.max(np.abs(blocks), axis=-1)
    g6 = np.float32(g * np.float32(6.0))
    s_bits = e4m3_encode((bamax / g6).astype(np.float32))
    s_val = e4m3_decode(s_bits)
    denom = (s_val * g).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        rcp = np.where(denom > 0, np.float32(1.0) / denom, np.float32(0)).astype(np.float32)
    v = (blocks * rcp[..., None]).astype(np.float32)
    codes = e2m1_encode(v)
    codes = np.where((s_val > 0)[..., None], codes, np.uint8(0)).reshape(n, k)
    return pack_codes(codes), s_bits, g


MIN_AMAX = np.float32(2.0 ** -64)
MAX_TERMS = 8


def quantize_act_terms(x: np.ndarray, terms: int, group_size: int = 16, row_scale: np.ndarray | None = None):
    """Bit-exact specification of adallm_b200's activation quantiser (csrc/quant.cuh).

    row_scale: the rows' g (terms == 1) or g_0 (terms >= 2) as a producer chose them, used as
    given instead of being derived from the exact amax (the RMSNorm producers derive it from a
    bound on the amax, which is never below it).
    x: [M, K] (bf16 values given as fp32).  Per row, with amax = max|x| (a row whose amax
    is below 2^-64 quantises to zero with scale 1.0):
      terms == 1 (NVFP4, block scales): g = amax / 2688; per 16-block
          s = e4m3(blockamax / (g*6)), code = e2m1(x * (1 / (s*g)))   (0 when s == 0)
      terms >= 2 (row-scaled terms, unit block scales): g_0 = amax / 6, g_t = g_{t-1} / 6,
          r_0 = x, code_t = e2m1(r_t * (1 / g_t)), r_{t+1} = r_t - e2m1val(code_t) * g_t
    Every operation is one IEEE fp32 rounding (no fused multiply-add).
    Returns codes uint8 [T, M, K], block-scale bits uint8 [M, K/16] (terms == 1; None
    otherwise) and the row scale fp32 [M] (g, or g_0).
    """
    x = np.asarray(x, dtype=np.float32)
    if not 1 <= terms <= MAX_TERMS:
        raise ValueError("terms must be in 1..8")
    m, k = x.shape
    groups = k // group_size
    amax = np.max(np.abs(x), axis=1).astype(np.float32) if k else np.zeros(m, np.float32)
    live = amax >= MIN_AMAX
    if terms == 1:
        g = np.where(live, (amax / np.float32(GLOBAL_DIV)).astype(np.float32), np.float32(1.0)).astype(np.float32)
        if row_scale is not None:
            g = np.asarray(row_scale, np.float32).reshape(m).copy()
        g6 = (g * np.float32(6.0)).astype(np.float32)
        r = x.reshape(m, groups, group_size)
        bamax = np.max(np.abs(r), axis=-1).astype(np.float32)
        sb = e4m3_encode((bamax / g6[:, None]).astype(np.float32))
        sv = e4m3_decode(sb)
        denom = (sv * g[:, None]).astype(np.float32)
        with np.errstate(divide="ignore", invalid="ignore"):
            rcp = np.where(denom > 0, np.float32(1.0) / denom, np.float32(0)).astype(np.float32)
        c = e2m1_encode((r * rcp[..., None]).astype(np.float32))
        c = np.where((sv > 0)[..., None], c, np.uint8(0))
        return c.reshape(1, m, k), sb, g
    g0 = np.where(live, (amax / np.float32(6.0)).astype(np.float32), np.float32(1.0)).astype(np.float32)
    if row_scale is not None:
        g0 = np.asarray(row_scale, np.float32).reshape(m).copy()
    g = g0.copy()
    r = x.copy()
    codes = np.zeros((terms, m, k), np.uint8)
    for t in range(terms):
        rcp = (np.float32(1.0) / g).astype(np.float32)
        c = e2m1_encode((r * rcp[:, None]).astype(np.float32))
        deq = (e2m1_decode(c) * g[:, None]).astype(np.float32)
        r = (r - deq).astype(np.float32)
        codes[t] = c
        g = (g / np.float32(6.0)).astype(np.float32)
    return codes, None, g0


def term_scales(g0: np.ndarray, terms: int) -> np.ndarray:
    """Scale of each row-scaled term: [T, M] with g_t = g_{t-1} / 6 (fp32)."""
    g = np.asarray(g0, np.float32).copy()
    out = np.zeros((terms,) + g.shape, np.float32)
    for t in range(terms):
        out[t] = g
        g = (g / np.float32(6.0)).astype(np.float32)
    return out


def dequant_act_terms(codes: np.ndarray, sbits, g: np.ndarray, group_size: int = 16) -> np.ndarray:
    """Value the GEMM sees for the quantised activations -> fp32 [M, K] (sum of terms in float64)."""
    t, m, k = codes.shape
    vals = e2m1_decode(codes).astype(np.float64)
    if t == 1:
        s = e4m3_decode(sbits).astype(np.float64) * np.asarray(g, np.float64)[:, None]
        return (vals[0].reshape(m, k // group_size, group_size) * s[..., None]).reshape(m, k).astype(np.float32)
    gt = term_scales(g, t).astype(np.float64)
    return (vals * gt[:, :, None]).sum(axis=0).astype(np.float32)


def linear_ref(x: np.ndarray, packed: np.ndarray, scale: np.ndarray, scale_2, bias=None) -> np.ndarray:
    """Dequantise-then-matmul oracle of nvfp4_linear (adallm/ops/nvfp4_gemm.py:460-564,
    run as the reference's "dequant" mode does: adallm/infra/loader.py:92-102 then
    adallm/ops/linear.py:74).  fp32 result [M, N]."""
    w = dequant_nvfp4(packed, scale, scale_2)
    y = np.asarray(x, dtype=np.float32) @ w.T
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)
    return y.astype(np.float32)


def linear_w4a16_ref(x, packed, scale, scale_2, bias=None):
    """The W4A16 product of the reference's fp16 NVFP4 GEMM (adallm/ops/nvfp4_gemm.py:58-136,
    launched by nvfp4_linear :460-564 with NVFP4_FP8 unset): the activation tile cast to fp16
    (:100-105), the weight element LUT[code] * e4m3 block scale (:118-126; exact in fp16), fp32
    accumulation (:128).  Here the sum is taken in float64 over those fp16 operands and scale_2
    is applied after it (the arithmetic of adallm_b200's W4A16 kernel, which does not fold scale_2
    into fp16 weights as :126 does), bias last.  float64 torch [M, N]."""
    import torch
    w = dequant_nvfp4_torch(packed, np.asarray(scale, dtype=np.float32), None).double()
    y = (torch.as_tensor(x).cpu().to(torch.float16).double() @ w.t()) * float(scale_2)
    if bias is not None:
        y = y + torch.as_tensor(bias).cpu().double()
    return y


def linear_terms_ref(codes, sbits, g, packed, scale, scale_2) -> np.ndarray:
    """Dequantise-both oracle for the mxf4nvf4 GEMM: the exact math the tensor
    cores perform (fp32 [M, N])."""
    xq = dequant_act_terms(codes, sbits, g)
    w = dequant_nvfp4(packed, scale, scale_2)
    return (xq.astype(np.float64) @ w.T.astype(np.float64)).astype(np.float32)


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
