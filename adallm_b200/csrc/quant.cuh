// Activation quantiser shared by every kernel that produces an operand of the
// tensor-core NVFP4 GEMM (bit-exact spec: oracle/nvfp4.py quantize_act_terms).
//
// Two operand modes, selected by `terms`:
//   terms == 1   NVFP4 activations (W4A4): g = amax(row) / 2688, per 16-element block
//                s = e4m3(blockamax / (6g)), code = e2m1(x * (1 / (s*g))) (0 when s == 0).
//   terms 2..8   the row is a sum of `terms` e2m1 terms with unit block scales and one fp32
//                scale per (row, term): g_0 = amax(row) / 6, g_t = g_{t-1} / 6,
//                code_t = e2m1(r_t * (1 / g_t)), r_0 = x, r_{t+1} = r_t - e2m1val(code_t) * g_t.
//                The residual of a term is at most g_t in magnitude, so term t + 1 never
//                saturates; 4 terms are within ~1e-3 relative L2 of the input, 6 within ~1e-4.
// Only the row amax couples the elements of a row, so a row may be quantised by many CTAs
// once that one reduction is done.  A row whose amax is below 2^-64 quantises to zero
// (g = 1).  Every operation is one IEEE fp32 rounding (explicit _rn: no fused multiply-add).
//
// Operand layout for token m = mt*bn + j (tile mt of bn tokens), term t -> row t*bn + j:
//   xq  [m_tiles][terms*bn][K/2]   packed e2m1, even K in the low nibble
//   sfx [m_tiles][K/64][512]       (terms == 1 only) ue4m3 scales in the block-scaled MMA
//                                  layout: row r of a 128-row block at (r%32)*16 + (r/32)*4
//   gx  [m_pad]                    g (terms == 1) or g_0 (terms >= 2); 1.0 for padding rows
#pragma once

#include "common.cuh"

namespace ada {
namespace q {

constexpr int MAX_TERMS = 8;
constexpr float MIN_AMAX = 5.421010862427522e-20f;  // 2^-64

struct QuantDst {
  uint8_t* xq;
  uint8_t* sfx;  // terms == 1 only
  float* gx;
  int terms, bn, k;
};

__device__ __forceinline__ float e4m3_value(uint8_t b) {
  const uint32_t h = e4m3x2_to_f16x2((uint16_t)b);
  return __half2float(__ushort_as_half((unsigned short)(h & 0xFFFFu)));
}

// Scale of term t of a row with scale g_0 (terms >= 2); the GEMM epilogue derives the
// term scales from gx with the same recurrence.
__device__ __forceinline__ float next_term_scale(float g) { return __fdiv_rn(g, 6.f); }

// Per-row constants, derived from the row amax.
struct RowQ {
  float g[2];  // terms >= 2: g[0] = g_0 (the term scales follow by next_term_scale);
               // terms == 1: g[0] = g, g[1] = 6g
  int terms;
};
__device__ __forceinline__ RowQ make_rowq(float amax, int terms) {
  RowQ q;
  q.terms = terms;
  const bool live = amax >= MIN_AMAX;
  if (terms == 1) {
    q.g[0] = live ? __fdiv_rn(amax, 2688.f) : 1.f;
    q.g[1] = __fmul_rn(q.g[0], 6.f);
    return q;
  }
  q.g[0] = live ? __fdiv_rn(amax, 6.f) : 1.f;
  q.g[1] = 0.f;
  return q;
}

__device__ __forceinline__ uint8_t* xq_row(const QuantDst& d, int m, int t) {
  const int mt = m / d.bn, j = m - mt * d.bn;
  return d.xq + ((size_t)mt * d.terms * d.bn + (size_t)t * d.bn + j) * ((size_t)d.k >> 1);
}
__device__ __forceinline__ uint8_t* sf_byte(const QuantDst& d, int m, int blk) {
  const int mt = m / d.bn, j = m - mt * d.bn;
  return d.sfx + ((size_t)mt * (d.k >> 6) + (blk >> 2)) * 512 + (j & 31) * 16 + (j >> 5) * 4 + (blk & 3);
}

// Quantise the 8 elements r[0..8) of octet `oc` (elements 8*oc .. 8*oc+7) of token m
// (r is clobbered for terms >= 2).  For terms == 1 the two octets of a 16-element block
// are held by lanes l and l^1 of one warp, which share the block amax: every lane of the
// warp calls this together; lanes with valid == false contribute zeros and store nothing.
__device__ __forceinline__ void quant_oct(const QuantDst& d, int m, int oc, float* r, const RowQ& q, bool valid) {
  if (q.terms == 1) {
    float bamax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) bamax = fmaxf(bamax, valid ? fabsf(r[i]) : 0.f);
    bamax = fmaxf(bamax, __shfl_xor_sync(0xffffffffu, bamax, 1));
    const uint8_t sb = (uint8_t)(f32x2_to_e4m3x2(__fdiv_rn(bamax, q.g[1]), 0.f) & 0xFFu);
    const float sv = e4m3_value(sb);
    uint32_t codes = 0;
    if (sv > 0.f) {
      const float rcp = __fdiv_rn(1.f, __fmul_rn(sv, q.g[0]));
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(r[i], rcp);
      codes = f32x8_to_e2m1x8(v);
    }
    if (valid) {
      *reinterpret_cast<uint32_t*>(xq_row(d, m, 0) + (size_t)oc * 4) = codes;
      if (!(oc & 1)) *sf_byte(d, m, oc >> 1) = sb;
    }
    return;
  }
  // one term per iteration (kept rolled: short code for a path every producer kernel runs once)
  float g = q.g[0];
  uint8_t* row = xq_row(d, m, 0) + (size_t)oc * 4;
  const size_t term_stride = (size_t)d.bn * ((size_t)d.k >> 1);
#pragma unroll 1
  for (int t = 0; t < q.terms; ++t) {
    const float rcp = __frcp_rn(g);  // correctly rounded 1 / g_t (g_t is normal: >= 2^-64 / 6^8)
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(r[i], rcp);
    const uint32_t codes = f32x8_to_e2m1x8(v);
    if (t + 1 < q.terms) {
      uint32_t h[4];
      e2m1x8_to_f16x8(codes, h);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint16_t hb = (uint16_t)(h[i >> 1] >> (16 * (i & 1)));
        r[i] = __fsub_rn(r[i], __fmul_rn(__half2float(__ushort_as_half(hb)), g));
      }
    }
    if (valid) *reinterpret_cast<uint32_t*>(row + (size_t)t * term_stride) = codes;
    g = next_term_scale(g);
  }
}

// Codes (and block scales) of a padding token m in [M, m_pad): zero.
__device__ __forceinline__ void zero_oct(const QuantDst& d, int m, int oc) {
  for (int t = 0; t < d.terms; ++t) *reinterpret_cast<uint32_t*>(xq_row(d, m, t) + (size_t)oc * 4) = 0u;
  if (d.terms == 1 && !(oc & 1)) *sf_byte(d, m, oc >> 1) = 0;
}

// Valid operand configuration: terms 1..8, token tile 16/32/64/128 with terms*bn <= 128,
// K a multiple of 256 (one GEMM pipeline stage), block scales present iff terms == 1.
__host__ __device__ inline bool dst_ok(int terms, int bn, int k) {
  if (terms < 1 || terms > MAX_TERMS) return false;
  if (bn != 16 && bn != 32 && bn != 64 && bn != 128) return false;
  return terms * bn <= 128 && k > 0 && k % 256 == 0;
}

}  // namespace q
}  // namespace ada
