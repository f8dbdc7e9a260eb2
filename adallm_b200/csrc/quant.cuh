// Multi-term NVFP4 activation quantiser shared by every kernel that produces an
// input of the tensor-core NVFP4 GEMM (bit-exact spec: oracle/nvfp4.py
// quantize_act_terms).  A row of K values is written as `terms` NVFP4 terms that
// share the fp32 row scale g = amax(row) / 2688; term t quantises, per 16-element
// block, the residual left by terms < t: s = e4m3(blockamax / (6g)), code =
// e2m1(r / (s*g)), r -= lut[code] * s * g.  Every operation is one IEEE fp32
// rounding (explicit _rn intrinsics: no fused multiply-add).
//
// Operand layout for token m = mt*bn + j (tile mt of bn tokens), term t -> row t*bn + j:
//   xq  [m_tiles][terms*bn][K/2]   packed e2m1, even K in the low nibble
//   sfx [m_tiles][K/64][512]       ue4m3 scales in the block-scaled MMA layout
//                                  (row r of a 128-row block at (r%32)*16 + (r/32)*4)
//   gx  [m_pad]                    g per token (1.0 for zero padding rows)
#pragma once

#include "common.cuh"

namespace ada {
namespace q {

struct QuantDst {
  uint8_t* xq;
  uint8_t* sfx;
  float* gx;
  int terms, bn, k;
};

__device__ __forceinline__ float e2m1_value(uint32_t c) {
  const uint32_t mag = c & 7u;
  float v = mag < 2u ? 0.5f * (float)mag : (float)(2u + (mag & 1u)) * __int_as_float((int)(((mag >> 1) + 125u) << 23));
  return (c & 8u) ? -v : v;
}
__device__ __forceinline__ float e4m3_value(uint8_t b) {
  const uint32_t h = e4m3x2_to_f16x2((uint16_t)b);
  return __half2float(__ushort_as_half((unsigned short)(h & 0xFFFFu)));
}

__device__ __forceinline__ float row_scale(float amax) { return amax > 0.f ? __fdiv_rn(amax, 2688.f) : 1.f; }

// Quantise one 16-element block `blk` of token m (values r[], consumed in place).
__device__ __forceinline__ void quant_block16(const QuantDst& d, int m, int blk, float* r, float g, float g6) {
  const int mt = m / d.bn, j = m - mt * d.bn;
  const int kb64 = d.k >> 6;
  const size_t khalf = (size_t)d.k >> 1;
  for (int t = 0; t < d.terms; ++t) {
    float bamax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) bamax = fmaxf(bamax, fabsf(r[i]));
    const uint8_t sb = (uint8_t)(f32x2_to_e4m3x2(__fdiv_rn(bamax, g6), 0.f) & 0xFFu);
    const float sv = e4m3_value(sb);
    uint2 codes = make_uint2(0, 0);
    if (sv > 0.f) {
      const float denom = __fmul_rn(sv, g);
      const float rcp = __fdiv_rn(1.f, denom);
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = __fmul_rn(r[i], rcp);
      codes.x = f32x8_to_e2m1x8(v);
      codes.y = f32x8_to_e2m1x8(v + 8);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t c = ((i < 8 ? codes.x : codes.y) >> (4 * (i & 7))) & 0xFu;
        r[i] = __fsub_rn(r[i], __fmul_rn(e2m1_value(c), denom));
      }
    }
    const int row = t * d.bn + j;
    *reinterpret_cast<uint2*>(d.xq + ((size_t)mt * d.terms * d.bn + row) * khalf + (size_t)blk * 8) = codes;
    d.sfx[((size_t)mt * kb64 + (blk >> 2)) * 512 + (row & 31) * 16 + (row >> 5) * 4 + (blk & 3)] = sb;
  }
}

// Zero codes / scales of a padding token (m in [M, m_pad)): one block per call.
__device__ __forceinline__ void zero_block16(const QuantDst& d, int m, int blk) {
  const int mt = m / d.bn, j = m - mt * d.bn;
  const int kb64 = d.k >> 6;
  const size_t khalf = (size_t)d.k >> 1;
  for (int t = 0; t < d.terms; ++t) {
    const int row = t * d.bn + j;
    *reinterpret_cast<uint2*>(d.xq + ((size_t)mt * d.terms * d.bn + row) * khalf + (size_t)blk * 8) = make_uint2(0, 0);
    d.sfx[((size_t)mt * kb64 + (blk >> 2)) * 512 + (row & 31) * 16 + (row >> 5) * 4 + (blk & 3)] = 0;
  }
}

// Block-wide max of non-negative values (blockDim.x multiple of 32, <= 1024).
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r = fmaxf(r, red[i]);
  return r;
}

}  // namespace q
}  // namespace ada
