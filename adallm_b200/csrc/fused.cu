// Producers of the NVFP4 GEMM operand with the activation quantiser fused in
// (layout and arithmetic: quant.cuh), so a decode layer needs no separate
// quantisation launch before its four projections:
//   * residual-add + RMSNorm / GemmaRMSNorm -> quantised operand of qkv_proj / gate_up_proj
//     (reference adallm/ops/layernorm.py:16-40, :64-92)
//   * SiLU(gate) * up / GELU(tanh)(gate) * up -> quantised operand of down_proj
//     (reference adallm/ops/activation.py:6-26)
// The bf16 value each kernel quantises is exactly the value the unfused op would
// have returned (same rounding order), so fused and unfused paths agree bit for bit.
#include <type_traits>

#include "quant.cuh"

namespace ada {
namespace fused {

constexpr int THREADS = 256;

template <typename T>
__device__ __forceinline__ void load16(const T* p, float* f) {
  unpack8<T>(*reinterpret_cast<const uint4*>(p), f);
  unpack8<T>(*reinterpret_cast<const uint4*>(p + 8), f + 8);
}
template <typename T>
__device__ __forceinline__ void store16(T* p, const float* f) {
  *reinterpret_cast<uint4*>(p) = pack8<T>(f);
  *reinterpret_cast<uint4*>(p + 8) = pack8<T>(f + 8);
}
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f32(from_f32<T>(v));
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r += red[i];
  return r;
}

// One CTA per (padded) token row; thread i owns 16-element blocks i, i + 256, ...
template <typename T, int MAXU>
__global__ void __launch_bounds__(THREADS) rmsnorm_quant_kernel(const T* __restrict__ x, int64_t ldx, const T* res,
                                                                int64_t ldr, T* res_out, int64_t ldro,
                                                                const T* __restrict__ w, T* y, int64_t ldy, int rows,
                                                                int hidden, float eps, int gemma, q::QuantDst dst) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[THREADS / 32];
  const int m = blockIdx.x;
  const int nblk = hidden >> 4;
  if (m >= rows) {
    for (int b = threadIdx.x; b < nblk; b += THREADS) q::zero_block16(dst, m, b);
    if (threadIdx.x == 0) dst.gx[m] = 1.f;
    return;
  }
  float v[MAXU][16];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int b = threadIdx.x + u * THREADS;
    if (b < nblk) {
      load16<T>(x + (int64_t)m * ldx + b * 16, v[u]);
      if (res) {
        float r[16];
        load16<T>(res + (int64_t)m * ldr + b * 16, r);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          v[u][i] = __fadd_rn(v[u][i], r[i]);
          if (gemma && std::is_same<T, __nv_bfloat16>::value) v[u][i] = round_to<T>(v[u][i]);
        }
        store16<T>(res_out + (int64_t)m * ldro + b * 16, v[u]);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) ss = fmaf(v[u][i], v[u][i], ss);
    }
  }
  const float rs = rsqrtf(block_sum(ss, red) / (float)hidden + eps);
  float amax = 0.f;
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int b = threadIdx.x + u * THREADS;
    if (b < nblk) {
      float wf[16];
      load16<T>(w + b * 16, wf);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float xn = __fmul_rn(v[u][i], rs);
        v[u][i] = gemma ? round_to<T>(__fmul_rn(xn, __fadd_rn(1.f, wf[i])))
                        : round_to<T>(__fmul_rn(round_to<T>(xn), wf[i]));
        amax = fmaxf(amax, fabsf(v[u][i]));
      }
      if (y) store16<T>(y + (int64_t)m * ldy + b * 16, v[u]);
    }
  }
  const float g = q::row_scale(q::block_max(amax, red));
  const float g6 = __fmul_rn(g, 6.f);
  if (threadIdx.x == 0) dst.gx[m] = g;
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int b = threadIdx.x + u * THREADS;
    if (b < nblk) q::quant_block16(dst, m, b, v[u], g, g6);
  }
}

__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.f, expf(-x))); }
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float inner = k0 * (x + k1 * x * x * x);
  return 0.5f * x * (1.f + tanhf(inner));
}

template <typename T, int MAXU>
__global__ void __launch_bounds__(THREADS) gated_act_quant_kernel(const T* __restrict__ x, int64_t ldx, T* y,
                                                                  int64_t ldy, int rows, int inter, int act,
                                                                  q::QuantDst dst) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[THREADS / 32];
  const int m = blockIdx.x;
  const int nblk = inter >> 4;
  if (m >= rows) {
    for (int b = threadIdx.x; b < nblk; b += THREADS) q::zero_block16(dst, m, b);
    if (threadIdx.x == 0) dst.gx[m] = 1.f;
    return;
  }
  float v[MAXU][16];
  float amax = 0.f;
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int b = threadIdx.x + u * THREADS;
    if (b < nblk) {
      float gt[16], up[16];
      load16<T>(x + (int64_t)m * ldx + b * 16, gt);
      load16<T>(x + (int64_t)m * ldx + inter + b * 16, up);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float a = act == 0 ? silu_f(gt[i]) : gelu_tanh_f(gt[i]);
        v[u][i] = round_to<T>(__fmul_rn(round_to<T>(a), up[i]));
        amax = fmaxf(amax, fabsf(v[u][i]));
      }
      if (y) store16<T>(y + (int64_t)m * ldy + b * 16, v[u]);
    }
  }
  const float g = q::row_scale(q::block_max(amax, red));
  const float g6 = __fmul_rn(g, 6.f);
  if (threadIdx.x == 0) dst.gx[m] = g;
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int b = threadIdx.x + u * THREADS;
    if (b < nblk) q::quant_block16(dst, m, b, v[u], g, g6);
  }
}

}  // namespace fused
}  // namespace ada

using namespace ada;

static bool quant_args_ok(int terms, int block_n, int k, const void* xq, const void* sfx, const void* gx) {
  if (terms < 1 || terms > 3) return false;
  if (block_n != 16 && block_n != 32 && block_n != 64 && block_n != 128) return false;
  if (terms * block_n > 128 || k % 256) return false;
  return xq && sfx && gx && (((uintptr_t)xq & 15) == 0);
}

extern "C" int ada_rmsnorm_quant(const void* x, int64_t ldx, const void* residual, int64_t ld_res, void* residual_out,
                                 int64_t ld_res_out, const void* weight, void* y, int64_t ldy, int64_t rows,
                                 int32_t hidden, float eps, int gemma, int dtype, int terms, int block_n, uint8_t* xq,
                                 uint8_t* sfx, float* gx, void* stream) {
  if (rows <= 0 || hidden <= 0 || !x || !weight || (residual && !residual_out)) return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (!quant_args_ok(terms, block_n, hidden, xq, sfx, gx)) return ADA_ERR_INVALID_ARG;
  const int nblk = hidden / 16;
  const int maxu = (nblk + fused::THREADS - 1) / fused::THREADS;
  if (maxu > 4) return ADA_ERR_UNSUPPORTED;
  auto a16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (!a16(x) || !a16(weight) || (ldx & 7) || (y && (!a16(y) || (ldy & 7)))) return ADA_ERR_ALIGNMENT;
  if (residual && (!a16(residual) || !a16(residual_out) || (ld_res & 7) || (ld_res_out & 7))) return ADA_ERR_ALIGNMENT;
  const int64_t m_pad = cdiv(rows, block_n) * block_n;
  const q::QuantDst dst{xq, sfx, gx, terms, block_n, hidden};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define ADA_RQ(T, MU)                                                                                               \
  (void)launch_k(fused::rmsnorm_quant_kernel<T, MU>, dim3((unsigned)m_pad), dim3(fused::THREADS), 0, st,            \
                 (const T*)x, ldx, (const T*)residual, ld_res, (T*)residual_out, ld_res_out, (const T*)weight, (T*)y, \
                 ldy, (int)rows, (int)hidden, eps, gemma, dst)
#define ADA_RQT(T)                    \
  if (maxu == 1) ADA_RQ(T, 1);        \
  else if (maxu == 2) ADA_RQ(T, 2);   \
  else ADA_RQ(T, 4);
  if (dtype == ADA_DT_BF16) {
    ADA_RQT(__nv_bfloat16)
  } else {
    ADA_RQT(__half)
  }
#undef ADA_RQT
#undef ADA_RQ
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

extern "C" int ada_gated_act_quant(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t rows, int32_t inter,
                                   int act, int dtype, int terms, int block_n, uint8_t* xq, uint8_t* sfx, float* gx,
                                   void* stream) {
  if (rows <= 0 || inter <= 0 || !x || (act != 0 && act != 1)) return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (!quant_args_ok(terms, block_n, inter, xq, sfx, gx)) return ADA_ERR_INVALID_ARG;
  const int nblk = inter / 16;
  const int maxu = (nblk + fused::THREADS - 1) / fused::THREADS;
  if (maxu > 8) return ADA_ERR_UNSUPPORTED;
  if (((uintptr_t)x & 15) || (ldx & 7) || (y && (((uintptr_t)y & 15) || (ldy & 7)))) return ADA_ERR_ALIGNMENT;
  const int64_t m_pad = cdiv(rows, block_n) * block_n;
  const q::QuantDst dst{xq, sfx, gx, terms, block_n, inter};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define ADA_GQ(T, MU)                                                                                     \
  (void)launch_k(fused::gated_act_quant_kernel<T, MU>, dim3((unsigned)m_pad), dim3(fused::THREADS), 0, st, \
                 (const T*)x, ldx, (T*)y, ldy, (int)rows, (int)inter, act, dst)
#define ADA_GQT(T)                    \
  if (maxu == 1) ADA_GQ(T, 1);        \
  else if (maxu == 2) ADA_GQ(T, 2);   \
  else if (maxu <= 4) ADA_GQ(T, 4);   \
  else ADA_GQ(T, 8);
  if (dtype == ADA_DT_BF16) {
    ADA_GQT(__nv_bfloat16)
  } else {
    ADA_GQT(__half)
  }
#undef ADA_GQT
#undef ADA_GQ
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}
