// Small memory-bound kernels of the decode path (sm_100a):
//   * FP8 KV-cache store          (reference adallm/ops/attention.py:11-31, :236-251)
//   * RMSNorm / GemmaRMSNorm      (reference adallm/ops/layernorm.py:16-40, :64-92)
//   * rotary embedding            (reference adallm/ops/rotary_embedding.py:6-14, :45-56)
//   * SiluAndMul / GeluAndMul     (reference adallm/ops/activation.py:6-26)
//   * embedding gather, argmax    (reference adallm/ops/embed_head.py:35-42; greedy pick)
// Rounding follows the reference's eager torch order (explicit _rn intrinsics
// where torch performs separate roundings, so no FMA contraction changes bits).
#include <atomic>
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "parts.cuh"

namespace ada {
namespace fused {
int launch_rmsnorm16(const void* x, int64_t ldx, const void* res, int64_t ldr, void* ro, int64_t ldro,
                     const void* w, void* y, int64_t ldy, int64_t rows, int hidden, float eps, int gemma, int dtype,
                     cudaStream_t st);
}
namespace small {

// ---------------------------------------------------------------------------
// FP8 KV store: one CTA per token, 8 elements per thread and step.
template <typename T>
__global__ void __launch_bounds__(128) store_kv_kernel(const T* __restrict__ key, const T* __restrict__ value,
                                                       int64_t ks, int64_t vs, const int32_t* __restrict__ slots,
                                                       uint8_t* __restrict__ kc, uint8_t* __restrict__ vc,
                                                       int64_t crs, int hd, float k_scale, float v_scale) {
  pdl_wait();
  pdl_trigger();

  const int t = blockIdx.x;
  const int slot = __ldg(slots + t);
  if (slot < 0) return;  // -1 marks a padded token (attention.py:21)
  const T* kr = key + (int64_t)t * ks;
  const T* vr = value + (int64_t)t * vs;
  uint8_t* ko = kc + (int64_t)slot * crs;
  uint8_t* vo = vc + (int64_t)slot * crs;
  for (int e = threadIdx.x * 8; e < hd; e += blockDim.x * 8) {
    float fk[8], fv[8];
    unpack8<T>(*reinterpret_cast<const uint4*>(kr + e), fk);
    unpack8<T>(*reinterpret_cast<const uint4*>(vr + e), fv);
    if (k_scale != 1.f) {
#pragma unroll
      for (int i = 0; i < 8; ++i) fk[i] = __fdiv_rn(fk[i], k_scale);
    }
    if (v_scale != 1.f) {
#pragma unroll
      for (int i = 0; i < 8; ++i) fv[i] = __fdiv_rn(fv[i], v_scale);
    }
    uint2 ok, ov;
    ok.x = (uint32_t)f32x2_to_e4m3x2(fk[0], fk[1]) | ((uint32_t)f32x2_to_e4m3x2(fk[2], fk[3]) << 16);
    ok.y = (uint32_t)f32x2_to_e4m3x2(fk[4], fk[5]) | ((uint32_t)f32x2_to_e4m3x2(fk[6], fk[7]) << 16);
    ov.x = (uint32_t)f32x2_to_e4m3x2(fv[0], fv[1]) | ((uint32_t)f32x2_to_e4m3x2(fv[2], fv[3]) << 16);
    ov.y = (uint32_t)f32x2_to_e4m3x2(fv[4], fv[5]) | ((uint32_t)f32x2_to_e4m3x2(fv[6], fv[7]) << 16);
    *reinterpret_cast<uint2*>(ko + e) = ok;
    *reinterpret_cast<uint2*>(vo + e) = ov;
  }
}

// ---------------------------------------------------------------------------
// Block-wide sum (blockDim.x multiple of 32, <= 1024).
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (w == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (l == 0) red[0] = t;
  }
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

// RMSNorm family, one CTA per row, the row kept in registers (<= MAXV 8-wide vectors per thread).
template <typename T, int MAXV>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T* __restrict__ x, int64_t ldx, const T* res, int64_t ldr,
                                                      T* res_out, int64_t ldro, const T* __restrict__ w, T* y,
                                                      int64_t ldy, int hidden, float eps, int gemma) {
  pdl_wait();
  pdl_trigger();

  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = hidden >> 3;
  const T* xr = x + row * ldx;
  float v[MAXV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < nvec) {
      unpack8<T>(*reinterpret_cast<const uint4*>(xr + idx * 8), v[i]);
      if (res) {
        float r[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(res + row * ldr + idx * 8), r);
        const bool native_bf16_add = gemma && std::is_same<T, __nv_bfloat16>::value;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[i][j] = __fadd_rn(v[i][j], r[j]);
          // Gemma adds bf16 natively (layernorm.py:83-87): the normalised input is the rounded sum
          if (native_bf16_add) v[i][j] = to_f32(from_f32<T>(v[i][j]));
        }
        *reinterpret_cast<uint4*>(res_out + row * ldro + idx * 8) = pack8<T>(v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[i][j], v[i][j], ss);
    }
  }
  const float var = block_sum(ss, red) / (float)hidden;
  const float rs = rsqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < nvec) {
      float wf[8], o[8];
      unpack8<T>(*reinterpret_cast<const uint4*>(w + idx * 8), wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xn = __fmul_rn(v[i][j], rs);
        if (gemma) {
          o[j] = __fmul_rn(xn, __fadd_rn(1.f, wf[j]));
        } else {
          // cast to the activation dtype BEFORE the weight multiply (layernorm.py:24-25)
          o[j] = __fmul_rn(to_f32(from_f32<T>(xn)), wf[j]);
        }
      }
      *reinterpret_cast<uint4*>(y + row * ldy + idx * 8) = pack8<T>(o);
    }
  }
}

// ---------------------------------------------------------------------------
// RoPE: one CTA per token; a work item = 8 rotation pairs of one head.
template <typename T>
__global__ void __launch_bounds__(128) rope_kernel(const int64_t* __restrict__ pos, const T* q, int64_t qs,
                                                   const T* k, int64_t ks, T* qo, T* ko, int hq, int hk, int d,
                                                   const float* __restrict__ cs, int64_t max_pos) {
  pdl_wait();
  pdl_trigger();

  const int t = blockIdx.x;
  const int half = d >> 1;
  const int per_head = half >> 3;
  const int items = (hq + hk) * per_head;
  const int64_t p = min(max(__ldg(pos + t), (int64_t)0), max_pos - 1);
  const float* c = cs + p * (int64_t)d;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int h = it / per_head, i0 = (it - h * per_head) * 8;
    const T* src;
    T* dst;
    if (h < hq) {
      src = q + (int64_t)t * qs + (int64_t)h * d;
      dst = qo + ((int64_t)t * hq + h) * d;
    } else {
      src = k + (int64_t)t * ks + (int64_t)(h - hq) * d;
      dst = ko + ((int64_t)t * hk + (h - hq)) * d;
    }
    float x1[8], x2[8], y1[8], y2[8];
    unpack8<T>(*reinterpret_cast<const uint4*>(src + i0), x1);
    unpack8<T>(*reinterpret_cast<const uint4*>(src + half + i0), x2);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float co = __ldg(c + i0 + j), si = __ldg(c + half + i0 + j);
      y1[j] = __fsub_rn(__fmul_rn(x1[j], co), __fmul_rn(x2[j], si));
      y2[j] = __fadd_rn(__fmul_rn(x2[j], co), __fmul_rn(x1[j], si));
    }
    *reinterpret_cast<uint4*>(dst + i0) = pack8<T>(y1);
    *reinterpret_cast<uint4*>(dst + half + i0) = pack8<T>(y2);
  }
}


// ---------------------------------------------------------------------------
// Fused decode prologue of the attention block (Qwen3Attention.forward,
// adallm/architectures/qwen3.py:476-486): per token, per head of the fused qkv row
//   q, k : RMSNorm over head_dim with q_norm / k_norm (skipped when the weight is null),
//          then NeoX RoPE at positions[t]  (rotary_embedding.py:6-14)
//   k, v : e4m3 store into the paged cache at slot_mapping[t] (attention.py:11-31)
//   q    : written to q_out [T, hq, D]; k (normed + roped, bf16) optionally to k_out.
// One warp per (token, head) item, 4 warps per CTA; a lane owns 4 consecutive elements
// and the rotate-half partner lives 16 lanes away.  Implemented for head_dim == 128.
template <typename T>
__global__ void __launch_bounds__(128) qk_norm_rope_store_kernel(
    const T* __restrict__ qkv, int64_t ld, int hq, int hkv, const T* __restrict__ qw, const T* __restrict__ kw,
    float eps, const int64_t* __restrict__ pos, const float* __restrict__ cs, int64_t max_pos,
    const int32_t* __restrict__ slots, uint8_t* __restrict__ kc, uint8_t* __restrict__ vc, float k_scale,
    float v_scale, T* __restrict__ q_out, T* __restrict__ k_out, int64_t num_tokens, PartIn pin, int gemma) {
  pdl_wait();
  pdl_trigger();

  constexpr int D = 128;
  const int lane = threadIdx.x & 31;
  const int nheads = hq + 2 * hkv;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= num_tokens * nheads) return;
  const int64_t t = item / nheads;
  const int h = (int)(item - t * nheads);
  const int64_t p = min(max(__ldg(pos + t), (int64_t)0), max_pos - 1);
  const float* c = cs + p * D;
  const int slot = __ldg(slots + t);
  const int i0 = (lane & 15) * 4;  // rotation-pair index of this lane's first element
  {
    float x[4];
    if (pin.n) {  // the qkv GEMM's split-K planes
      load_parts<T, 4>(pin, t, (int64_t)h * D + lane * 4, x);
    } else {
      const T* src = qkv + (int64_t)t * ld + (int64_t)h * D + lane * 4;
      const uint2 u = *reinterpret_cast<const uint2*>(src);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = to_f32(e[j]);
    }
    const bool is_q = h < hq, is_k = !is_q && h < hq + hkv;
    if (is_q || is_k) {
      const T* w = is_q ? qw : kw;
      if (w) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) ss = fmaf(x[j], x[j], ss);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rs = rsqrtf(ss / (float)D + eps);
        const uint2 wu = *reinterpret_cast<const uint2*>(w + lane * 4);
        const T* we = reinterpret_cast<const T*>(&wu);
        if (gemma) {
#pragma unroll
          for (int j = 0; j < 4; ++j)  // layernorm.py:70-73: x * rs * (1 + w) in fp32, then cast
            x[j] = to_f32(from_f32<T>(__fmul_rn(__fmul_rn(x[j], rs), __fadd_rn(1.f, to_f32(we[j])))));
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)  // layernorm.py:24-25: cast, then weight multiply, cast again
            x[j] = to_f32(from_f32<T>(__fmul_rn(to_f32(from_f32<T>(__fmul_rn(x[j], rs))), to_f32(we[j]))));
        }
      }
      float y[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[j], 16);
        const float co = __ldg(c + i0 + j), si = __ldg(c + D / 2 + i0 + j);
        y[j] = lane < 16 ? __fsub_rn(__fmul_rn(x[j], co), __fmul_rn(partner, si))
                         : __fadd_rn(__fmul_rn(x[j], co), __fmul_rn(partner, si));
        y[j] = to_f32(from_f32<T>(y[j]));
      }
      if (is_q) {
        uint2 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) oe[j] = from_f32<T>(y[j]);
        *reinterpret_cast<uint2*>(q_out + ((int64_t)t * hq + h) * D + lane * 4) = o;
      } else {
        if (k_out) {
          uint2 o;
          T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
          for (int j = 0; j < 4; ++j) oe[j] = from_f32<T>(y[j]);
          *reinterpret_cast<uint2*>(k_out + ((int64_t)t * hkv + (h - hq)) * D + lane * 4) = o;
        }
        if (slot >= 0) {
          float s[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) s[j] = k_scale != 1.f ? __fdiv_rn(y[j], k_scale) : y[j];
          const uint32_t b = (uint32_t)f32x2_to_e4m3x2(s[0], s[1]) | ((uint32_t)f32x2_to_e4m3x2(s[2], s[3]) << 16);
          *reinterpret_cast<uint32_t*>(kc + ((int64_t)slot * hkv + (h - hq)) * D + lane * 4) = b;
        }
      }
    } else if (slot >= 0) {  // v head: straight e4m3 store
      float s[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) s[j] = v_scale != 1.f ? __fdiv_rn(x[j], v_scale) : x[j];
      const uint32_t b = (uint32_t)f32x2_to_e4m3x2(s[0], s[1]) | ((uint32_t)f32x2_to_e4m3x2(s[2], s[3]) << 16);
      *reinterpret_cast<uint32_t*>(vc + ((int64_t)slot * hkv + (h - hq - hkv)) * D + lane * 4) = b;
    }
  }
}

// ---------------------------------------------------------------------------
__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.f, expf(-x))); }
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float inner = k0 * (x + k1 * x * x * x);
  return 0.5f * x * (1.f + tanhf(inner));
}

template <typename T>
__global__ void gated_act_kernel(const T* __restrict__ x, int64_t ldx, T* __restrict__ y, int64_t ldy, int64_t rows,
                                 int inter, int act) {
  pdl_wait();
  pdl_trigger();

  const int nvec = inter >> 3;
  const int64_t total = rows * nvec;
  for (int64_t it = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; it < total; it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = it / nvec;
    const int i = (int)(it - r * nvec) * 8;
    float a[8], b[8], o[8];
    unpack8<T>(*reinterpret_cast<const uint4*>(x + r * ldx + i), a);
    unpack8<T>(*reinterpret_cast<const uint4*>(x + r * ldx + inter + i), b);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float g = act == 0 ? silu_f(a[j]) : gelu_tanh_f(a[j]);
      o[j] = __fmul_rn(to_f32(from_f32<T>(g)), b[j]);  // act rounds to dtype, then the product does
    }
    *reinterpret_cast<uint4*>(y + r * ldy + i) = pack8<T>(o);
  }
}

// ---------------------------------------------------------------------------
__global__ void embedding_kernel(const int64_t* __restrict__ ids, const uint4* __restrict__ table, int64_t v0,
                                 int64_t v1, int nvec, uint4* __restrict__ y) {
  pdl_wait();
  pdl_trigger();

  const int t = blockIdx.x;
  const int64_t id = __ldg(ids + t);
  const bool in = id >= v0 && id < v1;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x)
    y[(int64_t)t * nvec + i] = in ? table[(id - v0) * nvec + i] : make_uint4(0, 0, 0, 0);
}

// Greedy argmax in two stages: stage 1 splits every row into chunks of 8-aligned
// columns (16-byte loads) and writes one (max, index) pair per chunk; stage 2 picks
// the first maximum of each row.  Ties resolve to the lowest index (torch.argmax).
__device__ __forceinline__ void better(float& bv, int64_t& bi, float v, int64_t i) {
  if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

template <typename T>
__global__ void __launch_bounds__(256) argmax_stage1(const T* __restrict__ x, int64_t ld, int64_t cols,
                                                     int64_t chunk, float* __restrict__ pv,
                                                     int64_t* __restrict__ pi) {
  pdl_wait();
  pdl_trigger();

  __shared__ float sv[8];
  __shared__ int64_t si[8];
  const int64_t r = blockIdx.y;
  const int64_t c0 = (int64_t)blockIdx.x * chunk;
  const int64_t c1 = min(cols, c0 + chunk);
  float bv = -INFINITY;
  int64_t bi = 0x7fffffffffffffffLL;
  const T* row = x + r * ld;
  const bool vec = ((ld & 7) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  if (vec) {
    for (int64_t j = c0 + threadIdx.x * 8; j < c1; j += blockDim.x * 8) {
      if (j + 8 <= c1) {
        float f[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(row + j), f);
#pragma unroll
        for (int q = 0; q < 8; ++q) better(bv, bi, f[q], j + q);
      } else {
        for (int64_t q = j; q < c1; ++q) better(bv, bi, to_f32(row[q]), q);
      }
    }
  } else {
    for (int64_t j = c0 + threadIdx.x; j < c1; j += blockDim.x) better(bv, bi, to_f32(row[j]), j);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int q = 1; q < (int)(blockDim.x >> 5); ++q) better(bv, bi, sv[q], si[q]);
    pv[r * gridDim.x + blockIdx.x] = bv;
    pi[r * gridDim.x + blockIdx.x] = bi;
  }
}

__global__ void __launch_bounds__(32) argmax_stage2(const float* __restrict__ pv, const int64_t* __restrict__ pi,
                                                    int chunks, int64_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();

  const int64_t r = blockIdx.x;
  float bv = -INFINITY;
  int64_t bi = 0x7fffffffffffffffLL;
  for (int c = threadIdx.x; c < chunks; c += 32) better(bv, bi, pv[r * chunks + c], pi[r * chunks + c]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  if (threadIdx.x == 0) out[r] = bi == 0x7fffffffffffffffLL ? 0 : bi;
}

static inline int argmax_chunks(int64_t cols) {
  int64_t c = (cols + 2047) / 2048;  // ~2048 columns per CTA
  if (c > 256) c = 256;
  return (int)(c < 1 ? 1 : c);
}

}  // namespace small
}  // namespace ada

using namespace ada;

static inline bool a16(const void* p) { return ((uintptr_t)p & 15) == 0; }

extern "C" int ada_store_kvcache_fp8(const void* key, const void* value, int in_dtype, int64_t num_tokens,
                                     int32_t num_kv_heads, int32_t head_dim, int64_t key_stride, int64_t value_stride,
                                     const int32_t* slot_mapping, uint8_t* k_cache, uint8_t* v_cache,
                                     int64_t cache_row_stride, float k_scale, float v_scale, void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0) return ADA_ERR_INVALID_ARG;
  if (num_tokens == 0) return ADA_OK;
  if (!key || !value || !slot_mapping || !k_cache || !v_cache) return ADA_ERR_INVALID_ARG;
  if (in_dtype != ADA_DT_BF16 && in_dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (!(k_scale > 0.f) || !(v_scale > 0.f)) return ADA_ERR_INVALID_ARG;
  const int hd = num_kv_heads * head_dim;
  if (hd % 8 || cache_row_stride < hd) return ADA_ERR_UNSUPPORTED;
  if (!a16(key) || !a16(value) || (key_stride & 7) || (value_stride & 7)) return ADA_ERR_ALIGNMENT;
  if (((uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)cache_row_stride) & 7) return ADA_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (in_dtype == ADA_DT_BF16)
    (void)ada::launch_k(small::store_kv_kernel<__nv_bfloat16>, dim3((unsigned)num_tokens), dim3(128), 0, st, 
        (const __nv_bfloat16*)key, (const __nv_bfloat16*)value, key_stride, value_stride, slot_mapping, k_cache,
        v_cache, cache_row_stride, hd, k_scale, v_scale);
  else
    (void)ada::launch_k(small::store_kv_kernel<__half>, dim3((unsigned)num_tokens), dim3(128), 0, st, 
        (const __half*)key, (const __half*)value, key_stride, value_stride, slot_mapping, k_cache, v_cache,
        cache_row_stride, hd, k_scale, v_scale);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

template <typename T>
static int launch_rmsnorm(const void* x, int64_t ldx, const void* res, int64_t ldr, void* ro, int64_t ldro,
                          const void* w, void* y, int64_t ldy, int64_t rows, int hidden, float eps, int gemma,
                          cudaStream_t st) {
  const int nvec = hidden / 8;
  int threads = nvec >= 256 ? 256 : ((nvec + 31) / 32) * 32;
  const int per = (nvec + threads - 1) / threads;
#define ADA_RMS(MV)                                                                                         \
  (void)ada::launch_k(small::rmsnorm_kernel<T, MV>, dim3((unsigned)rows), dim3(threads), 0, st, (const T*)x, ldx, (const T*)res, ldr,    \
                                                                   (T*)ro, ldro, (const T*)w, (T*)y, ldy,   \
                                                                   hidden, eps, gemma)
  if (per <= 1) ADA_RMS(1);
  else if (per <= 2) ADA_RMS(2);
  else if (per <= 4) ADA_RMS(4);
  else if (per <= 8) ADA_RMS(8);
  else return ADA_ERR_UNSUPPORTED;
#undef ADA_RMS
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

extern "C" int ada_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ld_res, void* residual_out,
                           int64_t ld_res_out, const void* weight, void* y, int64_t ldy, int64_t rows, int32_t hidden,
                           float eps, int gemma, int dtype, void* stream) {
  if (rows < 0 || hidden <= 0) return ADA_ERR_INVALID_ARG;
  if (rows == 0) return ADA_OK;
  if (!x || !weight || !y || (residual && !residual_out)) return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (hidden % 8) return ADA_ERR_UNSUPPORTED;
  if (!a16(x) || !a16(weight) || !a16(y) || (ldx & 7) || (ldy & 7)) return ADA_ERR_ALIGNMENT;
  if (residual && (!a16(residual) || !a16(residual_out) || (ld_res & 7) || (ld_res_out & 7))) return ADA_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (hidden % 16 == 0 && hidden / 16 <= 4 * 256)
    return ada::fused::launch_rmsnorm16(x, ldx, residual, ld_res, residual_out, ld_res_out, weight, y, ldy, rows,
                                        hidden, eps, gemma, dtype, st);
  if (dtype == ADA_DT_BF16)
    return launch_rmsnorm<__nv_bfloat16>(x, ldx, residual, ld_res, residual_out, ld_res_out, weight, y, ldy, rows,
                                         hidden, eps, gemma, st);
  return launch_rmsnorm<__half>(x, ldx, residual, ld_res, residual_out, ld_res_out, weight, y, ldy, rows, hidden, eps,
                                gemma, st);
}

extern "C" int ada_rope(const int64_t* positions, const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                        void* q_out, void* k_out, int64_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                        int32_t head_dim, const float* cos_sin, int64_t max_position, int dtype, void* stream) {
  if (num_tokens < 0 || num_q_heads < 0 || num_kv_heads < 0 || head_dim <= 0) return ADA_ERR_INVALID_ARG;
  if (num_tokens == 0) return ADA_OK;
  if (!positions || !q || !k || !q_out || !k_out || !cos_sin || max_position <= 0) return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (head_dim % 16) return ADA_ERR_UNSUPPORTED;
  if (!a16(q) || !a16(k) || !a16(q_out) || !a16(k_out) || (q_stride & 7) || (k_stride & 7)) return ADA_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == ADA_DT_BF16)
    (void)ada::launch_k(small::rope_kernel<__nv_bfloat16>, dim3((unsigned)num_tokens), dim3(128), 0, st, 
        positions, (const __nv_bfloat16*)q, q_stride, (const __nv_bfloat16*)k, k_stride, (__nv_bfloat16*)q_out,
        (__nv_bfloat16*)k_out, num_q_heads, num_kv_heads, head_dim, cos_sin, max_position);
  else
    (void)ada::launch_k(small::rope_kernel<__half>, dim3((unsigned)num_tokens), dim3(128), 0, st, positions, (const __half*)q, q_stride,
                                                                     (const __half*)k, k_stride, (__half*)q_out,
                                                                     (__half*)k_out, num_q_heads, num_kv_heads,
                                                                     head_dim, cos_sin, max_position);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

static int qk_norm_rope_store_impl(const void* qkv, int64_t ld, const PartIn& pin, int64_t num_tokens,
                                   int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, const void* q_norm_w,
                                   const void* k_norm_w, float eps, const int64_t* positions, const float* cos_sin,
                                   int64_t max_position, const int32_t* slot_mapping, uint8_t* k_cache,
                                   uint8_t* v_cache, float k_scale, float v_scale, void* q_out, void* k_out, int dtype,
                                   void* stream, int gemma = 0) {
  if (num_tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0) return ADA_ERR_INVALID_ARG;
  if (gemma != 0 && gemma != 1) return ADA_ERR_INVALID_ARG;
  if (num_tokens == 0) return ADA_OK;
  if (!positions || !cos_sin || !slot_mapping || !k_cache || !v_cache || !q_out || max_position <= 0)
    return ADA_ERR_INVALID_ARG;
  if (!(k_scale > 0.f) || !(v_scale > 0.f)) return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (head_dim != 128) return ADA_ERR_UNSUPPORTED;
  const int64_t width = (int64_t)(num_q_heads + 2 * num_kv_heads) * head_dim;
  if (pin.n) {
    if (!parts_ok(pin, num_tokens, width)) return ADA_ERR_INVALID_ARG;
  } else {
    if (!qkv || ld < width) return ADA_ERR_INVALID_ARG;
    if (((uintptr_t)qkv & 7) || (ld & 3)) return ADA_ERR_ALIGNMENT;
  }
  if (((uintptr_t)q_out & 7) || ((uintptr_t)k_out & 7) || ((uintptr_t)q_norm_w & 7) || ((uintptr_t)k_norm_w & 7) ||
      ((uintptr_t)k_cache & 3) || ((uintptr_t)v_cache & 3))
    return ADA_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t items = num_tokens * (num_q_heads + 2 * num_kv_heads);
  const unsigned blocks = (unsigned)((items + 3) / 4);
#define ADA_QK(T)                                                                                                \
  (void)ada::launch_k(small::qk_norm_rope_store_kernel<T>, dim3(blocks), dim3(128), 0, st, (const T*)qkv, ld,      \
                      num_q_heads, num_kv_heads, (const T*)q_norm_w, (const T*)k_norm_w, eps, positions, cos_sin, \
                      max_position, slot_mapping, k_cache, v_cache, k_scale, v_scale, (T*)q_out, (T*)k_out,       \
                      num_tokens, pin, gemma)
  if (dtype == ADA_DT_BF16) ADA_QK(__nv_bfloat16);
  else ADA_QK(__half);
#undef ADA_QK
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

extern "C" int ada_qk_norm_rope_store(const void* qkv, int64_t ld, int64_t num_tokens, int32_t num_q_heads,
                                      int32_t num_kv_heads, int32_t head_dim, const void* q_norm_w,
                                      const void* k_norm_w, float eps, const int64_t* positions, const float* cos_sin,
                                      int64_t max_position, const int32_t* slot_mapping, uint8_t* k_cache,
                                      uint8_t* v_cache, float k_scale, float v_scale, void* q_out, void* k_out,
                                      int dtype, void* stream) {
  return qk_norm_rope_store_impl(qkv, ld, PartIn{nullptr, 0, 0, 0}, num_tokens, num_q_heads, num_kv_heads, head_dim,
                                 q_norm_w, k_norm_w, eps, positions, cos_sin, max_position, slot_mapping, k_cache,
                                 v_cache, k_scale, v_scale, q_out, k_out, dtype, stream);
}

extern "C" int ada_qk_norm_rope_store_parts(const float* parts, int32_t nparts, int64_t plane, int64_t ldp,
                                            int64_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                                            int32_t head_dim, const void* q_norm_w, const void* k_norm_w, float eps,
                                            const int64_t* positions, const float* cos_sin, int64_t max_position,
                                            const int32_t* slot_mapping, uint8_t* k_cache, uint8_t* v_cache,
                                            float k_scale, float v_scale, void* q_out, void* k_out, int dtype,
                                            void* stream) {
  if (nparts < 1) return ADA_ERR_INVALID_ARG;
  return qk_norm_rope_store_impl(nullptr, 0, PartIn{parts, nparts, plane, ldp}, num_tokens, num_q_heads,
                                 num_kv_heads, head_dim, q_norm_w, k_norm_w, eps, positions, cos_sin, max_position,
                                 slot_mapping, k_cache, v_cache, k_scale, v_scale, q_out, k_out, dtype, stream);
}

extern "C" int ada_qk_norm_rope_store_parts_ex(const float* parts, int32_t nparts, int64_t plane, int64_t ldp,
                                               int64_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                                               int32_t head_dim, const void* q_norm_w, const void* k_norm_w, float eps,
                                               int gemma, const int64_t* positions, const float* cos_sin,
                                               int64_t max_position, const int32_t* slot_mapping, uint8_t* k_cache,
                                               uint8_t* v_cache, float k_scale, float v_scale, void* q_out, void* k_out,
                                               int dtype, void* stream) {
  if (nparts < 1) return ADA_ERR_INVALID_ARG;
  return qk_norm_rope_store_impl(nullptr, 0, PartIn{parts, nparts, plane, ldp}, num_tokens, num_q_heads,
                                 num_kv_heads, head_dim, q_norm_w, k_norm_w, eps, positions, cos_sin, max_position,
                                 slot_mapping, k_cache, v_cache, k_scale, v_scale, q_out, k_out, dtype, stream, gemma);
}

extern "C" int ada_qk_norm_rope_store_ex(const void* qkv, int64_t ld, int64_t num_tokens, int32_t num_q_heads,
                                         int32_t num_kv_heads, int32_t head_dim, const void* q_norm_w,
                                         const void* k_norm_w, float eps, int gemma, const int64_t* positions,
                                         const float* cos_sin, int64_t max_position, const int32_t* slot_mapping,
                                         uint8_t* k_cache, uint8_t* v_cache, float k_scale, float v_scale, void* q_out,
                                         void* k_out, int dtype, void* stream) {
  return qk_norm_rope_store_impl(qkv, ld, PartIn{nullptr, 0, 0, 0}, num_tokens, num_q_heads, num_kv_heads, head_dim,
                                 q_norm_w, k_norm_w, eps, positions, cos_sin, max_position, slot_mapping, k_cache,
                                 v_cache, k_scale, v_scale, q_out, k_out, dtype, stream, gemma);
}

extern "C" int ada_gated_act(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t rows, int32_t inter, int act,
                             int dtype, void* stream) {
  if (rows < 0 || inter <= 0 || (act != 0 && act != 1)) return ADA_ERR_INVALID_ARG;
  if (rows == 0) return ADA_OK;
  if (!x || !y) return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (inter % 8) return ADA_ERR_UNSUPPORTED;
  if (!a16(x) || !a16(y) || (ldx & 7) || (ldy & 7)) return ADA_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t total = rows * (inter / 8);
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 8);
  if (dtype == ADA_DT_BF16)
    (void)ada::launch_k(small::gated_act_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st, (const __nv_bfloat16*)x, ldx, (__nv_bfloat16*)y,
                                                                   ldy, rows, inter, act);
  else
    (void)ada::launch_k(small::gated_act_kernel<__half>, dim3(blocks), dim3(256), 0, st, (const __half*)x, ldx, (__half*)y, ldy, rows, inter, act);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

extern "C" int ada_embedding(const int64_t* ids, int64_t num_tokens, const void* table, int64_t vocab_start,
                             int64_t vocab_end, int32_t hidden, void* y, int dtype, void* stream) {
  if (num_tokens < 0 || hidden <= 0 || vocab_end < vocab_start) return ADA_ERR_INVALID_ARG;
  if (num_tokens == 0) return ADA_OK;
  if (!ids || !table || !y) return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (hidden % 8) return ADA_ERR_UNSUPPORTED;
  if (!a16(table) || !a16(y)) return ADA_ERR_ALIGNMENT;
  (void)ada::launch_k(small::embedding_kernel, dim3((unsigned)num_tokens), dim3(128), 0, reinterpret_cast<cudaStream_t>(stream), 
      ids, (const uint4*)table, vocab_start, vocab_end, hidden / 8, (uint4*)y);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

extern "C" size_t ada_argmax_workspace_size(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return (size_t)rows * small::argmax_chunks(cols) * (sizeof(float) + sizeof(int64_t)) + 16;
}

extern "C" int ada_argmax(const void* logits, int64_t ld, int64_t rows, int64_t cols, int dtype, int64_t* out,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (rows < 0 || cols <= 0 || ld < cols) return ADA_ERR_INVALID_ARG;
  if (rows == 0) return ADA_OK;
  if (!logits || !out || !workspace) return ADA_ERR_INVALID_ARG;
  if (rows > 65535) return ADA_ERR_UNSUPPORTED;
  if (workspace_bytes < ada_argmax_workspace_size(rows, cols)) return ADA_ERR_WORKSPACE;
  if ((uintptr_t)workspace & 7) return ADA_ERR_ALIGNMENT;
  const int chunks = small::argmax_chunks(cols);
  const int64_t chunk = ((cols + chunks - 1) / chunks + 7) & ~int64_t(7);
  int64_t* pi = reinterpret_cast<int64_t*>(workspace);
  float* pv = reinterpret_cast<float*>(pi + rows * chunks);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dim3 g1(chunks, (unsigned)rows);
  if (dtype == ADA_DT_BF16)
    (void)ada::launch_k(small::argmax_stage1<__nv_bfloat16>, dim3(g1), dim3(256), 0, st, (const __nv_bfloat16*)logits, ld, cols, chunk, pv, pi);
  else if (dtype == ADA_DT_F16)
    (void)ada::launch_k(small::argmax_stage1<__half>, dim3(g1), dim3(256), 0, st, (const __half*)logits, ld, cols, chunk, pv, pi);
  else
    return ADA_ERR_INVALID_ARG;
  ADA_CHECK_LAUNCH();
  (void)ada::launch_k(small::argmax_stage2, dim3((unsigned)rows), dim3(32), 0, st, pv, pi, chunks, out);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

// ---------------------------------------------------------------------------
// Greedy argmax without a caller workspace.  For callers that cannot allocate device
// memory where they sample: a host runtime that binds this C ABI directly (no caching
// allocator) and launches into work it is recording, where cudaMalloc is not allowed.
// The two stages exchange their per-chunk partials through this file-scope scratch instead.
// Limit: rows * chunks(cols) * 12 + 16 <= ADA_ARGMAX_SCRATCH_BYTES (256 KiB; the Qwen3 vocab
// of 151936 splits into 75 chunks, so up to 291 rows).  Nothing in it needs to start at zero:
// stage 1 writes every (row, chunk) slot before stage 2 reads it.  One scratch per device:
// calls that overlap in time on one device (different streams, or host threads) race.
#define ADA_ARGMAX_SCRATCH_BYTES (256u * 1024u)
static __device__ __align__(256) unsigned char g_argmax_scratch[ADA_ARGMAX_SCRATCH_BYTES];

// Device address of g_argmax_scratch for the current device, looked up once per device (the
// first call on each device; make it before capturing launches into a graph -- a call with
// rows == 0 does only this look-up).  Host threads may race on the first look-up of a device:
// the entries are atomics, and every writer stores the same address.
static int argmax_scratch(void** ptr) {
  static std::atomic<void*> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ADA_ERR_CUDA;
  void* p = cache[dev].load(std::memory_order_acquire);
  if (!p) {
    if (cudaGetSymbolAddress(&p, g_argmax_scratch) != cudaSuccess || !p) {
      (void)cudaGetLastError();
      return ADA_ERR_CUDA;
    }
    cache[dev].store(p, std::memory_order_release);
  }
  *ptr = p;
  return ADA_OK;
}

extern "C" int ada_argmax_noalloc(const void* logits, int64_t ld, int64_t rows, int64_t cols, int dtype,
                                  int64_t* out, void* stream) {
  if (rows < 0 || cols <= 0 || ld < cols) return ADA_ERR_INVALID_ARG;
  void* scratch = nullptr;
  if (rows == 0) return argmax_scratch(&scratch);  // set-up only: the per-device look-up
  if (!logits || !out) return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (rows > 65535) return ADA_ERR_UNSUPPORTED;
  if (ada_argmax_workspace_size(rows, cols) > ADA_ARGMAX_SCRATCH_BYTES) return ADA_ERR_WORKSPACE;
  const int rc = argmax_scratch(&scratch);
  if (rc != ADA_OK) return rc;
  const int chunks = small::argmax_chunks(cols);
  const int64_t chunk = ((cols + chunks - 1) / chunks + 7) & ~int64_t(7);
  int64_t* pi = reinterpret_cast<int64_t*>(scratch);
  float* pv = reinterpret_cast<float*>(pi + rows * chunks);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 g1(chunks, (unsigned)rows);
  if (dtype == ADA_DT_BF16)
    (void)ada::launch_k(small::argmax_stage1<__nv_bfloat16>, g1, dim3(256), 0, st, (const __nv_bfloat16*)logits, ld,
                        cols, chunk, pv, pi);
  else
    (void)ada::launch_k(small::argmax_stage1<__half>, g1, dim3(256), 0, st, (const __half*)logits, ld, cols, chunk, pv,
                        pi);
  ADA_CHECK_LAUNCH();
  (void)ada::launch_k(small::argmax_stage2, dim3((unsigned)rows), dim3(32), 0, st, pv, pi, chunks, out);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

extern "C" const char* ada_status_string(int status) {
  switch (status) {
    case ADA_OK: return "ok";
    case ADA_ERR_INVALID_ARG: return "invalid argument";
    case ADA_ERR_UNSUPPORTED: return "unsupported shape or configuration";
    case ADA_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case ADA_ERR_WORKSPACE: return "workspace too small";
    case ADA_ERR_LAUNCH: return "kernel launch failed";
    case ADA_ERR_TIMEOUT: return "device-side wait timed out";
    case ADA_ERR_CUDA: return "CUDA runtime error";
    default: return "unknown status";
  }
}

extern "C" int ada_abi_version(void) { return 1; }

extern "C" int ada_set_pdl(int enable) {
  const int prev = ada::g_pdl_enabled ? 1 : 0;
  ada::g_pdl_enabled = enable != 0;
  return prev;
}
