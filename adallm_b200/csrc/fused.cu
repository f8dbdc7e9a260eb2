// Producers of the NVFP4 GEMM operand with the activation quantiser fused in
// (layout and arithmetic: quant.cuh), so a decode layer needs no separate
// quantisation launch before its four projections:
//   * residual-add + RMSNorm / GemmaRMSNorm -> quantised operand of qkv_proj / gate_up_proj
//     (reference adallm/ops/layernorm.py:16-40, :64-92)
//   * SiLU(gate) * up / GELU(tanh)(gate) * up -> quantised operand of down_proj
//     (reference adallm/ops/activation.py:6-26)
//   * plain quantisation of a bf16/fp16 matrix (the prologue of ada_nvfp4_linear)
// The bf16 value each kernel quantises is exactly the value the unfused op would have returned
// (same rounding order).  The gated-activation and plain producers quantise it exactly as
// ada_nvfp4_act_quant does; the RMSNorm producers scale by a bound on the row amax carried with
// the sum of squares (one cluster exchange instead of two), with the same codes for that scale.
//
// Decode rows are short (16 tokens x 4096..21504 values), so each row is spread over
// a thread-block cluster of up to 8 CTAs (cluster.cuh): grid (ctas, rows), every CTA
// owns a contiguous slice of the row, and the row reductions (sum of squares, amax)
// are combined across the cluster through distributed shared memory.
#include <type_traits>

#include "cluster.cuh"
#include "parts.cuh"
#include "quant.cuh"

namespace ada {
namespace fused {

template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f32(from_f32<T>(v));
}

// 1 + 2^-6: the margin of the RMSNorm producers' bound on the normalised row's amax.
constexpr float AMAX_BOUND_MARGIN = 1.015625f;

// Octet `u` of this thread (u < MAXU) in the CTA's slice [o0, o1), or -1.
__device__ __forceinline__ int my_oct(int u, int o0, int o1) {
  const int o = o0 + (int)threadIdx.x + u * (int)blockDim.x;
  return o < o1 ? o : -1;
}
__device__ __forceinline__ void slice_of(int k, int& o0, int& o1) {
  o0 = cl::slice_octet(k >> 4, blockIdx.x, gridDim.x);
  o1 = cl::slice_octet(k >> 4, blockIdx.x + 1, gridDim.x);
}

// Quantise the slice held in v once the row amax is known; CTA 0 records the row scale.
// Every thread calls it (terms == 1 pairs lanes of a warp).
template <int MAXU>
__device__ __forceinline__ void quant_slice(const q::QuantDst& dst, int m, float (&v)[MAXU][8], int o0, int o1,
                                            float amax) {
  const q::RowQ rq = q::make_rowq(amax, dst.terms);
  if (blockIdx.x == 0 && threadIdx.x == 0) dst.gx[m] = rq.g[0];
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int o = my_oct(u, o0, o1);
    q::quant_oct(dst, m, o < 0 ? 0 : o, v[u], rq, o >= 0);
  }
}
// Padding token of the last token tile: zero codes, unit scale.
__device__ __forceinline__ void zero_slice(const q::QuantDst& dst, int m, int o0, int o1) {
  for (int o = o0 + (int)threadIdx.x; o < o1; o += blockDim.x) q::zero_oct(dst, m, o);
  if (blockIdx.x == 0 && threadIdx.x == 0) dst.gx[m] = 1.f;
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* f) {
  unpack8<T>(*reinterpret_cast<const uint4*>(p), f);
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float* f) {
  *reinterpret_cast<uint4*>(p) = pack8<T>(f);
}

// grid (ctas, m_pad), cluster (ctas, 1, 1).  dst.xq == null: plain RMSNorm (ada_rmsnorm).
// wpre != null: the loaded row first goes through a GemmaRMSNorm of its own (weight wpre; the
// post-attention / post-feedforward norm of a Gemma3 layer, applied to the projection output
// before it joins the residual stream), then the residual add and the main norm as usual.
template <typename T, int MAXU>
__global__ void __launch_bounds__(512) rmsnorm_quant_kernel(const T* __restrict__ x, int64_t ldx, const T* res,
                                                            int64_t ldr, T* res_out, int64_t ldro,
                                                            const T* __restrict__ w, const T* __restrict__ wpre, T* y,
                                                            int64_t ldy, int rows, int hidden, float eps, int gemma,
                                                            q::QuantDst dst, PartIn pin, PeerWait pw, SlotIn sin) {
  __shared__ float red[2 * cl::MAX_WARPS];
  __shared__ cl::Exchange xpre;    // the Gemma post-norm's sum of squares
  __shared__ cl::Exchange2 xmain;  // the sum of squares and max |x * w| together
  if (threadIdx.x == 0) {
    cl::exchange2_init(&xmain);
    if (wpre) cl::exchange_init(&xpre);
    cl::fence_exchange_init();
  }
  cl::cluster_arrive_relaxed();
  const int m = blockIdx.y;
  int o0, o1;
  slice_of(hidden, o0, o1);
  const bool quant = dst.xq != nullptr;
  float wf[MAXU][8];  // the norm weights never depend on the previous kernel: load them first
  float wp[MAXU][8];
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int o = my_oct(u, o0, o1);
    if (o >= 0 && m < rows) {
      load8<T>(w + o * 8, wf[u]);
      if (wpre) load8<T>(wpre + o * 8, wp[u]);
    }
  }
  pdl_wait();
  pdl_trigger();
  if (m >= rows) {
    if (quant) zero_slice(dst, m, o0, o1);
    cl::cluster_wait();
    return;
  }
  const unsigned int tag = pw.epoch ? peer_tag(pw) : 0u;
  float v[MAXU][8];
  float ss = 0.f, aw = 0.f;
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int o = my_oct(u, o0, o1);
    if (o >= 0) {
      if (pw.epoch)  // tensor parallelism: every rank's planes, polled until this step's tag
        load_parts_tagged<T, 8>(pin, m, o * 8, pw, tag, v[u]);
      else if (pin.n)
        load_parts<T, 8>(pin, m, o * 8, v[u]);  // the producing GEMM's split-K planes
      else if (sin.y)
        load_slots<T, 8>(sin, m, o * 8, v[u]);  // the MoE block's weighted combine of the expert rows
      else
        load8<T>(x + (int64_t)m * ldx + o * 8, v[u]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
    }
  }
  if (wpre) {  // GemmaRMSNorm of the loaded row (layernorm.py:64-74): x * rs * (1 + w), then cast
    float ss0 = 0.f;
#pragma unroll
    for (int u = 0; u < MAXU; ++u)
#pragma unroll
      for (int i = 0; i < 8; ++i) ss0 = fmaf(v[u][i], v[u][i], ss0);
    cl::cluster_wait();
    const float rs0 = rsqrtf(cl::cluster_allreduce_x<cl::OpSum>(ss0, red, &xpre) / (float)hidden + eps);
#pragma unroll
    for (int u = 0; u < MAXU; ++u)
      if (my_oct(u, o0, o1) >= 0)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v[u][i] = round_to<T>(__fmul_rn(__fmul_rn(v[u][i], rs0), __fadd_rn(1.f, wp[u][i])));
  }
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int o = my_oct(u, o0, o1);
    if (o >= 0) {
      if (res) {
        float r[8];
        load8<T>(res + (int64_t)m * ldr + o * 8, r);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[u][i] = __fadd_rn(v[u][i], r[i]);
          if (gemma && std::is_same<T, __nv_bfloat16>::value) v[u][i] = round_to<T>(v[u][i]);
        }
        store8<T>(res_out + (int64_t)m * ldro + o * 8, v[u]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ss = fmaf(v[u][i], v[u][i], ss);
        aw = fmaxf(aw, fabsf(__fmul_rn(v[u][i], gemma ? __fadd_rn(1.f, wf[u][i]) : wf[u][i])));
      }
    }
  }
  if (!wpre) cl::cluster_wait();  // all CTAs of the cluster run: their shared memory may be written
  // One exchange for both row reductions.  The quantiser's row scale comes from the bound
  // rs * max|x * w| * (1 + 2^-6) on the normalised row's amax instead of its exact value: the
  // normalised element is x * rs * w rounded to bf16 at most twice (a factor <= (1 + 2^-8)^2 over
  // the exact product), so the bound is never below it, and the terms never saturate.
  const float2 red2 = cl::cluster_allreduce2_x<cl::OpSum, cl::OpMax>(ss, aw, red, &xmain);
  const float rs = rsqrtf(red2.x / (float)hidden + eps);
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int o = my_oct(u, o0, o1);
    if (o >= 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xn = __fmul_rn(v[u][i], rs);
        v[u][i] = gemma ? round_to<T>(__fmul_rn(xn, __fadd_rn(1.f, wf[u][i])))
                        : round_to<T>(__fmul_rn(round_to<T>(xn), wf[u][i]));
      }
      if (y) store8<T>(y + (int64_t)m * ldy + o * 8, v[u]);
    }
  }
  if (!quant) return;
  quant_slice<MAXU>(dst, m, v, o0, o1, __fmul_rn(__fmul_rn(rs, red2.y), AMAX_BOUND_MARGIN));
}

// SiLU with the hardware exponential (within 2 ulp of fp32 before the bf16 rounding).
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.f + __expf(-x)); }
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float inner = k0 * (x + k1 * x * x * x);
  return 0.5f * x * (1.f + tanhf(inner));
}

// grid (ctas, m_pad), cluster (ctas, 1, 1).  Grouped operands (dest != null): grid (ctas, rows),
// input row r goes to operand row dest[r] (< 0: not routed here, nothing written).
template <typename T, int MAXU>
__global__ void __launch_bounds__(512) gated_act_quant_kernel(const T* __restrict__ x, int64_t ldx, T* y, int64_t ldy,
                                                              int rows, int inter, int act, q::QuantDst dst,
                                                              PartIn pin, const int* dest) {
  __shared__ float red[cl::MAX_WARPS];
  __shared__ cl::Exchange xch;
  cl::cluster_start(&xch, 1);
  pdl_wait();
  pdl_trigger();
  const int src = blockIdx.y;
  const int m = dest ? dest[src] : src;
  int o0, o1;
  slice_of(inter, o0, o1);
  if (m < 0) {  // cluster-uniform: every CTA of the cluster has this row
    cl::cluster_wait();
    return;
  }
  if (src >= rows) {
    zero_slice(dst, m, o0, o1);
    cl::cluster_wait();
    return;
  }
  float v[MAXU][8];
  float amax = 0.f;
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int o = my_oct(u, o0, o1);
    if (o >= 0) {
      float gt[8], up[8];
      if (pin.n) {
        load_parts<T, 8>(pin, src, o * 8, gt);
        load_parts<T, 8>(pin, src, inter + o * 8, up);
      } else {
        load8<T>(x + (int64_t)src * ldx + o * 8, gt);
        load8<T>(x + (int64_t)src * ldx + inter + o * 8, up);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float a = act == 0 ? silu_f(gt[i]) : gelu_tanh_f(gt[i]);
        v[u][i] = round_to<T>(__fmul_rn(round_to<T>(a), up[i]));
        amax = fmaxf(amax, fabsf(v[u][i]));
      }
      if (y) store8<T>(y + (int64_t)src * ldy + o * 8, v[u]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
    }
  }
  cl::cluster_wait();
  quant_slice<MAXU>(dst, m, v, o0, o1, cl::cluster_allreduce_x<cl::OpMax>(amax, red, &xch));
}

// grid (ctas, m_pad), cluster (ctas, 1, 1): operand row m from input row m; rows past `rows`
// are zero padding.  Grouped operands (dest != null): grid (ctas, rows), input row r goes to
// operand row dest[r] (< 0: not routed here, nothing written); the operand rows no input row
// maps to are left as they are, since the grouped GEMM discards their output columns.
// row_div > 1: input row r reads row r / row_div of x (the rows of a token's expert slots all
// read that token's row: the gather of the grouped MoE operand).
template <typename T, int MAXU>
__global__ void __launch_bounds__(512) act_quant_kernel(const T* __restrict__ x, int64_t ldx, int rows, int k,
                                                        q::QuantDst dst, const int* dest, int row_div) {
  __shared__ float red[cl::MAX_WARPS];
  __shared__ cl::Exchange xch;
  cl::cluster_start(&xch, 1);
  pdl_wait();
  pdl_trigger();
  const int src = blockIdx.y;
  const int m = dest ? dest[src] : src;
  int o0, o1;
  slice_of(k, o0, o1);
  if (m < 0) {  // cluster-uniform: every CTA of the cluster has this row
    cl::cluster_wait();
    return;
  }
  if (src >= rows) {
    zero_slice(dst, m, o0, o1);
    cl::cluster_wait();
    return;
  }
  float v[MAXU][8];
  float amax = 0.f;
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int o = my_oct(u, o0, o1);
    if (o >= 0) {
      load8<T>(x + (int64_t)(src / row_div) * ldx + o * 8, v[u]);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[u][i]));
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
    }
  }
  cl::cluster_wait();
  quant_slice<MAXU>(dst, m, v, o0, o1, cl::cluster_allreduce_x<cl::OpMax>(amax, red, &xch));
}

static inline bool a16(const void* p) { return ((uintptr_t)p & 15) == 0; }

bool quant_args_ok(const q::QuantDst& d) {
  if (!q::dst_ok(d.terms, d.bn, d.k)) return false;
  if (!d.xq || !d.gx || (d.terms == 1 && !d.sfx)) return false;
  return a16(d.xq) && ((uintptr_t)d.gx & 3) == 0;
}

// Row kernels dispatch on the dtype and on the per-thread unit count of the row split.
#define ADA_ROW_DISPATCH(KERNEL, T_, SPLIT, ...)                                                       \
  do {                                                                                                 \
    const dim3 blk_((unsigned)(SPLIT).threads);                                                        \
    switch ((SPLIT).maxu) {                                                                            \
      case 1: err_ = launch_kc(KERNEL<T_, 1>, grid_, blk_, 0, st, (SPLIT).ctas, __VA_ARGS__); break;   \
      case 2: err_ = launch_kc(KERNEL<T_, 2>, grid_, blk_, 0, st, (SPLIT).ctas, __VA_ARGS__); break;   \
      case 4: err_ = launch_kc(KERNEL<T_, 4>, grid_, blk_, 0, st, (SPLIT).ctas, __VA_ARGS__); break;   \
      default: err_ = launch_kc(KERNEL<T_, 8>, grid_, blk_, 0, st, (SPLIT).ctas, __VA_ARGS__); break;  \
    }                                                                                                  \
  } while (0)

// RMSNorm (quantised or not) of `launch_rows` rows (rows beyond `rows` are padding).
int launch_rmsnorm(const void* x, int64_t ldx, const void* res, int64_t ldr, void* ro, int64_t ldro, const void* w,
                   void* y, int64_t ldy, int64_t rows, int64_t launch_rows, int hidden, float eps, int gemma,
                   int dtype, const q::QuantDst& dst, cudaStream_t st, const PartIn& pin = PartIn{nullptr, 0, 0, 0},
                   const PeerWait& pw = PeerWait{nullptr, 0, 0, nullptr}, const void* wpre = nullptr,
                   const SlotIn& sin = SlotIn{nullptr, 0, nullptr, 0}) {
  if (hidden % 16) return ADA_ERR_UNSUPPORTED;
  const cl::RowSplit sp = cl::row_split(hidden / 16);
  if (!sp.maxu || launch_rows > 65535) return ADA_ERR_UNSUPPORTED;
  const dim3 grid_((unsigned)sp.ctas, (unsigned)launch_rows);
  cudaError_t err_;
  if (dtype == ADA_DT_BF16) {
    using TT = __nv_bfloat16;
    ADA_ROW_DISPATCH(rmsnorm_quant_kernel, TT, sp, (const TT*)x, ldx, (const TT*)res, ldr, (TT*)ro, ldro,
                     (const TT*)w, (const TT*)wpre, (TT*)y, ldy, (int)rows, hidden, eps, gemma, dst, pin, pw, sin);
  } else {
    using TT = __half;
    ADA_ROW_DISPATCH(rmsnorm_quant_kernel, TT, sp, (const TT*)x, ldx, (const TT*)res, ldr, (TT*)ro, ldro,
                     (const TT*)w, (const TT*)wpre, (TT*)y, ldy, (int)rows, hidden, eps, gemma, dst, pin, pw, sin);
  }
  return err_ == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

// Plain RMSNorm through the same kernel (ada_rmsnorm for hidden % 16 == 0), so fused and
// unfused paths round identically.
int launch_rmsnorm16(const void* x, int64_t ldx, const void* res, int64_t ldr, void* ro, int64_t ldro,
                     const void* w, void* y, int64_t ldy, int64_t rows, int hidden, float eps, int gemma, int dtype,
                     cudaStream_t st) {
  const q::QuantDst none{nullptr, nullptr, nullptr, 1, 16, hidden};
  return launch_rmsnorm(x, ldx, res, ldr, ro, ldro, w, y, ldy, rows, rows, hidden, eps, gemma, dtype, none, st);
}

// Quantise x [m, k] into the GEMM operand (prologue of ada_nvfp4_linear).
int launch_act_quant(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t m_pad, const q::QuantDst& dst,
                     cudaStream_t st, const int* dest = nullptr, int row_div = 1) {
  const cl::RowSplit sp = cl::row_split(dst.k / 16);
  if (!sp.maxu || m_pad > 65535) return ADA_ERR_UNSUPPORTED;
  const dim3 grid_((unsigned)sp.ctas, (unsigned)(dest ? m : m_pad));
  cudaError_t err_;
  if (x_dtype == ADA_DT_BF16) {
    using TT = __nv_bfloat16;
    ADA_ROW_DISPATCH(act_quant_kernel, TT, sp, (const TT*)x, ldx, (int)m, dst.k, dst, dest, row_div);
  } else {
    using TT = __half;
    ADA_ROW_DISPATCH(act_quant_kernel, TT, sp, (const TT*)x, ldx, (int)m, dst.k, dst, dest, row_div);
  }
  return err_ == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace fused
}  // namespace ada

using namespace ada;

extern "C" int ada_rmsnorm_quant(const void* x, int64_t ldx, const void* residual, int64_t ld_res, void* residual_out,
                                 int64_t ld_res_out, const void* weight, void* y, int64_t ldy, int64_t rows,
                                 int32_t hidden, float eps, int gemma, int dtype, int terms, int block_n, uint8_t* xq,
                                 uint8_t* sfx, float* gx, void* stream) {
  if (rows <= 0 || hidden <= 0 || !x || !weight || (residual && !residual_out)) return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  const q::QuantDst dst{xq, sfx, gx, terms, block_n, hidden};
  if (!fused::quant_args_ok(dst)) return ADA_ERR_INVALID_ARG;
  if (!fused::a16(x) || !fused::a16(weight) || (ldx & 7) || (y && (!fused::a16(y) || (ldy & 7))))
    return ADA_ERR_ALIGNMENT;
  if (residual && (!fused::a16(residual) || !fused::a16(residual_out) || (ld_res & 7) || (ld_res_out & 7)))
    return ADA_ERR_ALIGNMENT;
  const int64_t m_pad = cdiv(rows, block_n) * block_n;
  return fused::launch_rmsnorm(x, ldx, residual, ld_res, residual_out, ld_res_out, weight, y, ldy, rows, m_pad,
                               hidden, eps, gemma, dtype, dst, reinterpret_cast<cudaStream_t>(stream));
}

namespace ada {
namespace fused {
int gated_act_quant_impl(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t rows, int32_t inter, int act,
                         int dtype, int terms, int block_n, uint8_t* xq, uint8_t* sfx, float* gx, void* stream,
                         const PartIn& pin, const int* dest) {
  if (rows <= 0 || inter <= 0 || (act != 0 && act != 1)) return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  const q::QuantDst dst{xq, sfx, gx, terms, block_n, inter};
  if (!fused::quant_args_ok(dst)) return ADA_ERR_INVALID_ARG;
  if (pin.n) {
    if (!parts_ok(pin, rows, 2 * (int64_t)inter)) return ADA_ERR_INVALID_ARG;
  } else if (!x) {
    return ADA_ERR_INVALID_ARG;
  } else if (!fused::a16(x) || (ldx & 7)) {
    return ADA_ERR_ALIGNMENT;
  }
  if (y && (!fused::a16(y) || (ldy & 7))) return ADA_ERR_ALIGNMENT;
  const cl::RowSplit sp = cl::row_split(inter / 16);
  const int64_t m_pad = dest ? rows : cdiv(rows, block_n) * block_n;  // grouped rows: no padding rows
  if (!sp.maxu || m_pad > 65535) return ADA_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid_((unsigned)sp.ctas, (unsigned)m_pad);
  cudaError_t err_;
  if (dtype == ADA_DT_BF16) {
    using TT = __nv_bfloat16;
    ADA_ROW_DISPATCH(gated_act_quant_kernel, TT, sp, (const TT*)x, ldx, (TT*)y, ldy, (int)rows, (int)inter, act, dst,
                     pin, dest);
  } else {
    using TT = __half;
    ADA_ROW_DISPATCH(gated_act_quant_kernel, TT, sp, (const TT*)x, ldx, (TT*)y, ldy, (int)rows, (int)inter, act, dst,
                     pin, dest);
  }
  return err_ == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}
}  // namespace fused
}  // namespace ada

extern "C" int ada_gated_act_quant(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t rows, int32_t inter,
                                   int act, int dtype, int terms, int block_n, uint8_t* xq, uint8_t* sfx, float* gx,
                                   void* stream) {
  return fused::gated_act_quant_impl(x, ldx, y, ldy, rows, inter, act, dtype, terms, block_n, xq, sfx, gx, stream,
                                     PartIn{nullptr, 0, 0, 0}, nullptr);
}

extern "C" int ada_gated_act_quant_parts(const float* parts, int32_t nparts, int64_t plane, int64_t ldp, void* y,
                                         int64_t ldy, int64_t rows, int32_t inter, int act, int dtype, int terms,
                                         int block_n, uint8_t* xq, uint8_t* sfx, float* gx, void* stream) {
  if (nparts < 1) return ADA_ERR_INVALID_ARG;
  return fused::gated_act_quant_impl(nullptr, 0, y, ldy, rows, inter, act, dtype, terms, block_n, xq, sfx, gx,
                                     stream, PartIn{parts, nparts, plane, ldp}, nullptr);
}

static int rmsnorm_quant_parts_impl(const float* parts, int32_t nparts, int64_t plane, int64_t ldp,
                                    const void* residual, int64_t ld_res, void* residual_out, int64_t ld_res_out,
                                    const void* weight, void* y, int64_t ldy, int64_t rows, int32_t hidden, float eps,
                                    int gemma, int dtype, int terms, int block_n, uint8_t* xq, uint8_t* sfx, float* gx,
                                    void* stream, const PeerWait& pw, const void* pre_weight = nullptr) {
  if (rows <= 0 || hidden <= 0 || !weight || (residual && !residual_out) || nparts < 1) return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  const PartIn pin{parts, nparts, plane, ldp};
  if (!parts_ok(pin, rows, hidden)) return ADA_ERR_INVALID_ARG;
  const bool quant = xq != nullptr;  // without a quantised output this is a plain RMSNorm into y
  const q::QuantDst dst{xq, sfx, gx, quant ? terms : 1, quant ? block_n : 16, hidden};
  if (quant ? !fused::quant_args_ok(dst) : !y) return ADA_ERR_INVALID_ARG;
  if (!fused::a16(weight) || (y && (!fused::a16(y) || (ldy & 7)))) return ADA_ERR_ALIGNMENT;
  if (pre_weight && !fused::a16(pre_weight)) return ADA_ERR_ALIGNMENT;
  if (residual && (!fused::a16(residual) || !fused::a16(residual_out) || (ld_res & 7) || (ld_res_out & 7)))
    return ADA_ERR_ALIGNMENT;
  const int64_t launch_rows = quant ? cdiv(rows, block_n) * block_n : rows;
  return fused::launch_rmsnorm(nullptr, 0, residual, ld_res, residual_out, ld_res_out, weight, y, ldy, rows,
                               launch_rows, hidden, eps, gemma, dtype, dst, reinterpret_cast<cudaStream_t>(stream), pin,
                               pw, pre_weight);
}

extern "C" int ada_rmsnorm_quant_combine(const void* y_rows, int64_t ld_rows, const void* route_w, int32_t topk,
                                         const void* residual, int64_t ld_res, void* residual_out, int64_t ld_res_out,
                                         const void* weight, void* y, int64_t ldy, int64_t rows, int32_t hidden,
                                         float eps, int gemma, int dtype, int terms, int block_n, uint8_t* xq,
                                         uint8_t* sfx, float* gx, void* stream) {
  if (rows <= 0 || hidden <= 0 || !weight || !y_rows || !route_w || topk < 1 || ld_rows < hidden ||
      (residual && !residual_out))
    return ADA_ERR_INVALID_ARG;
  if (dtype != ADA_DT_BF16 && dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  const bool quant = xq != nullptr;  // without a quantised output this is a plain RMSNorm into y
  const q::QuantDst dst{xq, sfx, gx, quant ? terms : 1, quant ? block_n : 16, hidden};
  if (quant ? !fused::quant_args_ok(dst) : !y) return ADA_ERR_INVALID_ARG;
  if (!fused::a16(weight) || !fused::a16(y_rows) || (ld_rows & 7) || (y && (!fused::a16(y) || (ldy & 7))))
    return ADA_ERR_ALIGNMENT;
  if (residual && (!fused::a16(residual) || !fused::a16(residual_out) || (ld_res & 7) || (ld_res_out & 7)))
    return ADA_ERR_ALIGNMENT;
  const int64_t launch_rows = quant ? cdiv(rows, block_n) * block_n : rows;
  return fused::launch_rmsnorm(nullptr, 0, residual, ld_res, residual_out, ld_res_out, weight, y, ldy, rows,
                               launch_rows, hidden, eps, gemma, dtype, dst, reinterpret_cast<cudaStream_t>(stream),
                               PartIn{nullptr, 0, 0, 0}, PeerWait{nullptr, 0, 0, nullptr}, nullptr,
                               SlotIn{y_rows, ld_rows, route_w, topk});
}

extern "C" int ada_gemma_norm2_quant_parts(const float* parts, int32_t nparts, int64_t plane, int64_t ldp,
                                           const void* post_weight, const void* residual, int64_t ld_res,
                                           void* residual_out, int64_t ld_res_out, const void* weight, void* y,
                                           int64_t ldy, int64_t rows, int32_t hidden, float eps, int dtype, int terms,
                                           int block_n, uint8_t* xq, uint8_t* sfx, float* gx, void* stream) {
  if (!post_weight || !residual) return ADA_ERR_INVALID_ARG;
  return rmsnorm_quant_parts_impl(parts, nparts, plane, ldp, residual, ld_res, residual_out, ld_res_out, weight, y,
                                  ldy, rows, hidden, eps, 1, dtype, terms, block_n, xq, sfx, gx, stream,
                                  PeerWait{nullptr, 0, 0, nullptr}, post_weight);
}

extern "C" int ada_rmsnorm_quant_parts(const float* parts, int32_t nparts, int64_t plane, int64_t ldp,
                                       const void* residual, int64_t ld_res, void* residual_out, int64_t ld_res_out,
                                       const void* weight, void* y, int64_t ldy, int64_t rows, int32_t hidden,
                                       float eps, int gemma, int dtype, int terms, int block_n, uint8_t* xq,
                                       uint8_t* sfx, float* gx, void* stream) {
  return rmsnorm_quant_parts_impl(parts, nparts, plane, ldp, residual, ld_res, residual_out, ld_res_out, weight, y,
                                  ldy, rows, hidden, eps, gemma, dtype, terms, block_n, xq, sfx, gx, stream,
                                  PeerWait{nullptr, 0, 0, nullptr});
}

extern "C" int ada_rmsnorm_quant_peer(const void* inbox, int32_t nparts, int64_t plane, int64_t ldp,
                                      const void* residual, int64_t ld_res, void* residual_out, int64_t ld_res_out,
                                      const void* weight, void* y, int64_t ldy, int64_t rows, int32_t hidden,
                                      float eps, int gemma, int dtype, int terms, int block_n, uint8_t* xq,
                                      uint8_t* sfx, float* gx, const uint32_t* epoch, uint32_t tag_mul,
                                      uint32_t tag_add, uint32_t* err, void* stream) {
  if (!epoch || !inbox) return ADA_ERR_INVALID_ARG;
  if (((uintptr_t)epoch & 3) || ((uintptr_t)err & 3) || ((uintptr_t)inbox & 15) || (plane & 1) || (ldp & 1))
    return ADA_ERR_ALIGNMENT;
  return rmsnorm_quant_parts_impl(reinterpret_cast<const float*>(inbox), nparts, plane, ldp, residual, ld_res,
                                  residual_out, ld_res_out, weight, y, ldy, rows, hidden, eps, gemma, dtype, terms,
                                  block_n, xq, sfx, gx, stream, PeerWait{epoch, tag_mul, tag_add, err});
}
