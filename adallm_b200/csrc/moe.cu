// Mixture-of-experts routing around the grouped NVFP4 GEMM (sm_100a), restating
// Qwen3MoeSparseMoeBlock.forward (adallm/architectures/qwen3.py:1026-1032 and the weighted sum of
// the expert outputs that follows):
//   route:   w = softmax(router_logits) in fp32; (w, ids) = top-k of w; w /= sum(w) when
//            norm_topk_prob; w cast to the activation dtype.  One warp per token; the top-k is
//            k rounds of a warp argmax (ties: the lower expert index first).
//   combine: out[t] = sum_j w[t, j] * y[t * k + j] over the token's k expert rows, fp32 in
//            expert-slot order, rounded once to the activation dtype.
#include <algorithm>
#include <cfloat>
#include <type_traits>

#include "cluster.cuh"

namespace ada {
namespace moe {

constexpr int MAX_EXPERTS = 1024;  // 32 per lane
constexpr int MAX_TOPK = 32;

// Softmax, top-k and renormalisation of token t's router logits (logit(e) for e < experts), by
// one warp.  PER: experts per lane (experts <= 32 * PER).
template <typename T, int PER, typename Logit>
__device__ __forceinline__ void route_token(int t, int experts, int topk, int norm, Logit logit,
                                            int32_t* __restrict__ ids, T* __restrict__ weights) {
  const int lane = threadIdx.x & 31;
  float p[PER];
  float mx = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = i * 32 + lane;
    p[i] = e < experts ? logit(e) : -FLT_MAX;
    mx = fmaxf(mx, p[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = i * 32 + lane;
    p[i] = e < experts ? expf(p[i] - mx) : 0.f;
    sum += p[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  float sel_w[MAX_TOPK];
  int sel_e[MAX_TOPK];
  float wsum = 0.f;
  for (int j = 0; j < topk; ++j) {
    float best = -1.f;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      if (e < experts && (p[i] > best || (p[i] == best && e < be))) {
        best = p[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ob > best || (ob == best && oe < be)) {
        best = ob;
        be = oe;
      }
    }
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (i * 32 + lane == be) p[i] = -2.f;  // taken
    sel_w[j] = best / sum;
    sel_e[j] = be;
    wsum += sel_w[j];
  }
  if (lane == 0)
    for (int j = 0; j < topk; ++j) {
      ids[(int64_t)t * topk + j] = sel_e[j];
      weights[(int64_t)t * topk + j] = from_f32<T>(norm ? sel_w[j] / wsum : sel_w[j]);
    }
}

// One warp per token over router logits in memory.
template <typename T, int PER>
__global__ void __launch_bounds__(128) route_kernel(const T* __restrict__ logits, int64_t ld, int tokens, int experts,
                                                    int topk, int norm, int32_t* __restrict__ ids,
                                                    T* __restrict__ weights) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  route_token<T, PER>(t, experts, topk, norm, [&](int e) { return to_f32(logits[(int64_t)t * ld + e]); }, ids,
                      weights);
}

// The router GEMM fused with the routing: grid (ctas, tokens), cluster (ctas, 1, 1).  CTA r of
// token t's cluster computes the logits of experts [r * per, (r + 1) * per) -- one warp per expert
// at a time, lanes over the hidden dimension in 8-element steps, a fixed xor-shuffle reduction,
// rounded to the activation dtype as the reference's bf16 F.linear output -- and sends them into
// CTA 0's shared memory (st.async, counted by an mbarrier); CTA 0's first warp then routes.
constexpr int ROUTER_WARPS = 8;
template <typename T, int PER>
__global__ void __launch_bounds__(ROUTER_WARPS * 32) router_route_kernel(const T* __restrict__ x, int64_t ldx,
                                                                        const T* __restrict__ w, int64_t ldw,
                                                                        int hidden, int experts, int per, int topk,
                                                                        int norm, int32_t* __restrict__ ids,
                                                                        T* __restrict__ weights,
                                                                        unsigned int* err) {
  __shared__ float logits[MAX_EXPERTS];
  __shared__ unsigned long long bar;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cl::ctarank();
  if (rank == 0 && threadIdx.x == 0) {
    cl::exchange_init_bytes(&bar, (uint32_t)experts * 4u);
    cl::fence_exchange_init();
  }
  cl::cluster_arrive_relaxed();
  const int t = blockIdx.y;
  const int e0 = (int)rank * per, e1 = min(experts, e0 + per);
  const T* xr = x + (int64_t)t * ldx;
  pdl_wait();
  pdl_trigger();
  float acc[2] = {0.f, 0.f};  // two experts per warp step
  cl::cluster_wait();  // CTA 0's barrier is initialised: its shared memory may be written
  const uint32_t dst_bar = cl::mapa(&bar, 0);
  for (int e = e0 + 2 * warp; e < e1; e += 2 * ROUTER_WARPS) {
    const bool two = e + 1 < e1;
    acc[0] = acc[1] = 0.f;
    const T* w0p = w + (int64_t)e * ldw;
    const T* w1p = w + (int64_t)(two ? e + 1 : e) * ldw;
    constexpr int CH = 8;  // 8-element chunks per lane whose loads are in flight together
    for (int c0 = lane * 8; c0 < hidden; c0 += 256 * CH) {
      uint4 xa[CH], wa[CH], wb[CH];
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const int c = c0 + 256 * i;
        if (c < hidden) {
          xa[i] = *reinterpret_cast<const uint4*>(xr + c);
          wa[i] = *reinterpret_cast<const uint4*>(w0p + c);
          wb[i] = *reinterpret_cast<const uint4*>(w1p + c);
        }
      }
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        if (c0 + 256 * i >= hidden) break;
        float xv[8], f0[8], f1[8];
        unpack8<T>(xa[i], xv);
        unpack8<T>(wa[i], f0);
        unpack8<T>(wb[i], f1);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[0] = fmaf(xv[j], f0[j], acc[0]);
          acc[1] = fmaf(xv[j], f1[j], acc[1]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], o);
      acc[1] += __shfl_xor_sync(0xffffffffu, acc[1], o);
    }
    if (lane == 0) cl::st_async_f32(cl::mapa(&logits[e], 0), to_f32(from_f32<T>(acc[0])), dst_bar);
    if (lane == 1 && two) cl::st_async_f32(cl::mapa(&logits[e + 1], 0), to_f32(from_f32<T>(acc[1])), dst_bar);
  }
  if (rank != 0 || warp != 0) return;  // CTA 0 stays until every logit has arrived
  if (!cl::exchange_wait(&bar)) {
    if (lane == 0) atomicOr(err, 0x80u);  // a logit never arrived
    return;
  }
  route_token<T, PER>(t, experts, topk, norm, [&](int e) { return logits[e]; }, ids, weights);
}

// One CTA per token, 8 hidden elements per thread and step.
// With ids (expert parallelism): slots whose expert is outside [expert_base, expert_base +
// num_local) belong to another rank and are skipped (their expert rows were not computed here).
// OutT float keeps the rank's fp32 sum unrounded, so that an fp32 sum over the ranks rounds once,
// as the single-GPU combine does.
template <typename T, typename OutT>
__global__ void __launch_bounds__(256) combine_kernel(const T* __restrict__ y, int64_t ldy, const T* __restrict__ w,
                                                      int topk, int hidden, OutT* __restrict__ out, int64_t ldo,
                                                      const int32_t* __restrict__ ids, int expert_base, int num_local) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < hidden; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < topk; ++j) {
      if (ids) {
        const int e = __ldg(ids + (int64_t)t * topk + j) - expert_base;
        if (e < 0 || e >= num_local) continue;
      }
      const float wj = to_f32(w[(int64_t)t * topk + j]);
      float v[8];
      unpack8<T>(*reinterpret_cast<const uint4*>(y + ((int64_t)t * topk + j) * ldy + c), v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(wj, v[i], acc[i]);
    }
    if constexpr (std::is_same<OutT, float>::value) {
      float4* o = reinterpret_cast<float4*>(out + (int64_t)t * ldo + c);
      o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
      *reinterpret_cast<uint4*>(out + (int64_t)t * ldo + c) = pack8<T>(acc);
    }
  }
}

}  // namespace moe
}  // namespace ada

using namespace ada;

extern "C" int ada_moe_route_topk(const void* logits, int dtype, int64_t ld, int64_t tokens, int32_t experts,
                                  int32_t topk, int32_t norm_topk_prob, int32_t* ids, void* weights, void* stream) {
  if (tokens < 0 || experts <= 0 || topk <= 0 || ld < experts) return ADA_ERR_INVALID_ARG;
  if (tokens == 0) return ADA_OK;
  if (!logits || !ids || !weights) return ADA_ERR_INVALID_ARG;
  if (experts > moe::MAX_EXPERTS || topk > moe::MAX_TOPK || topk > experts) return ADA_ERR_UNSUPPORTED;
  if (tokens > (int64_t)65535 * 4) return ADA_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)cdiv(tokens, 4));
#define ADA_ROUTE(TT, PER_)                                                                                      \
  (void)launch_k(moe::route_kernel<TT, PER_>, grid, dim3(128), 0, st, (const TT*)logits, ld, (int)tokens,       \
                 (int)experts, (int)topk, (int)norm_topk_prob, ids, (TT*)weights)
#define ADA_ROUTE_PER(TT)                 \
  do {                                    \
    if (experts <= 64)                    \
      ADA_ROUTE(TT, 2);                   \
    else if (experts <= 128)              \
      ADA_ROUTE(TT, 4);                   \
    else if (experts <= 256)              \
      ADA_ROUTE(TT, 8);                   \
    else                                  \
      ADA_ROUTE(TT, moe::MAX_EXPERTS / 32); \
  } while (0)
  if (dtype == ADA_DT_BF16)
    ADA_ROUTE_PER(__nv_bfloat16);
  else if (dtype == ADA_DT_F16)
    ADA_ROUTE_PER(__half);
  else
    return ADA_ERR_INVALID_ARG;
#undef ADA_ROUTE_PER
#undef ADA_ROUTE
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

extern "C" int ada_moe_router_topk(const void* x, int dtype, int64_t ldx, int64_t tokens, const void* router_w,
                                   int64_t ldw, int32_t hidden, int32_t experts, int32_t topk,
                                   int32_t norm_topk_prob, int32_t* ids, void* weights, unsigned int* err,
                                   void* stream) {
  if (tokens < 0 || experts <= 0 || topk <= 0 || hidden <= 0 || ldx < hidden || ldw < hidden) return ADA_ERR_INVALID_ARG;
  if (tokens == 0) return ADA_OK;
  if (!x || !router_w || !ids || !weights || !err) return ADA_ERR_INVALID_ARG;
  if (experts > moe::MAX_EXPERTS || topk > moe::MAX_TOPK || topk > experts) return ADA_ERR_UNSUPPORTED;
  if (hidden % 8 || tokens > 65535) return ADA_ERR_UNSUPPORTED;
  if (((uintptr_t)x & 15) || ((uintptr_t)router_w & 15) || (ldx & 7) || (ldw & 7) || ((uintptr_t)err & 3))
    return ADA_ERR_ALIGNMENT;
  const int ctas = (int)std::min<int64_t>(cl::MAX_CLUSTER, cdiv(experts, 16));
  const int per = (int)cdiv(experts, ctas);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)ctas, (unsigned)tokens), block(moe::ROUTER_WARPS * 32);
  cudaError_t e_;
#define ADA_RR(TT, PER_)                                                                                          \
  e_ = launch_kc(moe::router_route_kernel<TT, PER_>, grid, block, 0, st, ctas, (const TT*)x, ldx,                \
                 (const TT*)router_w, ldw, (int)hidden, (int)experts, per, (int)topk, (int)norm_topk_prob, ids,  \
                 (TT*)weights, err)
#define ADA_RR_PER(TT)                       \
  do {                                       \
    if (experts <= 64)                       \
      ADA_RR(TT, 2);                         \
    else if (experts <= 128)                 \
      ADA_RR(TT, 4);                         \
    else if (experts <= 256)                 \
      ADA_RR(TT, 8);                         \
    else                                     \
      ADA_RR(TT, moe::MAX_EXPERTS / 32);     \
  } while (0)
  if (dtype == ADA_DT_BF16)
    ADA_RR_PER(__nv_bfloat16);
  else if (dtype == ADA_DT_F16)
    ADA_RR_PER(__half);
  else
    return ADA_ERR_INVALID_ARG;
#undef ADA_RR_PER
#undef ADA_RR
  return e_ == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

static int combine_impl(const void* y, int dtype, int64_t ldy, const void* weights, const int32_t* ids,
                        int32_t expert_base, int32_t num_local, int64_t tokens, int32_t topk, int32_t hidden,
                        void* out, int64_t ldo, void* stream, bool out_f32 = false) {
  if (tokens < 0 || topk <= 0 || hidden <= 0 || ldy < hidden || ldo < hidden) return ADA_ERR_INVALID_ARG;
  if (tokens == 0) return ADA_OK;
  if (!y || !weights || !out) return ADA_ERR_INVALID_ARG;
  if (hidden % 8 || tokens > 0x7fffffff) return ADA_ERR_UNSUPPORTED;
  if (((uintptr_t)y & 15) || ((uintptr_t)out & 15) || (ldy & 7) || (ldo & 7)) return ADA_ERR_ALIGNMENT;
  if (out_f32 && (ldo & 3)) return ADA_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)tokens);
  if (dtype == ADA_DT_BF16 && out_f32)
    (void)launch_k(moe::combine_kernel<__nv_bfloat16, float>, grid, dim3(256), 0, st, (const __nv_bfloat16*)y, ldy,
                   (const __nv_bfloat16*)weights, (int)topk, (int)hidden, (float*)out, ldo, ids, (int)expert_base,
                   (int)num_local);
  else if (dtype == ADA_DT_BF16)
    (void)launch_k(moe::combine_kernel<__nv_bfloat16, __nv_bfloat16>, grid, dim3(256), 0, st,
                   (const __nv_bfloat16*)y, ldy, (const __nv_bfloat16*)weights, (int)topk, (int)hidden,
                   (__nv_bfloat16*)out, ldo, ids, (int)expert_base, (int)num_local);
  else if (dtype == ADA_DT_F16 && out_f32)
    (void)launch_k(moe::combine_kernel<__half, float>, grid, dim3(256), 0, st, (const __half*)y, ldy,
                   (const __half*)weights, (int)topk, (int)hidden, (float*)out, ldo, ids, (int)expert_base,
                   (int)num_local);
  else if (dtype == ADA_DT_F16)
    (void)launch_k(moe::combine_kernel<__half, __half>, grid, dim3(256), 0, st, (const __half*)y, ldy,
                   (const __half*)weights, (int)topk, (int)hidden, (__half*)out, ldo, ids, (int)expert_base,
                   (int)num_local);
  else
    return ADA_ERR_INVALID_ARG;
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

extern "C" int ada_moe_combine(const void* y, int dtype, int64_t ldy, const void* weights, int64_t tokens,
                               int32_t topk, int32_t hidden, void* out, int64_t ldo, void* stream) {
  return combine_impl(y, dtype, ldy, weights, nullptr, 0, 0, tokens, topk, hidden, out, ldo, stream);
}

extern "C" int ada_moe_combine_ep(const void* y, int dtype, int64_t ldy, const void* weights,
                                  const int32_t* expert_ids, int32_t expert_base, int32_t num_local, int64_t tokens,
                                  int32_t topk, int32_t hidden, void* out, int64_t ldo, void* stream) {
  if (!expert_ids || expert_base < 0 || num_local <= 0) return ADA_ERR_INVALID_ARG;
  return combine_impl(y, dtype, ldy, weights, expert_ids, expert_base, num_local, tokens, topk, hidden, out, ldo,
                      stream);
}

extern "C" int ada_moe_combine_ep_f32(const void* y, int dtype, int64_t ldy, const void* weights,
                                      const int32_t* expert_ids, int32_t expert_base, int32_t num_local,
                                      int64_t tokens, int32_t topk, int32_t hidden, float* out, int64_t ldo,
                                      void* stream) {
  if (!expert_ids || expert_base < 0 || num_local <= 0) return ADA_ERR_INVALID_ARG;
  return combine_impl(y, dtype, ldy, weights, expert_ids, expert_base, num_local, tokens, topk, hidden, out, ldo,
                      stream, true);
}
