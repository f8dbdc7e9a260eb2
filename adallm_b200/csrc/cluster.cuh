// Thread-block-cluster helpers (sm_90+ PTX, used here on sm_100a): a row that is
// too short to keep one CTA busy for long is split over the CTAs of one cluster,
// which combine their partial reductions through distributed shared memory.
//
// Protocol of a cluster row kernel (every thread of every CTA runs all of it up to its
// last reduction; a padding CTA returns only after cluster_wait()):
//   cluster_start(xch, n)                  right after start: n exchanges, one per reduction
//   ... load the slice, local partial ...
//   cluster_wait()                         every CTA of the cluster is running: DSMEM is live
//   v = cluster_allreduce_x<Op>(v, red, &xch[i])   one per reduction
// A CTA is written by its peers only before its own wait on that exchange completes, so no
// CTA exits while a peer still writes into it.
#pragma once

#include <cstdlib>

#include "common.cuh"

namespace ada {
namespace cl {

constexpr int MAX_CLUSTER = 8;

__device__ __forceinline__ uint32_t ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync() {
  cluster_arrive();
  cluster_wait();
}

// Shared-memory address of `p` (a __shared__ object of this CTA) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa(const void* p, uint32_t rank) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p)), r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

struct OpMax {
  __device__ static float apply(float a, float b) { return fmaxf(a, b); }
};
struct OpSum {
  __device__ static float apply(float a, float b) { return __fadd_rn(a, b); }
};

constexpr int MAX_WARPS = 16;  // row kernels run <= 512 threads

// CTA-wide reduction (blockDim.x a multiple of 32, <= 32 * MAX_WARPS; `red` holds MAX_WARPS
// floats), warps combined in order.
template <typename Op>
__device__ __forceinline__ float block_reduce(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = Op::apply(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) r = Op::apply(r, red[i]);
  return r;
}

// ---- cross-CTA reduction: asynchronous DSMEM stores counted by mbarriers -----------------
// Thread r of each CTA sends the CTA's partial into its slot of CTA r with st.async, which
// completes 4 bytes of transaction on CTA r's mbarrier; every thread then waits on its own
// CTA's barrier until all n partials have landed (acquire at cluster scope).  Each barrier is
// initialised with one arrival that is made at once with the expected n * 4 bytes, before the
// cluster's start barrier, and completes exactly one phase: every exchange serves one
// reduction.  Unlike barrier.cluster it waits for the partials only, not for every thread of
// every CTA, and each partial is one one-way transaction.
struct Exchange {
  float slots[MAX_CLUSTER];
  unsigned long long bar;
};
// One arrival (made here) plus `bytes` of transactions complete the barrier's first phase.
__device__ __forceinline__ void exchange_init_bytes(unsigned long long* bar, uint32_t bytes) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(bar);
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(a) : "memory");
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void exchange_init(Exchange* x) { exchange_init_bytes(&x->bar, nctarank() * 4u); }
__device__ __forceinline__ void fence_exchange_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void st_async_f32(uint32_t cluster_addr, float v, uint32_t cluster_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(cluster_addr), "f"(v),
               "r"(cluster_bar)
               : "memory");
}
// 16 bytes into another CTA's shared memory, completing 16 bytes of transaction on its barrier
// (both addresses 16-byte aligned).
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, float a, float b, float c, float d,
                                            uint32_t cluster_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   cluster_addr),
               "f"(a), "f"(b), "f"(c), "f"(d), "r"(cluster_bar)
               : "memory");
}
// Bounded wait (about 2 s) for phase 0 of an exchange barrier; false when it gave up.
__device__ __forceinline__ bool exchange_wait(unsigned long long* bar) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(bar);
  uint64_t t0 = 0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a)
        : "memory");
    if (ok) return true;
    if ((it & 63u) == 63u) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > 2000000000ull || it > (1u << 30)) return false;
    }
  }
}

// Two reductions in one exchange: each CTA sends (a, b) as one 8-byte transaction.
struct Exchange2 {
  float2 slots[MAX_CLUSTER];
  unsigned long long bar;
};
__device__ __forceinline__ void exchange2_init(Exchange2* x) { exchange_init_bytes(&x->bar, nctarank() * 8u); }
__device__ __forceinline__ void st_async_v2(uint32_t cluster_addr, float a, float b, uint32_t cluster_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
                   cluster_addr),
               "f"(a), "f"(b), "r"(cluster_bar)
               : "memory");
}

// Start of a cluster row kernel: initialise its `count` exchanges, then arrive on the
// cluster's start barrier (the matching cluster_wait() makes the initialisation visible).
__device__ __forceinline__ void cluster_start(Exchange* xs, int count) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < count; ++i) exchange_init(&xs[i]);
    fence_exchange_init();
  }
  cluster_arrive_relaxed();
}

// Cluster-wide reduction through an Exchange: CTA partials combined in rank order
// (deterministic for sums).
template <typename Op>
__device__ __forceinline__ float cluster_allreduce_x(float v, float* red, Exchange* x) {
  v = block_reduce<Op>(v, red);
  const uint32_t n = nctarank();
  if (n == 1) return v;
  if (threadIdx.x < n) st_async_f32(mapa(&x->slots[ctarank()], threadIdx.x), v, mapa(&x->bar, threadIdx.x));
  exchange_wait(&x->bar);
  float r = x->slots[0];
  for (uint32_t i = 1; i < n; ++i) r = Op::apply(r, x->slots[i]);
  return r;
}

// Cluster-wide reduction of two values at once (OpA on a, OpB on b; `red` holds 2 * MAX_WARPS
// floats): one exchange, CTA partials combined in rank order for each.
template <typename OpA, typename OpB>
__device__ __forceinline__ float2 cluster_allreduce2_x(float a, float b, float* red, Exchange2* x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a = OpA::apply(a, __shfl_xor_sync(0xffffffffu, a, o));
    b = OpB::apply(b, __shfl_xor_sync(0xffffffffu, b, o));
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    red[w] = a;
    red[MAX_WARPS + w] = b;
  }
  __syncthreads();
  float ra = red[0], rb = red[MAX_WARPS];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) {
    ra = OpA::apply(ra, red[i]);
    rb = OpB::apply(rb, red[MAX_WARPS + i]);
  }
  const uint32_t n = nctarank();
  if (n == 1) return make_float2(ra, rb);
  if (threadIdx.x < n) st_async_v2(mapa(&x->slots[ctarank()], threadIdx.x), ra, rb, mapa(&x->bar, threadIdx.x));
  exchange_wait(&x->bar);
  float2 r = x->slots[0];
  for (uint32_t i = 1; i < n; ++i) {
    r.x = OpA::apply(r.x, x->slots[i].x);
    r.y = OpB::apply(r.y, x->slots[i].y);
  }
  return r;
}

// How a row of `units` 16-element blocks is spread over a cluster: `ctas` CTAs, each
// owning a contiguous slice of blocks, of `threads` threads that each own up to `maxu`
// octets (8 consecutive elements; the two octets of a block sit in adjacent lanes).
// Depends on the row length only, so every kernel reducing rows of one length rounds alike.
struct RowSplit {
  int ctas, threads, maxu;
};
// Largest cluster a row is spread over: 8, or ADALLM_B200_ROW_CLUSTER (1..8; a tuning knob read
// once per process -- every kernel of the process then rounds its rows alike).
inline int row_cluster_cap() {
  static int cap = [] {
    const char* e = std::getenv("ADALLM_B200_ROW_CLUSTER");
    const int v = e ? std::atoi(e) : MAX_CLUSTER;
    return v >= 1 && v <= MAX_CLUSTER ? v : MAX_CLUSTER;
  }();
  return cap;
}
inline RowSplit row_split(int units) {
  RowSplit s;
  const int cap = row_cluster_cap();
  s.ctas = units / 32;
  s.ctas = s.ctas < 1 ? 1 : s.ctas > cap ? cap : s.ctas;
  const int octets = 2 * ((units + s.ctas - 1) / s.ctas);
  s.threads = ((octets + 31) / 32) * 32;
  if (s.threads > 512) s.threads = 512;
  const int mu = (octets + s.threads - 1) / s.threads;
  s.maxu = mu <= 1 ? 1 : mu <= 2 ? 2 : mu <= 4 ? 4 : mu <= 8 ? 8 : 0;  // 0: row too long
  return s;
}
// First octet of CTA `rank`'s slice (slices are whole 16-element blocks).
__host__ __device__ __forceinline__ int slice_octet(int units, int rank, int ctas) {
  return 2 * (int)(((int64_t)units * rank) / ctas);
}

}  // namespace cl
}  // namespace ada
