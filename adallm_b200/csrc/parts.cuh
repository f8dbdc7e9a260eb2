// Split-K partial planes as a kernel input.  A GEMM run in partial mode
// (ada_nvfp4_gemm_partials) leaves its output as `n` fp32 planes, one per K split; the kernel
// that consumes the output sums them in plane order and rounds to the activation dtype, which
// is bit-identical to the GEMM reducing the same split itself and storing bf16/fp16.
#pragma once

#include "common.cuh"

namespace ada {

struct PartIn {
  const float* p;  // plane 0
  int n;           // planes (0: the input is a plain bf16/fp16 tensor instead)
  int64_t plane;   // floats between planes
  int64_t ld;      // floats between rows
};

// The MoE block's weighted combine as an input: element (t, c) is sum_j w[t][j] * y[t * topk + j][c]
// (fp32 fma in slot order from 0, as the combine kernel accumulates), rounded to T.
struct SlotIn {
  const void* y;  // [tokens * topk, ldy] expert rows (T); null: not this input mode
  int64_t ldy;
  const void* w;  // [tokens, topk] routing weights (T)
  int topk;
};

template <typename T, int N>
__device__ __forceinline__ void load_slots(const SlotIn& si, int64_t row, int64_t col, float* f) {
  static_assert(N == 8, "one 16-byte vector of T");
  const T* y = reinterpret_cast<const T*>(si.y);
  const T* w = reinterpret_cast<const T*>(si.w);
  float acc[N];
#pragma unroll
  for (int i = 0; i < N; ++i) acc[i] = 0.f;
  for (int j = 0; j < si.topk; ++j) {
    const float wj = to_f32(w[row * si.topk + j]);
    float v[N];
    unpack8<T>(*reinterpret_cast<const uint4*>(y + (row * si.topk + j) * si.ldy + col), v);
#pragma unroll
    for (int i = 0; i < N; ++i) acc[i] = fmaf(wj, v[i], acc[i]);
  }
#pragma unroll
  for (int i = 0; i < N; ++i) f[i] = to_f32(from_f32<T>(acc[i]));
}

// Elements [col, col + N) of row `row`: sum of the planes (plane order), rounded to T.
template <typename T, int N>
__device__ __forceinline__ void load_parts(const PartIn& pi, int64_t row, int64_t col, float* f) {
  static_assert(N % 4 == 0, "whole float4s");
  constexpr int G = 8;
  const float* base = pi.p + row * pi.ld + col;
  for (int k = 0; k < pi.n; k += G) {  // G planes' loads in flight together, summed in plane order
    float4 a[G][N / 4];
#pragma unroll
    for (int j = 0; j < G; ++j)
      if (k + j < pi.n)
#pragma unroll
        for (int i = 0; i < N / 4; ++i)
          a[j][i] = *reinterpret_cast<const float4*>(base + (int64_t)(k + j) * pi.plane + 4 * i);
#pragma unroll
    for (int j = 0; j < G; ++j) {
      if (k + j >= pi.n) break;
#pragma unroll
      for (int i = 0; i < N / 4; ++i) {
        if (k + j == 0) {
          f[4 * i] = a[j][i].x;
          f[4 * i + 1] = a[j][i].y;
          f[4 * i + 2] = a[j][i].z;
          f[4 * i + 3] = a[j][i].w;
        } else {
          f[4 * i] = __fadd_rn(f[4 * i], a[j][i].x);
          f[4 * i + 1] = __fadd_rn(f[4 * i + 1], a[j][i].y);
          f[4 * i + 2] = __fadd_rn(f[4 * i + 2], a[j][i].z);
          f[4 * i + 3] = __fadd_rn(f[4 * i + 3], a[j][i].w);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) f[i] = to_f32(from_f32<T>(f[i]));
}

// Tensor parallelism over peer memory: the planes of every rank arrive in this rank's inbox
// from the peers' GEMM epilogues as 8-byte words (fp32 value bits | 32-bit tag << 32), each
// written by one single-copy-atomic 8-byte store.  A word belongs to the current step and
// projection when its tag equals epoch * tag_mul + tag_add (epoch: steps completed on this
// rank, ada_tp_epoch_advance), so the consumer needs no fence and no counter: it polls the
// words it reads until their tags are current (bounded: ~2 s, then ERR_PEER_WAIT and the
// stale values are used).  epoch == null: the planes are plain local fp32.
struct PeerWait {
  const unsigned int* epoch;
  unsigned int tag_mul, tag_add;
  unsigned int* err;
};
constexpr unsigned int ERR_PEER_WAIT = 0x50;

__device__ __forceinline__ unsigned int peer_tag(const PeerWait& pw) { return *pw.epoch * pw.tag_mul + pw.tag_add; }

__device__ __forceinline__ void ld_tagged2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// load_parts over tagged planes: elements [col, col + N) of row `row`, the sum of pi.n planes
// in plane order (pi.plane / pi.ld in 8-byte words), rounded to T.
template <typename T, int N>
__device__ __forceinline__ void load_parts_tagged(const PartIn& pi, int64_t row, int64_t col, const PeerWait& pw,
                                                  unsigned int tag, float* f) {
  static_assert(N % 2 == 0, "whole word pairs");
  const unsigned long long* base = reinterpret_cast<const unsigned long long*>(pi.p) + row * pi.ld + col;
  constexpr int G = 4;  // planes whose words are in flight together
  uint64_t t0 = 0;
  bool late = false, timed = false;
  for (int k0 = 0; k0 < pi.n; k0 += G) {
    unsigned long long w[G][N];
#pragma unroll
    for (int j = 0; j < G; ++j)
      if (k0 + j < pi.n)
#pragma unroll
        for (int i = 0; i < N; i += 2) ld_tagged2(base + (int64_t)(k0 + j) * pi.plane + i, w[j][i], w[j][i + 1]);
#pragma unroll
    for (int j = 0; j < G; ++j) {
      if (k0 + j >= pi.n) break;
      const unsigned long long* pk = base + (int64_t)(k0 + j) * pi.plane;
      for (uint32_t it = 0;; ++it) {  // re-poll until this plane's words carry the tag
        bool ok = true;
#pragma unroll
        for (int i = 0; i < N; ++i) ok = ok && (unsigned int)(w[j][i] >> 32) == tag;
        if (ok || late) break;
        if (!timed) {
          asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
          timed = true;
        }
        if ((it & 15u) == 15u) {
          uint64_t t;
          asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
          if (t - t0 > 2000000000ull) {
            late = true;
            if (pw.err) atomicOr(pw.err, ERR_PEER_WAIT);
          }
        }
#pragma unroll
        for (int i = 0; i < N; i += 2) ld_tagged2(pk + i, w[j][i], w[j][i + 1]);
      }
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const float v = __uint_as_float((unsigned int)(w[j][i] & 0xffffffffull));
        f[i] = k0 + j == 0 ? v : __fadd_rn(f[i], v);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) f[i] = to_f32(from_f32<T>(f[i]));
}

// Host-side check of a partial-plane descriptor covering rows x cols (16-byte float4 reads).
inline bool parts_ok(const PartIn& pi, int64_t rows, int64_t cols) {
  if (!pi.p || pi.n < 1 || pi.n > 64 || pi.ld < cols || pi.plane < rows * pi.ld) return false;
  return ((uintptr_t)pi.p & 15) == 0 && (pi.ld & 3) == 0 && (pi.plane & 3) == 0;
}

}  // namespace ada
