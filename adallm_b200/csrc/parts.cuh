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

// Elements [col, col + N) of row `row`: sum of the planes (plane order), rounded to T.
template <typename T, int N>
__device__ __forceinline__ void load_parts(const PartIn& pi, int64_t row, int64_t col, float* f) {
  static_assert(N % 4 == 0, "whole float4s");
  const float* base = pi.p + row * pi.ld + col;
#pragma unroll
  for (int i = 0; i < N; i += 4) {
    const float4 a = *reinterpret_cast<const float4*>(base + i);
    f[i] = a.x;
    f[i + 1] = a.y;
    f[i + 2] = a.z;
    f[i + 3] = a.w;
  }
  for (int k = 1; k < pi.n; ++k) {
    const float* b = base + (int64_t)k * pi.plane;
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 a = *reinterpret_cast<const float4*>(b + i);
      f[i] = __fadd_rn(f[i], a.x);
      f[i + 1] = __fadd_rn(f[i + 1], a.y);
      f[i + 2] = __fadd_rn(f[i + 2], a.z);
      f[i + 3] = __fadd_rn(f[i + 3], a.w);
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
