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

// Host-side check of a partial-plane descriptor covering rows x cols (16-byte float4 reads).
inline bool parts_ok(const PartIn& pi, int64_t rows, int64_t cols) {
  if (!pi.p || pi.n < 1 || pi.n > 64 || pi.ld < cols || pi.plane < rows * pi.ld) return false;
  return ((uintptr_t)pi.p & 15) == 0 && (pi.ld & 3) == 0 && (pi.plane & 3) == 0;
}

}  // namespace ada
