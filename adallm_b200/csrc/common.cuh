// Shared helpers for the adallm_b200 sm_100a kernels: status codes, dtype
// conversion, and thin wrappers over the PTX instructions used by the
// kernels (ld.global.nc, cvt to/from fp8 / fp4, mma.sync, ex2).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <atomic>
#include <mutex>
#include <utility>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/adallm_b200.h"

#define ADA_CHECK_LAUNCH()                                   \
  do {                                                       \
    cudaError_t _e = cudaGetLastError();                     \
    if (_e != cudaSuccess) return ADA_ERR_LAUNCH;            \
  } while (0)

namespace ada {

// ---- programmatic dependent launch -------------------------------------------
// Every kernel of this library is launched with programmatic stream serialization
// (unless disabled with ada_set_pdl(0)): it may start while the previous kernel on the
// stream is still running, and waits in pdl_wait() until that kernel has completed and
// its writes are visible.  Each kernel calls pdl_wait() before touching data another
// kernel produced (and every CTA calls it before exiting, so completion is transitive
// along the stream), then pdl_trigger() to let its own successor get resident early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool g_pdl_enabled = true;

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl_enabled ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Same, with thread-block clusters of `cluster_x` CTAs along x (grid.x a multiple of it).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kc(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl_enabled ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---- scalar conversions ----------------------------------------------------
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// 8 x 16-bit values <-> 8 floats
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f32(h[i]);
}
template <typename T>
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  T* h = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = from_f32<T>(f[i]);
  return u;
}

// ---- loads -------------------------------------------------------------------
// Streaming 16-byte load through the non-coherent path, not kept in L1.
__device__ __forceinline__ uint4 ldg_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---- fp8 / fp4 conversions (PTX cvt, sm_89+ / sm_100a) ---------------------
// Two e4m3 bytes (low byte = first element) -> f16x2 (low half = first element).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}
// Two floats -> two e4m3 bytes, round-to-nearest-even, saturating.  lo lands in
// the low byte (first element in memory).
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// Eight floats -> eight e2m1 nibbles (4 bytes), round-to-nearest-even,
// saturating.  Element 0 lands in the low nibble of byte 0 (even K index in
// the low nibble: the reference packing order).
__device__ __forceinline__ uint32_t f32x8_to_e2m1x8(const float* v) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return r;
}

// Eight e2m1 nibbles (element 0 in the low nibble) -> their exact values as four f16x2
// (low half = even element).  Integer-only: one byte permute per pair picks the f16 high
// byte of each magnitude {0, .5, 1, 1.5, 2, 3, 4, 6} = {00, 38, 3C, 3E, 40, 42, 44, 46}
// (low bytes are zero, and table entry 0 supplies the zero low bytes), then the sign bits
// are moved into place.
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t codes, uint32_t* h) {
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t c = codes >> (8 * p);
    const uint32_t sel = ((c & 0x7u) << 4) | ((c & 0x70u) << 8);
    const uint32_t sign = ((c & 0x8u) << 12) | ((c & 0x80u) << 24);
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(0x3E3C3800u), "r"(0x46444240u), "r"(sel));
    h[p] = r | sign;
  }
}

// 2^x via the SFU (ex2.approx); -inf -> 0.
__device__ __forceinline__ float fast_exp2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// ---- warp-level MMA (used by the memory-bound attention kernel) -------------
// D(16x8,f32) += A(16x16,f16,row) * B(16x8,f16,col)
__device__ __forceinline__ void mma_16816_f16(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace ada
