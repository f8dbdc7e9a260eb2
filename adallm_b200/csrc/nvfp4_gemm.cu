// NVFP4 linear for B200: y = x . dequant(W)^T on the 5th-generation tensor cores.
//
// Replaces nvfp4_linear / nvfp4_gemm_kernel (reference adallm/ops/nvfp4_gemm.py:58-136,
// :460-564).  The reference widens e2m1 weights to fp16 with a lookup table and a
// per-element scale gather inside the K loop; here the packed weights stay packed:
//
//   * W [N, K/2] e2m1 bytes (even K in the low nibble) is TMA-loaded as-is into
//     128-byte-swizzled shared memory; its e4m3 per-16 scales are re-laid out
//     once at load ("prepack") into the block-scaled MMA scale-factor layout.
//   * The bf16 activation row is quantised by a prologue kernel into T NVFP4
//     terms that share one fp32 per-row scale: term t quantises the residual
//     left by terms < t (T = 3 keeps the result within ~1e-3 of the fp32
//     dequantise-then-matmul oracle; T = 1 is plain W4A4).
//   * tcgen05.mma.kind::mxf4nvf4.block_scale.block16 with M = 128 weight rows
//     ("swap AB": tokens are the MMA N dimension), fp32 accumulation in TMEM;
//     the T terms are T MMAs into the same accumulator.
//   * Split-K over CTAs with a deterministic reduction: every split writes its
//     scaled fp32 partial, the last CTA of a tile sums the splits in order,
//     adds the bias and writes bf16/fp16.
//
// Warp roles (128 threads): warp 0 lane 0 issues TMA / bulk copies, warp 1
// lane 0 issues tcgen05.cp (scales -> TMEM) and MMAs, warp 1 owns the TMEM
// allocation, and all four warps run the epilogue (warp w reads TMEM lanes
// 32w..32w+31).  Every mbarrier wait is bounded (2 s); a timeout sets an error
// bit in the workspace and the CTA drains and exits.
#include "quant.cuh"
#include "sm100.cuh"

namespace ada {
namespace fp4 {

using namespace sm100;

constexpr int BM = 128;            // weight rows per tile (MMA M)
constexpr int KT = 256;            // K elements per pipeline stage (4 MMA k-blocks of 64)
constexpr int KT_BYTES = KT / 2;   // 128 bytes of packed e2m1 per row and stage
constexpr int SF_BLOCK = 512;      // scale bytes per 128 rows x 64 K
constexpr int MAX_STAGES = 8;

struct GemmParams {
  const uint8_t* sfw;  // [N/128][K/64][512]
  const uint8_t* sfx;  // [T][m_tiles][K/64][512]
  const float* gx;     // [m_pad] per-row activation scale
  const float* gw;     // weight_scale_2 (device scalar)
  const void* bias;    // [N] (out dtype) or null
  void* y;             // [M, ldy] out dtype
  float* partial;      // [ksplit][m_pad][N] fp32 (ksplit > 1)
  int* counters;       // [n_tiles * m_tiles]
  unsigned int* err;
  int M, N, K, ldy, m_pad, n_tiles, m_tiles, ksplit, stages, tmem_cols, out_dtype;
};

// The T activation terms of a token tile are stacked along the MMA N dimension:
// B operand rows [t*BN, (t+1)*BN) hold term t, so one MMA per 64-wide K block covers
// every term (NB = T*BN <= 128 rows, one scale-factor block).
template <int BN, int T>
struct Cfg {
  static constexpr int NB = BN * T;
  static_assert(NB % 16 == 0 && NB <= 128, "stacked terms must fit one 128-row scale block");
  static constexpr uint32_t A_BYTES = BM * KT_BYTES;      // 16 KiB
  static constexpr uint32_t B_BYTES = NB * KT_BYTES;      // all terms
  static constexpr uint32_t SFA_BYTES = 4 * SF_BLOCK;     // 2 KiB
  static constexpr uint32_t SFB_BYTES = 4 * SF_BLOCK;     // 2 KiB
  static constexpr uint32_t STAGE = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
  static constexpr uint32_t SF_COLS = 32;                 // TMEM columns of scales per stage
  static constexpr uint32_t CTRL = 256;
  static size_t smem_bytes(int stages) { return 1024 + (size_t)stages * STAGE + CTRL; }
  static uint32_t tmem_need(int stages) { return NB + stages * SF_COLS; }
};

__device__ __forceinline__ void store_out(void* y, int dtype, int64_t idx, float v) {
  if (dtype == ADA_DT_BF16)
    reinterpret_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<__half*>(y)[idx] = __float2half_rn(v);
}
__device__ __forceinline__ float load_bias(const void* b, int dtype, int n) {
  if (!b) return 0.f;
  return dtype == ADA_DT_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(b)[n])
                              : __half2float(reinterpret_cast<const __half*>(b)[n]);
}

template <int BN, int T>
__global__ void __launch_bounds__(128, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx, const GemmParams p) {
  // dependency wait placed inside (weights are prefetched before it)

  using C = Cfg<BN, T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)stages * C::STAGE);
  uint64_t* empty = full + MAX_STAGES;
  uint64_t* accf = empty + MAX_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* last_flag = abort_flag + 1;
  volatile int* abort_v = abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int n_tile = tile % p.n_tiles, m_tile = tile / p.n_tiles;
  const int split = blockIdx.y;
  const int kb64 = p.K / 64;
  const int nkt = p.K / KT;
  const int kt0 = (int)((int64_t)split * nkt / p.ksplit);
  const int kt1 = (int)((int64_t)(split + 1) * nkt / p.ksplit);
  const int nk = kt1 - kt0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, p.tmem_cols);
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmw);
    prefetch_tmap(&tmx);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: TMA tiles + bulk scale copies ----------------
      // The weights and their scales never depend on the previous kernel: the first
      // `stages` weight tiles are requested before the programmatic-launch dependency
      // wait, so they stream in while the producer of the activations finishes.
      const int pre = nk < stages ? nk : stages;
      for (int i = 0; i < pre; ++i) {
        uint8_t* st = smem + (size_t)i * C::STAGE;
        const int kt = kt0 + i;
        mbar_expect_tx(&full[i], C::A_BYTES + C::SFA_BYTES);
        tma_load_2d(st, &tmw, &full[i], kt * KT_BYTES, n_tile * BM);
        bulk_load(st + C::A_BYTES + C::B_BYTES, p.sfw + ((size_t)n_tile * kb64 + (size_t)kt * 4) * SF_BLOCK,
                  C::SFA_BYTES, &full[i]);
      }
      pdl_wait();
      for (int i = 0; i < nk; ++i) {
        const int s = i % stages;
        uint8_t* st = smem + (size_t)s * C::STAGE;
        const int kt = kt0 + i;
        if (i >= stages) {
          if (!mbar_wait_bounded(&empty[s], ((i / stages) & 1) ^ 1, abort_v, p.err, 1u)) break;
          mbar_expect_tx(&full[s], C::A_BYTES + C::SFA_BYTES);
          tma_load_2d(st, &tmw, &full[s], kt * KT_BYTES, n_tile * BM);
          bulk_load(st + C::A_BYTES + C::B_BYTES, p.sfw + ((size_t)n_tile * kb64 + (size_t)kt * 4) * SF_BLOCK,
                    C::SFA_BYTES, &full[s]);
        }
        mbar_arrive_expect_tx(&full[s], C::B_BYTES + C::SFB_BYTES);
        tma_load_2d(st + C::A_BYTES, &tmx, &full[s], kt * KT_BYTES, m_tile * C::NB);
        bulk_load(st + C::A_BYTES + C::B_BYTES + C::SFA_BYTES,
                  p.sfx + ((size_t)m_tile * kb64 + (size_t)kt * 4) * SF_BLOCK, C::SFB_BYTES, &full[s]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_mxf4nvf4(C::NB);
      for (int i = 0; i < nk; ++i) {
        const int s = i % stages;
        if (!mbar_wait_bounded(&full[s], (i / stages) & 1, abort_v, p.err, 2u)) break;
        tc_fence_after();
        uint8_t* st = smem + (size_t)s * C::STAGE;
        const uint32_t a_addr = smem_u32(st);
        const uint32_t b_addr = a_addr + C::A_BYTES;
        const uint32_t sfa_addr = b_addr + C::B_BYTES;
        const uint32_t sfb_addr = sfa_addr + C::SFA_BYTES;
        const uint32_t sf_col = tmem + C::NB + s * C::SF_COLS;
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          tmem_cp_32x128b_x4(sf_col + 4 * kb, desc_sf(sfa_addr + kb * SF_BLOCK));
          tmem_cp_32x128b_x4(sf_col + 16 + 4 * kb, desc_sf(sfb_addr + kb * SF_BLOCK));
        }
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
          mma_mxf4nvf4(tmem, desc_kmajor_sw128(a_addr + kb * 32), desc_kmajor_sw128(b_addr + kb * 32), idesc,
                       (i | kb) != 0, sf_col + 4 * kb, sf_col + 16 + 4 * kb);
        tc_commit(&empty[s]);  // stage reusable once these MMAs have read it
      }
      tc_commit(accf);  // accumulator complete (also issued after an abort, to drain)
    }
    __syncwarp();
  }

  // ---------------- epilogue: all 4 warps ----------------
  pdl_wait();     // activations / scales / workspace of earlier kernels are visible from here on
  pdl_trigger();  // the next kernel may get resident while this one drains
  const bool ok = mbar_wait_bounded(accf, 0, abort_v, p.err, 4u) && !*abort_v;
  tc_fence_after();
  __syncwarp();
  const int n = n_tile * BM + warp * 32 + lane;  // accumulator lane -> output column
  const float gw = __ldg(p.gw);
  const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
  // accumulator column t*BN + j holds term t of token m_tile*BN + j: sum the terms in order
  float out[BN];
#pragma unroll
  for (int j = 0; j < BN; ++j) out[j] = 0.f;
#pragma unroll
  for (int c = 0; c < C::NB; c += 16) {
    float v[16];
    tmem_ld16(lane_addr + c, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) out[(c % BN) + i] += v[i];
  }
  if (p.ksplit == 1) {
    if (ok) {
      const float b = load_bias(p.bias, p.out_dtype, n);
#pragma unroll
      for (int j = 0; j < BN; ++j) {
        const int m = m_tile * BN + j;
        if (m < p.M) store_out(p.y, p.out_dtype, (int64_t)m * p.ldy + n, out[j] * (gw * __ldg(p.gx + m)) + b);
      }
    }
  } else {
    float* part = p.partial + (size_t)split * p.m_pad * p.N;
    if (ok) {
#pragma unroll
      for (int j = 0; j < BN; ++j) {
        const int m = m_tile * BN + j;
        part[(size_t)m * p.N + n] = out[j] * (gw * __ldg(p.gx + m));
      }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0 && !*abort_v) *last_flag = (atomicAdd(&p.counters[tile], 1) == p.ksplit - 1);
    __syncthreads();
    if (*last_flag) {
      __threadfence();
      const float b = load_bias(p.bias, p.out_dtype, n);
      // splits summed in order (deterministic); each pass issues 16 independent L2 loads
#pragma unroll
      for (int j0 = 0; j0 < BN; j0 += 16) {
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.f;
        const float* col = p.partial + (size_t)(m_tile * BN + j0) * p.N + n;
        for (int s = 0; s < p.ksplit; ++s) {
          const float* ps = col + (size_t)s * p.m_pad * p.N;
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] += __ldcg(ps + (size_t)j * p.N);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m_tile * BN + j0 + j;
          if (m < p.M) store_out(p.y, p.out_dtype, (int64_t)m * p.ldy + n, acc[j] + b);
        }
      }
      if (threadIdx.x == 0) p.counters[tile] = 0;  // leave the workspace ready for the next call
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, p.tmem_cols);
}

// ---------------------------------------------------------------------------
// Activation quantiser (layout and arithmetic: quant.cuh).  One CTA per (padded) row.
template <typename TI>
__global__ void __launch_bounds__(256) act_quant_kernel(const TI* __restrict__ x, int64_t ldx, int M, int K, int terms,
                                                        int bn, int m_tiles, int m_pad, uint8_t* __restrict__ xq,
                                                        uint8_t* __restrict__ sfx, float* __restrict__ gx) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8];
  const int m = blockIdx.x;
  const int nblk = K >> 4;
  const q::QuantDst dst{xq, sfx, gx, terms, bn, K};
  if (m >= M) {
    for (int blk = threadIdx.x; blk < nblk; blk += blockDim.x) q::zero_block16(dst, m, blk);
    if (threadIdx.x == 0) gx[m] = 1.f;
    return;
  }
  const TI* xr = x + (int64_t)m * ldx;
  float amax = 0.f;
  for (int blk = threadIdx.x; blk < nblk; blk += blockDim.x) {
    float f[16];
    unpack8<TI>(*reinterpret_cast<const uint4*>(xr + blk * 16), f);
    unpack8<TI>(*reinterpret_cast<const uint4*>(xr + blk * 16 + 8), f + 8);
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(f[i]));
  }
  amax = q::block_max(amax, red);
  const float g = q::row_scale(amax);
  const float g6 = __fmul_rn(g, 6.f);
  if (threadIdx.x == 0) gx[m] = g;
  for (int blk = threadIdx.x; blk < nblk; blk += blockDim.x) {
    float r[16];
    unpack8<TI>(*reinterpret_cast<const uint4*>(xr + blk * 16), r);
    unpack8<TI>(*reinterpret_cast<const uint4*>(xr + blk * 16 + 8), r + 8);
    q::quant_block16(dst, m, blk, r, g, g6);
  }
}

// Scale prepack: [N, K/16] (fp16 holding e4m3 values, or raw e4m3 bytes) ->
// [N/128][K/64][512] bytes in the MMA scale-factor layout.
__global__ void __launch_bounds__(128) prepack_kernel(const void* __restrict__ scale, int is_fp16, int64_t ld, int N,
                                                      int K, uint8_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();

  const int kb64 = K >> 6;
  const int nb = blockIdx.x / kb64, kb = blockIdx.x - nb * kb64;
  const int r = threadIdx.x;
  const int n = nb * 128 + r;
  uint32_t packed = 0;
  if (n < N) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t idx = (int64_t)n * ld + kb * 4 + j;
      uint32_t b;
      if (is_fp16) {
        const float f = __half2float(reinterpret_cast<const __half*>(scale)[idx]);
        b = f32x2_to_e4m3x2(f, 0.f) & 0xFFu;  // exact: the values are e4m3-representable
      } else {
        b = reinterpret_cast<const uint8_t*>(scale)[idx];
      }
      packed |= b << (8 * j);
    }
  }
  *reinterpret_cast<uint32_t*>(out + ((size_t)nb * kb64 + kb) * 512 + (r & 31) * 16 + (r >> 5) * 4) = packed;
}

// ---------------------------------------------------------------------------
// Host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D byte matrix [rows, inner_bytes] with row stride `stride` bytes; box = 128 bytes x box_rows, 128B swizzle.
static bool make_map(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows, uint64_t stride,
                     uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner_bytes, rows};
  cuuint64_t strides[1] = {stride};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Token tile: the smallest of 16/32/64/128 covering m, capped so terms*bn <= 128.
static inline int block_n_for(int64_t m, int terms) {
  const int cap = terms == 1 ? 128 : terms == 2 ? 64 : 32;
  int bn = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : 128;
  return bn < cap ? bn : cap;
}

struct Plan {
  int terms, bn, m_tiles, m_pad, n_tiles, nkt, ksplit, stages, tmem_cols;
  size_t smem;
  // workspace layout (bytes, 256-aligned)
  size_t off_ctl, off_xq, off_sfx, off_gx, off_part, total;
};

static inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }
static inline uint32_t pow2_cols(uint32_t c) {
  uint32_t r = 32;
  while (r < c) r <<= 1;
  return r;
}

template <int BN, int T>
static void stages_for(int& stages, uint32_t& cols, size_t& smem) {
  using C = Cfg<BN, T>;
  // two CTAs per SM: <= 112 KiB shared memory and <= 256 TMEM columns each
  int s = 0;
  for (int k = MAX_STAGES; k >= 2; --k)
    if (C::smem_bytes(k) <= 112 * 1024 && C::tmem_need(k) <= 256) { s = k; break; }
  if (s == 0)  // one CTA per SM
    for (int k = MAX_STAGES; k >= 2; --k)
      if (C::smem_bytes(k) <= 220 * 1024 && C::tmem_need(k) <= 512) { s = k; break; }
  stages = s;
  cols = pow2_cols(C::tmem_need(s));
  smem = C::smem_bytes(s);
}

static void stages_dispatch(int bn, int t, int& stages, uint32_t& cols, size_t& smem) {
#define ADA_SD(B, TT) if (bn == B && t == TT) { stages_for<B, TT>(stages, cols, smem); return; }
  ADA_SD(16, 1) ADA_SD(16, 2) ADA_SD(16, 3) ADA_SD(32, 1) ADA_SD(32, 2) ADA_SD(32, 3)
  ADA_SD(64, 1) ADA_SD(64, 2) ADA_SD(128, 1)
#undef ADA_SD
  stages = 0;
}

static int make_plan(int64_t m, int64_t n, int64_t k, int terms, int force_ksplit, Plan& P) {
  if (m <= 0 || n <= 0 || k <= 0) return ADA_ERR_INVALID_ARG;
  if (terms < 1 || terms > 3) return ADA_ERR_INVALID_ARG;
  if (n % BM || k % KT) return ADA_ERR_UNSUPPORTED;
  if (m > (1 << 24) || n > (1 << 24) || k > (1 << 24)) return ADA_ERR_UNSUPPORTED;
  P.terms = terms;
  P.bn = block_n_for(m, terms);
  P.m_tiles = (int)cdiv(m, P.bn);
  P.m_pad = P.m_tiles * P.bn;
  P.n_tiles = (int)(n / BM);
  P.nkt = (int)(k / KT);
  const int tiles = P.n_tiles * P.m_tiles;
  int ks = 1;
  if (force_ksplit > 0) {
    ks = force_ksplit;
  } else if (tiles < 148) {
    ks = 296 / tiles;
    ks = ks < P.nkt / 2 ? ks : P.nkt / 2;
    if (ks < 1) ks = 1;
  }
  if (ks > P.nkt) ks = P.nkt;
  if (ks > 64) ks = 64;
  P.ksplit = ks;
  uint32_t cols = 0;
  stages_dispatch(P.bn, terms, P.stages, cols, P.smem);
  if (P.stages < 2) return ADA_ERR_UNSUPPORTED;
  P.tmem_cols = (int)cols;
  size_t off = 0;
  P.off_ctl = off;
  off = al256(off + (size_t)tiles * 4 + 16);
  P.off_xq = off;
  off = al256(off + (size_t)terms * P.m_pad * (size_t)(k / 2));
  P.off_sfx = off;
  off = al256(off + (size_t)P.m_tiles * (size_t)(k / 64) * 512);
  P.off_gx = off;
  off = al256(off + (size_t)P.m_pad * 4);
  P.off_part = off;
  if (P.ksplit > 1) off = al256(off + (size_t)P.ksplit * P.m_pad * (size_t)n * 4);
  P.total = off;
  return ADA_OK;
}

template <int BN, int T>
static int launch_gemm(const CUtensorMap& tmw, const CUtensorMap& tmx, const GemmParams& gp, const Plan& P,
                       cudaStream_t st) {
  auto kern = gemm_kernel<BN, T>;
  static size_t configured = 0;  // per instantiation
  if (P.smem > configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P.smem) != cudaSuccess)
      return ADA_ERR_CUDA;
    configured = P.smem;
  }
  dim3 grid(P.n_tiles * P.m_tiles, P.ksplit);
  (void)ada::launch_k(kern, dim3(grid), dim3(128), P.smem, st, tmw, tmx, gp);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

static int dispatch_gemm(const CUtensorMap& tmw, const CUtensorMap& tmx, const GemmParams& gp, const Plan& P,
                         cudaStream_t st) {
#define ADA_G(B, TT) if (P.bn == B && P.terms == TT) return launch_gemm<B, TT>(tmw, tmx, gp, P, st);
  ADA_G(16, 1) ADA_G(16, 2) ADA_G(16, 3) ADA_G(32, 1) ADA_G(32, 2) ADA_G(32, 3)
  ADA_G(64, 1) ADA_G(64, 2) ADA_G(128, 1)
#undef ADA_G
  return ADA_ERR_UNSUPPORTED;
}

static int run_gemm(const Plan& P, const uint8_t* xq, const uint8_t* sfx, const float* gx, int m, int n, int k,
                    const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w, const float* w_scale_2,
                    const void* bias, void* y, int y_dtype, int64_t ldy, uint8_t* ctl, uint8_t* part,
                    cudaStream_t st) {
  CUtensorMap tmw, tmx;
  if (!make_map(&tmw, w_packed, (uint64_t)(k / 2), (uint64_t)n, (uint64_t)ldw, BM)) return ADA_ERR_CUDA;
  if (!make_map(&tmx, xq, (uint64_t)(k / 2), (uint64_t)P.terms * P.m_pad, (uint64_t)(k / 2),
                (uint32_t)(P.terms * P.bn)))
    return ADA_ERR_CUDA;
  GemmParams gp;
  gp.sfw = sf_w;
  gp.sfx = sfx;
  gp.gx = gx;
  gp.gw = w_scale_2;
  gp.bias = bias;
  gp.y = y;
  gp.partial = reinterpret_cast<float*>(part);
  gp.counters = reinterpret_cast<int*>(ctl);
  gp.err = reinterpret_cast<unsigned int*>(ctl + (size_t)P.n_tiles * P.m_tiles * 4);
  gp.M = m;
  gp.N = n;
  gp.K = k;
  gp.ldy = (int)ldy;
  gp.m_pad = P.m_pad;
  gp.n_tiles = P.n_tiles;
  gp.m_tiles = P.m_tiles;
  gp.ksplit = P.ksplit;
  gp.stages = P.stages;
  gp.tmem_cols = P.tmem_cols;
  gp.out_dtype = y_dtype;
  return dispatch_gemm(tmw, tmx, gp, P, st);
}

// Workspace of the pre-quantised GEMM: control words + split-K partials only.
static size_t gemm_ws_bytes(const Plan& P, int64_t n) {
  size_t off = al256((size_t)P.n_tiles * P.m_tiles * 4 + 16);
  if (P.ksplit > 1) off = al256(off + (size_t)P.ksplit * P.m_pad * (size_t)n * 4);
  return off;
}

}  // namespace fp4
}  // namespace ada

using namespace ada;

static inline size_t al256_pub(size_t x) { return (x + 255) & ~size_t(255); }

extern "C" size_t ada_nvfp4_sf_bytes(int64_t n, int64_t k) {
  if (n <= 0 || k <= 0 || k % 64) return 0;
  return (size_t)cdiv(n, 128) * 128 * (size_t)(k / 16);
}

extern "C" int ada_nvfp4_prepack_scales(const void* scale, int scale_is_fp16, int64_t ld_scale, int64_t n, int64_t k,
                                        uint8_t* sf_out, void* stream) {
  if (!scale || !sf_out || n <= 0 || k <= 0) return ADA_ERR_INVALID_ARG;
  if (k % 64 || ld_scale < k / 16) return ADA_ERR_UNSUPPORTED;
  if ((uintptr_t)sf_out & 15) return ADA_ERR_ALIGNMENT;
  const int64_t blocks = cdiv(n, 128) * (k / 64);
  if (blocks > 0x7fffffff) return ADA_ERR_UNSUPPORTED;
  (void)ada::launch_k(fp4::prepack_kernel, dim3((unsigned)blocks), dim3(128), 0, reinterpret_cast<cudaStream_t>(stream), 
      scale, scale_is_fp16, ld_scale, (int)n, (int)k, sf_out);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

extern "C" size_t ada_nvfp4_linear_workspace_size(int64_t m, int64_t n, int64_t k, int terms) {
  fp4::Plan P;
  if (fp4::make_plan(m, n, k, terms, 0, P) != ADA_OK) return 0;
  return P.total;
}

extern "C" int ada_nvfp4_linear_ex(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k,
                                   const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w, const float* w_scale_2,
                                   int64_t n, const void* bias, void* y, int y_dtype, int64_t ldy, int terms,
                                   int force_ksplit, void* workspace, size_t workspace_bytes, void* stream) {
  if (m == 0) return ADA_OK;
  if (!x || !w_packed || !sf_w || !w_scale_2 || !y || !workspace) return ADA_ERR_INVALID_ARG;
  if ((x_dtype != ADA_DT_BF16 && x_dtype != ADA_DT_F16) || (y_dtype != ADA_DT_BF16 && y_dtype != ADA_DT_F16))
    return ADA_ERR_INVALID_ARG;
  if (ldx < k || ldy < n || ldw < k / 2) return ADA_ERR_INVALID_ARG;
  fp4::Plan P;
  int rc = fp4::make_plan(m, n, k, terms, force_ksplit, P);
  if (rc != ADA_OK) return rc;
  if (workspace_bytes < P.total) return ADA_ERR_WORKSPACE;
  if (((uintptr_t)x & 15) || (ldx & 7) || ((uintptr_t)w_packed & 15) || (ldw & 15) || ((uintptr_t)sf_w & 15) ||
      ((uintptr_t)workspace & 255))
    return ADA_ERR_ALIGNMENT;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  uint8_t* xq = ws + P.off_xq;
  uint8_t* sfx = ws + P.off_sfx;
  float* gx = reinterpret_cast<float*>(ws + P.off_gx);
  if (x_dtype == ADA_DT_BF16)
    (void)ada::launch_k(fp4::act_quant_kernel<__nv_bfloat16>, dim3(P.m_pad), dim3(256), 0, st, reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                                                                  (int)m, (int)k, terms, P.bn, P.m_tiles, P.m_pad, xq,
                                                                  sfx, gx);
  else
    (void)ada::launch_k(fp4::act_quant_kernel<__half>, dim3(P.m_pad), dim3(256), 0, st, reinterpret_cast<const __half*>(x), ldx, (int)m, (int)k,
                                                           terms, P.bn, P.m_tiles, P.m_pad, xq, sfx, gx);
  ADA_CHECK_LAUNCH();

  return fp4::run_gemm(P, xq, sfx, gx, (int)m, (int)n, (int)k, w_packed, ldw, sf_w, w_scale_2, bias, y, y_dtype,
                       ldy, ws + P.off_ctl, ws + P.off_part, st);
}

extern "C" int ada_nvfp4_linear(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k,
                                const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w, const float* w_scale_2,
                                int64_t n, const void* bias, void* y, int y_dtype, int64_t ldy, int terms,
                                void* workspace, size_t workspace_bytes, void* stream) {
  return ada_nvfp4_linear_ex(x, x_dtype, ldx, m, k, w_packed, ldw, sf_w, w_scale_2, n, bias, y, y_dtype, ldy, terms,
                             0, workspace, workspace_bytes, stream);
}

extern "C" int ada_nvfp4_act_quant(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k, int terms,
                                   int block_n, uint8_t* xq, uint8_t* sfx, float* gx, void* stream) {
  if (m <= 0 || k <= 0 || !x || !xq || !sfx || !gx) return ADA_ERR_INVALID_ARG;
  if (terms < 1 || terms > 3 || (x_dtype != ADA_DT_BF16 && x_dtype != ADA_DT_F16)) return ADA_ERR_INVALID_ARG;
  if (block_n != 16 && block_n != 32 && block_n != 64 && block_n != 128) return ADA_ERR_INVALID_ARG;
  if (terms * block_n > 128) return ADA_ERR_INVALID_ARG;
  if (k % 256 || ldx < k) return ADA_ERR_UNSUPPORTED;
  if (((uintptr_t)x & 15) || (ldx & 7) || ((uintptr_t)xq & 15)) return ADA_ERR_ALIGNMENT;
  const int m_tiles = (int)cdiv(m, block_n), m_pad = m_tiles * block_n;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (x_dtype == ADA_DT_BF16)
    (void)ada::launch_k(fp4::act_quant_kernel<__nv_bfloat16>, dim3(m_pad), dim3(256), 0, st, reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                                                                (int)m, (int)k, terms, block_n, m_tiles, m_pad, xq,
                                                                sfx, gx);
  else
    (void)ada::launch_k(fp4::act_quant_kernel<__half>, dim3(m_pad), dim3(256), 0, st, reinterpret_cast<const __half*>(x), ldx, (int)m, (int)k,
                                                         terms, block_n, m_tiles, m_pad, xq, sfx, gx);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

extern "C" int ada_nvfp4_workspace_status(const void* workspace, int64_t m, int64_t n, int64_t k, int terms,
                                          unsigned int* status_out, void* stream) {
  if (!workspace || !status_out) return ADA_ERR_INVALID_ARG;
  fp4::Plan P;
  int rc = fp4::make_plan(m, n, k, terms, 0, P);
  if (rc != ADA_OK) return rc;
  const uint8_t* errp = reinterpret_cast<const uint8_t*>(workspace) + P.off_ctl + (size_t)P.n_tiles * P.m_tiles * 4;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(status_out, errp, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return ADA_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return ADA_ERR_CUDA;
  return ADA_OK;
}

extern "C" int ada_nvfp4_block_n(int64_t m, int terms) {
  if (m <= 0 || terms < 1 || terms > 3) return 0;
  return fp4::block_n_for(m, terms);
}

extern "C" size_t ada_nvfp4_gemm_workspace_size(int64_t m, int64_t n, int64_t k, int terms) {
  fp4::Plan P;
  if (fp4::make_plan(m, n, k, terms, 0, P) != ADA_OK) return 0;
  return fp4::gemm_ws_bytes(P, n);
}

extern "C" int ada_nvfp4_gemm(const uint8_t* xq, const uint8_t* sfx, const float* gx, int64_t m, int terms,
                              int block_n, const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                              const float* w_scale_2, int64_t n, int64_t k, const void* bias, void* y, int y_dtype,
                              int64_t ldy, int force_ksplit, void* workspace, size_t workspace_bytes, void* stream) {
  if (m == 0) return ADA_OK;
  if (!xq || !sfx || !gx || !w_packed || !sf_w || !w_scale_2 || !y || !workspace) return ADA_ERR_INVALID_ARG;
  if (y_dtype != ADA_DT_BF16 && y_dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (ldy < n || ldw < k / 2) return ADA_ERR_INVALID_ARG;
  fp4::Plan P;
  int rc = fp4::make_plan(m, n, k, terms, force_ksplit, P);
  if (rc != ADA_OK) return rc;
  if (block_n != P.bn) return ADA_ERR_INVALID_ARG;
  if (workspace_bytes < fp4::gemm_ws_bytes(P, n)) return ADA_ERR_WORKSPACE;
  if (((uintptr_t)xq & 15) || ((uintptr_t)sfx & 15) || ((uintptr_t)w_packed & 15) || (ldw & 15) ||
      ((uintptr_t)sf_w & 15) || ((uintptr_t)workspace & 255))
    return ADA_ERR_ALIGNMENT;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  const size_t part_off = al256_pub((size_t)P.n_tiles * P.m_tiles * 4 + 16);
  return fp4::run_gemm(P, xq, sfx, gx, (int)m, (int)n, (int)k, w_packed, ldw, sf_w, w_scale_2, bias, y, y_dtype, ldy,
                       ws, ws + part_off, reinterpret_cast<cudaStream_t>(stream));
}
