// NVFP4 linear for B200: y = x . dequant(W)^T on the 5th-generation tensor cores.
//
// Replaces nvfp4_linear / nvfp4_gemm_kernel (reference adallm/ops/nvfp4_gemm.py:58-136,
// :460-564).  The reference widens e2m1 weights to fp16 with a lookup table and a
// per-element scale gather inside the K loop; here the packed weights stay packed:
//
//   * W [N, K/2] e2m1 bytes (even K in the low nibble) is TMA-loaded as-is into
//     128-byte-swizzled shared memory; its e4m3 per-16 scales are re-laid out
//     once at load ("prepack") into the block-scaled MMA scale-factor layout.
//   * The bf16 activation row is quantised by the producing kernel (quant.cuh) into
//     `terms` e2m1 terms: terms == 1 is NVFP4 with per-16 block scales (W4A4); terms >= 2
//     are row-scaled terms (unit block scales, one fp32 scale per row and term) whose sum
//     is within ~1e-3 (4 terms) of the bf16 activation.
//   * tcgen05.mma.kind::mxf4nvf4.block_scale.block16 with M = 128 weight rows ("swap AB":
//     tokens are the MMA N dimension); the terms are stacked along N (N = terms x tokens),
//     so one MMA per 64-wide K block covers every term.  fp32 accumulation in TMEM.  For
//     row-scaled terms the activation block scales are the constant 1.0, copied to TMEM once.
//   * The epilogue scales each term's accumulator column by its row scale, sums the terms,
//     and writes bf16/fp16.  Split-K: the CTAs sharing one output tile form a thread-block
//     cluster; each sends its scaled fp32 partial rows to the CTA owning them through
//     distributed shared memory, and the owner sums the partials in CTA-rank order
//     (deterministic, no global partials, no atomics).
//
// Warp roles (192 threads): warp 0 lane 0 issues TMA / bulk copies, warp 1 owns the TMEM
// allocation and lane 0 issues tcgen05.cp (scales -> TMEM) and the MMAs, warps 2..5 run the
// epilogue (warp w reads TMEM lanes 32*(w%4)..+31).  Every mbarrier wait is bounded (2 s);
// a timeout sets an error bit in the workspace and the CTA drains and exits.
#include "cluster.cuh"
#include "parts.cuh"
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
constexpr int MAX_PEERS = 8;
constexpr int MAX_KS = cl::MAX_CLUSTER;
constexpr uint32_t UNIT_SCALE4 = 0x38383838u;  // four ue4m3 1.0

struct GemmParams {
  const uint8_t* sfw;  // [N/128][K/64][512]
  const uint8_t* sfx;  // [m_tiles][K/64][512] (terms == 1)
  const float* gx;     // [m_pad] row scale (g or g_0)
  const float* gw;     // weight_scale_2 (device scalar)
  const void* bias;    // [N] (out dtype) or null
  void* y;             // [M, ldy] out dtype
  unsigned int* err;
  float* part;          // non-null: write scaled fp32 partial planes instead of reducing (no cluster)
  int64_t part_plane;   // floats between planes (one plane per K split)
  int part_ld;          // floats between rows of a plane
  int M, N, K, ldy, n_tiles, nkt, stages, tmem_cols, out_dtype, ks, rows_max;
  // tensor parallelism over peer memory (world > 1): the partial of K split s of this rank
  // goes to plane tp_rank * ks + s of every rank's inbox as tagged 8-byte words (value bits |
  // tag << 32, tag = *epoch * tag_mul + tag_add), which the consumer polls: no fence, no counter
  int world, tp_rank;
  // grouped (MoE) GEMM: m-tile t of the operand belongs to expert tile_expert[t] (< 0: unused
  // tile, the CTA exits), whose weights are rows [e * N, (e + 1) * N) of the stacked matrix;
  // operand row r is output row row_map[r] (< 0: padding, not stored).  Null: dense.
  const int* tile_expert;
  const int* row_map;
  int m_tiles_max;  // grouped: operand tiles in the plan (the routing uses a prefix of them)
  unsigned long long* inbox[MAX_PEERS];
  const unsigned int* epoch;
  unsigned int tag_mul, tag_add;
  // optional: byte ranges (the next projection's packed weights and scale factors) that this
  // launch's CTAs pull into L2 once their own loads are issued, so the next GEMM of a decode
  // layer finds its weights in L2 while the latency-bound kernels in between leave HBM idle
  const uint8_t* pf[2];
  int64_t pf_bytes[2];
};

// This CTA's share (CTA `id` of `n`) of `bytes` starting at `base`, requested into L2 in pieces
// of at most 32 KiB (16-byte aligned addresses and sizes; `bytes` a multiple of 16).
__device__ __forceinline__ void prefetch_share(const uint8_t* base, int64_t bytes, int64_t id, int64_t n) {
  if (!base || bytes <= 0) return;
  const int64_t chunk = ((bytes + n - 1) / n + 15) & ~int64_t(15);
  const int64_t b0 = id * chunk, b1 = b0 + chunk < bytes ? b0 + chunk : bytes;
  for (int64_t off = b0; off < b1; off += 32768) {
    const int64_t sz = b1 - off < 32768 ? b1 - off : 32768;
    sm100::bulk_prefetch_l2(base + off, (uint32_t)sz);
  }
}

template <int BN, int T>
struct Cfg {
  static constexpr int NB = BN * T;
  static_assert(NB % 16 == 0 && NB <= 128, "stacked terms must fit one 128-row scale block");
  static constexpr bool BLOCK_SF = T == 1;                // activation block scales per stage
  static constexpr uint32_t A_BYTES = BM * KT_BYTES;      // 16 KiB
  static constexpr uint32_t B_BYTES = NB * KT_BYTES;      // all terms
  static constexpr uint32_t SFA_BYTES = 4 * SF_BLOCK;     // 2 KiB
  static constexpr uint32_t SFB_BYTES = BLOCK_SF ? 4 * SF_BLOCK : 0;
  static constexpr uint32_t STAGE = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;  // multiple of 1024
  static constexpr uint32_t SF_COLS = BLOCK_SF ? 32 : 16;  // TMEM scale columns per stage
  static constexpr uint32_t CONST_SF = BLOCK_SF ? 0 : SF_BLOCK;
  static constexpr uint32_t CTRL = 1024;
  __host__ __device__ static size_t recv_bytes(int ks, int rows_max) { return ks > 1 ? (size_t)ks * rows_max * BN * 4 : 0; }
  static size_t smem_bytes(int stages, size_t recv) {
    return 1024 + (size_t)stages * STAGE + CONST_SF + recv + CTRL;
  }
  static uint32_t tmem_need(int stages) { return NB + stages * SF_COLS + (BLOCK_SF ? 0 : 4); }
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
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Split-K ownership of the 128 rows of a tile: row r belongs to CTA (r * ks) / 128.
__host__ __device__ __forceinline__ int owner_begin(int o, int ks) { return (o * BM + ks - 1) / ks; }

// grid (ks, tiles), cluster (ks, 1, 1) when ks > 1.  CTA `rank` of a cluster accumulates
// K steps [rank*nkt/ks, (rank+1)*nkt/ks) of tile blockIdx.y.
// Register budget: tiles of at most 96 MMA columns are held to 3 CTAs' worth (96 registers a
// thread), so two GEMM CTAs leave room on the SM for the CTAs of the kernels around them;
// wider tiles (which would spill) keep the 2-CTA budget.
template <int BN, int T>
__global__ void __launch_bounds__(192, (BN * T <= 96) ? 3 : 2)
    gemm_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx, const GemmParams p) {
  using C = Cfg<BN, T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = p.stages, ks = p.ks;
  const bool cluster = ks > 1 && p.part == nullptr;  // split-K reduced through the cluster
  uint8_t* const_sf = smem + (size_t)stages * C::STAGE;
  float* recv = reinterpret_cast<float*>(const_sf + C::CONST_SF);  // [ks][rows_max][BN]
  uint8_t* ctrl = reinterpret_cast<uint8_t*>(recv) + C::recv_bytes(cluster ? ks : 1, p.rows_max);
  uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
  uint64_t* empty = full + MAX_STAGES;
  uint64_t* accf = empty + MAX_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  // cluster split-K: counts the bytes of this CTA's rows arriving from the cluster (st.async)
  unsigned long long* rbar = reinterpret_cast<unsigned long long*>(ctrl + 144);
  float* gsc = reinterpret_cast<float*>(ctrl + 256);  // [T][BN] gw * term scale per token
  volatile int* abort_v = abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = blockIdx.x, tile = blockIdx.y;
  const int n_tile = tile % p.n_tiles, m_tile = tile / p.n_tiles;
  int expert = 0;
  if (p.tile_expert) {  // the routing written by the previous kernel decides whether this tile runs
    pdl_wait();
    expert = p.tile_expert[m_tile];
    if (expert < 0) return;  // before any barrier or TMEM: nothing to release
  }
  const int w_tile = expert * p.n_tiles + n_tile;  // 128-row block of the (stacked) weight matrix
  const int kt0 = (int)((int64_t)rank * p.nkt / ks), kt1 = (int)((int64_t)(rank + 1) * p.nkt / ks);
  const int nunits = kt1 - kt0;
  const int kb64 = p.K / 64;

  if (cluster) {
    if (threadIdx.x == 0) {  // before the cluster's start barrier: peers send into it after theirs
      const int own = owner_begin(rank + 1, ks) - owner_begin(rank, ks);
      cl::exchange_init_bytes(rbar, (uint32_t)(ks * own * BN * 4));
      cl::fence_exchange_init();
    }
    cl::cluster_arrive_relaxed();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (!C::BLOCK_SF && threadIdx.x < C::CONST_SF / 4) {
    reinterpret_cast<uint32_t*>(const_sf)[threadIdx.x] = UNIT_SCALE4;
    fence_proxy_async_smem();  // visible to tcgen05.cp
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
      // ---------------- producer ----------------
      // The weights never depend on the previous kernel: the first `stages` weight tiles
      // are requested before the programmatic-launch dependency wait.
      const int pre = nunits < stages ? nunits : stages;
      for (int i = 0; i < pre; ++i) {
        const int kt = kt0 + i;
        uint8_t* st = smem + (size_t)i * C::STAGE;
        mbar_expect_tx(&full[i], C::A_BYTES + C::SFA_BYTES);
        tma_load_2d(st, &tmw, &full[i], kt * KT_BYTES, w_tile * BM);
        bulk_load(st + C::A_BYTES + C::B_BYTES, p.sfw + ((size_t)w_tile * kb64 + (size_t)kt * 4) * SF_BLOCK,
                  C::SFA_BYTES, &full[i]);
      }
      // The rest of this CTA's weight slice is pulled into L2 while the previous kernel runs.
      for (int i = pre; i < nunits; ++i) {
        const int kt = kt0 + i;
        tma_prefetch_l2_2d(&tmw, kt * KT_BYTES, w_tile * BM);
        bulk_prefetch_l2(p.sfw + ((size_t)w_tile * kb64 + (size_t)kt * 4) * SF_BLOCK, C::SFA_BYTES);
      }
      pdl_wait();
      for (int i = 0; i < nunits; ++i) {
        const int s = i % stages;
        const int kt = kt0 + i;
        uint8_t* st = smem + (size_t)s * C::STAGE;
        if (i >= stages) {
          if (!mbar_wait_bounded(&empty[s], ((i / stages) & 1) ^ 1, abort_v, p.err, 1u)) break;
          mbar_expect_tx(&full[s], C::A_BYTES + C::SFA_BYTES);
          tma_load_2d(st, &tmw, &full[s], kt * KT_BYTES, w_tile * BM);
          bulk_load(st + C::A_BYTES + C::B_BYTES, p.sfw + ((size_t)w_tile * kb64 + (size_t)kt * 4) * SF_BLOCK,
                    C::SFA_BYTES, &full[s]);
        }
        mbar_arrive_expect_tx(&full[s], C::B_BYTES + C::SFB_BYTES);
        tma_load_2d(st + C::A_BYTES, &tmx, &full[s], kt * KT_BYTES, m_tile * C::NB);
        if (C::BLOCK_SF)
          bulk_load(st + C::A_BYTES + C::B_BYTES + C::SFA_BYTES,
                    p.sfx + ((size_t)m_tile * kb64 + (size_t)kt * 4) * SF_BLOCK, C::SFB_BYTES, &full[s]);
      }
      // every load of this CTA is issued: its share of the next projection's weights goes to L2
      const int64_t cta = (int64_t)blockIdx.y * gridDim.x + blockIdx.x, ctas = (int64_t)gridDim.x * gridDim.y;
      for (int r = 0; r < 2; ++r) prefetch_share(p.pf[r], p.pf_bytes[r], cta, ctas);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_mxf4nvf4(C::NB);
      const uint32_t sf_base = tmem + C::NB;
      const uint32_t sfb_unit = sf_base + stages * C::SF_COLS;  // constant 1.0 activation scales
      if (!C::BLOCK_SF) tmem_cp_32x128b_x4(sfb_unit, desc_sf(smem_u32(const_sf)));
      for (int i = 0; i < nunits; ++i) {
        const int s = i % stages;
        if (!mbar_wait_bounded(&full[s], (i / stages) & 1, abort_v, p.err, 2u)) break;
        tc_fence_after();
        uint8_t* st = smem + (size_t)s * C::STAGE;
        const uint32_t a_addr = smem_u32(st);
        const uint32_t b_addr = a_addr + C::A_BYTES;
        const uint32_t sfa_addr = b_addr + C::B_BYTES;
        const uint32_t sf_col = sf_base + s * C::SF_COLS;
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          tmem_cp_32x128b_x4(sf_col + 4 * kb, desc_sf(sfa_addr + kb * SF_BLOCK));
          if (C::BLOCK_SF) tmem_cp_32x128b_x4(sf_col + 16 + 4 * kb, desc_sf(sfa_addr + C::SFA_BYTES + kb * SF_BLOCK));
        }
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
          mma_mxf4nvf4(tmem, desc_kmajor_sw128(a_addr + kb * 32), desc_kmajor_sw128(b_addr + kb * 32), idesc,
                       (i | kb) != 0, sf_col + 4 * kb, C::BLOCK_SF ? sf_col + 16 + 4 * kb : sfb_unit);
        tc_commit(&empty[s]);  // stage reusable once these MMAs have read it
      }
      tc_commit(accf);  // accumulator complete (also after an abort: drains issued MMAs)
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5: TMEM lane quarter = warp % 4) ----------------
    pdl_wait();     // row scales written by the producing kernel are visible from here on
    pdl_trigger();  // let the next kernel get resident while this one streams
    const int q = warp & 3;
    const int et = threadIdx.x - 64;  // 0..127 within the epilogue group
    if (et < BN) {
      const float gw = __ldg(p.gw + expert);
      float g = __ldg(p.gx + m_tile * BN + et);
#pragma unroll
      for (int t = 0; t < T; ++t) {
        gsc[t * BN + et] = __fmul_rn(gw, g);
        g = q::next_term_scale(g);
      }
    }
    epi_bar();
    const bool ok = mbar_wait_bounded(accf, 0, abort_v, p.err, 4u) && !*abort_v;
    tc_fence_after();
    __syncwarp();
    float out[BN];
#pragma unroll
    for (int j = 0; j < BN; ++j) out[j] = 0.f;
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll
    for (int c = 0; c < C::NB; c += 16) {
      float v[16];
      tmem_ld16(lane_addr + c, v);
#pragma unroll
      for (int k = 0; k < 16; ++k) out[(c % BN) + k] = fmaf(v[k], gsc[c + k], out[(c % BN) + k]);  // terms in order
    }
    const int r = q * 32 + lane;
    if (p.part && p.world > 1) {
      // every rank's inbox gets this rank's partial of K split `rank` (peer stores over NVLink),
      // each value with this step's tag in the same 8-byte store (stale words are visible as such)
      const unsigned long long tag = (unsigned long long)(*p.epoch * p.tag_mul + p.tag_add) << 32;
      const int64_t off = (int64_t)(p.tp_rank * ks + rank) * p.part_plane + n_tile * BM + r;
      for (int d = 0; d < p.world; ++d) {
        unsigned long long* pp = p.inbox[d] + off;
#pragma unroll
        for (int j = 0; j < BN; ++j) {
          const int m = m_tile * BN + j;
          const float v = ok ? out[j] : __int_as_float(0x7fc00000);  // an aborted tile delivers NaN
          if (m < p.M) pp[(int64_t)m * p.part_ld] = tag | __float_as_uint(v);
        }
      }
    } else if (p.part) {
      // fp32 partial of this K split; the consumer sums the planes in split order
      if (ok) {
        float* pp = p.part + (int64_t)rank * p.part_plane + n_tile * BM + r;
#pragma unroll
        for (int j = 0; j < BN; ++j) {
          const int m = m_tile * BN + j;
          if (m < p.M) pp[(int64_t)m * p.part_ld] = out[j];
        }
      }
    } else if (ks == 1) {
      if (ok) {
        const int n = n_tile * BM + r;
        const float b = load_bias(p.bias, p.out_dtype, n);
#pragma unroll
        for (int j = 0; j < BN; ++j) {
          const int m = p.row_map ? p.row_map[m_tile * BN + j] : m_tile * BN + j;
          if (m >= 0 && m < p.M) store_out(p.y, p.out_dtype, (int64_t)m * p.ldy + n, out[j] + b);
        }
      }
    } else {
      const int owner = (r * ks) / BM;
      const int rl = r - owner_begin(owner, ks);
      cl::cluster_wait();  // every CTA of the cluster runs: its shared memory may be written
      const uint32_t dst = cl::mapa(recv + ((size_t)rank * p.rows_max + rl) * BN, (uint32_t)owner);
      const uint32_t obar = cl::mapa(rbar, (uint32_t)owner);
#pragma unroll
      for (int j = 0; j < BN; j += 4) cl::st_async_v4(dst + j * 4, out[j], out[j + 1], out[j + 2], out[j + 3], obar);
      cl::exchange_wait(rbar);  // every partial row this CTA owns has arrived (one-way stores)
      const int r0 = owner_begin(rank, ks), rows = owner_begin(rank + 1, ks) - r0;
      for (int e = et; e < rows * BN; e += 128) {
        const int rr = e % rows, j = e / rows;
        float acc = 0.f;
        for (int src = 0; src < ks; ++src) acc += recv[((size_t)src * p.rows_max + rr) * BN + j];  // rank order
        const int n = n_tile * BM + r0 + rr, m = m_tile * BN + j;
        if (ok && m < p.M) store_out(p.y, p.out_dtype, (int64_t)m * p.ldy + n, acc + load_bias(p.bias, p.out_dtype, n));
      }
    }
  }
  if (cluster && warp < 2) cl::cluster_wait();  // the producer and MMA warps complete the start barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, p.tmem_cols);
}

// ---- persistent form for large problems (prefill; grouped MoE with many routed tiles) ----
// One CTA per SM walks tiles t = blockIdx.x, + gridDim.x, ... (m-tile major, so neighbouring
// CTAs share the activation tile).  The pipeline ring runs on across tiles, and two TMEM
// accumulators alternate: the epilogue drains tile i from one while the MMA warp fills tile i + 1
// into the other.  One K split, no partial planes (the planner picks it for those grids).
// TMEM columns: [acc 0: NB][acc 1: NB][stage scale factors][unit scales].
template <int BN, int T>
__global__ void __launch_bounds__(192, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                           const GemmParams p) {
  using C = Cfg<BN, T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = p.stages;
  uint8_t* const_sf = smem + (size_t)stages * C::STAGE;
  uint8_t* ctrl = const_sf + C::CONST_SF;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
  uint64_t* empty = full + MAX_STAGES;
  uint64_t* accf = empty + MAX_STAGES;  // [2] accumulator b complete
  uint64_t* acce = accf + 2;            // [2] accumulator b drained by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* gsc = reinterpret_cast<float*>(ctrl + 256);  // [T][BN]
  volatile int* abort_v = abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grouped (MoE): the m-tiles come from the routing (written by an earlier kernel), the used
  // ones first; a tile whose expert is < 0 and every later one are skipped by all roles alike
  const int tiles = p.n_tiles * (p.tile_expert ? p.m_tiles_max : (p.M + BN - 1) / BN);
  const int kb64 = p.K / 64;
  const int nkt = p.nkt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (!C::BLOCK_SF && threadIdx.x < C::CONST_SF / 4) {
    reinterpret_cast<uint32_t*>(const_sf)[threadIdx.x] = UNIT_SCALE4;
    fence_proxy_async_smem();
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
    if (lane == 0) {  // ---------------- producer ----------------
      pdl_wait();
      uint32_t it = 0;
      // the routing of the next tile is read one tile ahead, off the issue path
      int expert = p.tile_expert && (int)blockIdx.x < tiles ? p.tile_expert[blockIdx.x / p.n_tiles] : 0;
      for (int t = blockIdx.x; t < tiles && !*abort_v; t += gridDim.x) {
        const int n_tile = t % p.n_tiles, m_tile = t / p.n_tiles;
        if (expert < 0) break;
        const int tn = t + (int)gridDim.x;
        const int expert_next = p.tile_expert && tn < tiles ? p.tile_expert[tn / p.n_tiles] : 0;
        const int w_tile = expert * p.n_tiles + n_tile;
        for (int kt = 0; kt < nkt; ++kt, ++it) {
          const int s = (int)(it % (uint32_t)stages);
          if (it >= (uint32_t)stages &&
              !mbar_wait_bounded(&empty[s], ((it / stages) & 1) ^ 1, abort_v, p.err, 1u))
            break;
          uint8_t* st = smem + (size_t)s * C::STAGE;
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          tma_load_2d(st, &tmw, &full[s], kt * KT_BYTES, w_tile * BM);
          tma_load_2d(st + C::A_BYTES, &tmx, &full[s], kt * KT_BYTES, m_tile * C::NB);
          bulk_load(st + C::A_BYTES + C::B_BYTES, p.sfw + ((size_t)w_tile * kb64 + (size_t)kt * 4) * SF_BLOCK,
                    C::SFA_BYTES, &full[s]);
          if (C::BLOCK_SF)
            bulk_load(st + C::A_BYTES + C::B_BYTES + C::SFA_BYTES,
                      p.sfx + ((size_t)m_tile * kb64 + (size_t)kt * 4) * SF_BLOCK, C::SFB_BYTES, &full[s]);
        }
        expert = expert_next;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_mxf4nvf4(C::NB);
      const uint32_t sf_base = tmem + 2 * C::NB;
      const uint32_t sfb_unit = sf_base + stages * C::SF_COLS;
      if (!C::BLOCK_SF) tmem_cp_32x128b_x4(sfb_unit, desc_sf(smem_u32(const_sf)));
      if (p.tile_expert) pdl_wait();  // the routing is read below
      uint32_t it = 0, lt = 0;
      int expert = p.tile_expert && (int)blockIdx.x < tiles ? p.tile_expert[blockIdx.x / p.n_tiles] : 0;
      for (int t = blockIdx.x; t < tiles && !*abort_v; t += gridDim.x, ++lt) {
        if (expert < 0) break;
        const int tn = t + (int)gridDim.x;
        const int expert_next = p.tile_expert && tn < tiles ? p.tile_expert[tn / p.n_tiles] : 0;  // one tile ahead
        const uint32_t b = lt & 1, use = lt >> 1;
        if (use > 0 && !mbar_wait_bounded(&acce[b], (use - 1) & 1, abort_v, p.err, 8u)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * C::NB;
        bool failed = false;
        for (int kt = 0; kt < nkt; ++kt, ++it) {
          const int s = (int)(it % (uint32_t)stages);
          if (!mbar_wait_bounded(&full[s], (it / stages) & 1, abort_v, p.err, 2u)) {
            failed = true;
            break;
          }
          tc_fence_after();
          uint8_t* st = smem + (size_t)s * C::STAGE;
          const uint32_t a_addr = smem_u32(st);
          const uint32_t b_addr = a_addr + C::A_BYTES;
          const uint32_t sfa_addr = b_addr + C::B_BYTES;
          const uint32_t sf_col = sf_base + s * C::SF_COLS;
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            tmem_cp_32x128b_x4(sf_col + 4 * kb, desc_sf(sfa_addr + kb * SF_BLOCK));
            if (C::BLOCK_SF) tmem_cp_32x128b_x4(sf_col + 16 + 4 * kb, desc_sf(sfa_addr + C::SFA_BYTES + kb * SF_BLOCK));
          }
#pragma unroll
          for (int kb = 0; kb < 4; ++kb)
            mma_mxf4nvf4(acc, desc_kmajor_sw128(a_addr + kb * 32), desc_kmajor_sw128(b_addr + kb * 32), idesc,
                         (kt | kb) != 0, sf_col + 4 * kb, C::BLOCK_SF ? sf_col + 16 + 4 * kb : sfb_unit);
          tc_commit(&empty[s]);
        }
        tc_commit(&accf[b]);  // also after a failure: drains the issued MMAs
        if (failed) break;
        expert = expert_next;
      }
    }
    __syncwarp();
  } else {  // ---------------- epilogue (warps 2..5) ----------------
    pdl_wait();
    pdl_trigger();
    const int q = warp & 3;
    const int et = threadIdx.x - 64;
    const int r = q * 32 + lane;
    uint32_t lt = 0;
    // the next tile's expert, row scale and (grouped, 16-token tiles) output rows are read one
    // tile ahead, while this tile's accumulator is still being computed
    constexpr bool RM_REGS = BN <= 16;
    int ex_n = 0, rm_n[RM_REGS ? BN : 1];
    float g_n = 1.f, gw_n = 1.f;
    auto read_ahead = [&](int t) {
      if (t >= tiles) return;
      const int mt = t / p.n_tiles;
      ex_n = p.tile_expert ? p.tile_expert[mt] : 0;
      if (et < BN) {
        g_n = p.gx[mt * BN + et];
        if (ex_n >= 0) gw_n = __ldg(p.gw + ex_n);
      }
      if (RM_REGS && p.row_map)
#pragma unroll
        for (int k = 0; k < (RM_REGS ? BN : 1); ++k) rm_n[k] = p.row_map[mt * BN + k];
    };
    read_ahead(blockIdx.x);
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++lt) {
      const int n_tile = t % p.n_tiles, m_tile = t / p.n_tiles;
      const int expert = ex_n;
      if (expert < 0) break;
      const float g_t = g_n, gw = gw_n;
      int rm[RM_REGS ? BN : 1];
#pragma unroll
      for (int k = 0; k < (RM_REGS ? BN : 1); ++k) rm[k] = rm_n[k];
      read_ahead(t + (int)gridDim.x);
      const uint32_t b = lt & 1, use = lt >> 1;
      if (et < BN) {
        float g = g_t;
#pragma unroll
        for (int tt = 0; tt < T; ++tt) {
          gsc[tt * BN + et] = __fmul_rn(gw, g);
          g = q::next_term_scale(g);
        }
      }
      epi_bar();
      const bool ok = mbar_wait_bounded(&accf[b], use & 1, abort_v, p.err, 4u) && !*abort_v;
      tc_fence_after();
      __syncwarp();
      const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + b * C::NB;
      const int n = n_tile * BM + r;
      const float bias = load_bias(p.bias, p.out_dtype, n);
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {  // 16 tokens at a time, terms summed in order
        float o[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) o[k] = 0.f;
        uint32_t v[T][16];  // every term's 16 columns in flight together, one wait
#pragma unroll
        for (int tt = 0; tt < T; ++tt) tmem_ld16_nowait(lane_addr + tt * BN + c, v[tt]);
        tmem_wait_ld();
#pragma unroll
        for (int tt = 0; tt < T; ++tt)
#pragma unroll
          for (int k = 0; k < 16; ++k) o[k] = fmaf(__uint_as_float(v[tt][k]), gsc[tt * BN + c + k], o[k]);
        if (ok) {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const int m = !p.row_map ? m_tile * BN + c + k : RM_REGS ? rm[(c + k) % (RM_REGS ? BN : 1)]
                                                                       : p.row_map[m_tile * BN + c + k];
            if (m >= 0 && m < p.M) store_out(p.y, p.out_dtype, (int64_t)m * p.ldy + n, o[k] + bias);
          }
        }
      }
      tc_fence_before();
      epi_bar();  // every lane has read accumulator b (and gsc may be rewritten)
      if (et == 0) mbar_arrive_plain(&acce[b]);
      if (!ok) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, p.tmem_cols);
}

// ---- CTA-pair persistent GEMM (W4A4 at prefill sizes) ------------------------------------
// Operand reuse per staged byte decides the prefill-size GEMM: with 128 x 128 tiles every K
// step moves 256 operand rows from L2 into shared memory per 128 x 128 outputs, which bounds the
// one-CTA kernel above by the L2 -> SM copy rate long before the tensor pipe.  Here two CTAs of a
// cluster (one per SM) share one tcgen05.mma.cta_group::2 of M 256 x N 256 x K 64: the
// activations are the A operand (256 token rows, 128 in each CTA), the weights the B operand
// (256 weight rows, 128 in each CTA), and each CTA's TMEM holds its 128 token rows x 256 weight
// rows in fp32.  Per CTA and K step that is 256 staged rows for 128 x 256 outputs: half the
// traffic per FLOP.  Not swapped (tokens are the MMA M): a TMEM lane is a token row, so the
// epilogue writes each row's 256 outputs as contiguous 16-byte vectors.
//
// Scale factors: the A scales (each CTA's 128 tokens) sit in its own TMEM, 4 columns per 64-wide K
// block; the B scales cover all 256 weight rows in both CTAs (8 columns per K block: rows 0-127,
// then 128-255), copied from each CTA's own shared memory by one cta_group::2 tcgen05.cp.
//
// Protocol (CTA rank 0 of the pair leads; no multicast anywhere):
//   full[s]  (rank 0): both CTAs' TMA loads of stage s complete_tx here (cta_group::2 loads);
//                      rank 0's producer arms it with both CTAs' bytes.
//   empty[s] (each):   the leader's MMA thread commits to both CTAs' copies after stage s is read.
//   accf     (each):   accumulator complete, committed to both CTAs after a tile's last MMA.
//   acce     (rank 0): the 8 epilogue warps of both CTAs arrive once their TMEM loads are done
//                      (16 arrivals): one accumulator, drained into registers before the stores.
// Every wait is bounded (2 s); a timeout sets an error bit and the CTA drains and exits.
namespace pair {
constexpr int BT = 256;                     // tokens per tile (MMA M, 128 per CTA)
constexpr int BW = 256;                     // weight rows per tile (MMA N, 128 per CTA)
constexpr uint32_t A_BYTES = 128 * KT_BYTES;   // this CTA's 128 token rows x 256 K (16 KiB)
constexpr uint32_t B_BYTES = 128 * KT_BYTES;   // this CTA's 128 weight rows (16 KiB)
constexpr uint32_t SFA_BYTES = 4 * SF_BLOCK;   // this CTA's tokens, 4 K blocks (2 KiB)
constexpr uint32_t SFB_BYTES = 8 * SF_BLOCK;   // all 256 weight rows, 4 K blocks (4 KiB)
constexpr uint32_t STAGE = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;  // 38 KiB, multiple of 1024
constexpr int STAGES = 5;
constexpr int PRE_COPY = 3;                 // stages whose scale copies precede the accumulator wait
constexpr uint32_t SF_COLS = 16 + 32;       // TMEM scale columns per stage (A 4 x 4, B 4 x 8)
constexpr uint32_t ACC_COLS = BW;
constexpr uint32_t TMEM_COLS = 512;         // 256 accumulator + 5 x 48 scale columns, power of 2
constexpr int EPI_WARPS = 8;                // two per TMEM lane quarter, 128 columns each
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE + 1024;
static_assert(ACC_COLS + STAGES * SF_COLS <= TMEM_COLS, "TMEM budget");
static_assert(STAGE % 1024 == 0, "stage alignment");
}  // namespace pair

__global__ void __launch_bounds__(pair::THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                     const __grid_constant__ CUtensorMap tsw, const __grid_constant__ CUtensorMap tsx,
                     const GemmParams p) {
  using namespace pair;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ctrl = smem + (size_t)STAGES * STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint64_t* acce = accf + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_v = abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cl::ctarank() & 1u, peer = rank ^ 1u;
  const int w_pairs = p.N / BW;
  const int t_tiles = (p.M + BT - 1) / BT;
  const int tiles = w_pairs * t_tiles;
  const int pair_id = (int)(blockIdx.x >> 1), pairs = (int)(gridDim.x >> 1);
  const int kb64 = p.K / 64;
  const int nkt = p.nkt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    mbar_init(acce, 2 * EPI_WARPS);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmw);
    prefetch_tmap(&tmx);
    prefetch_tmap(&tsw);
    prefetch_tmap(&tsx);
  }
  tc_fence_before();
  cl::cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any pair traffic
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---------------- producer (both CTAs) ----------------
      pdl_wait();
      const uint32_t full0 = cl::mapa(&full[0], 0);  // the leader's stage barriers
      uint32_t it = 0;
      for (int t = pair_id; t < tiles && !*abort_v; t += pairs) {
        const int wp = t % w_pairs, tt = t / w_pairs;
        const int x_row = tt * BT + (int)rank * 128;       // this CTA's token rows (A)
        const int w_row = wp * BW + (int)rank * 128;       // this CTA's weight rows (B)
        const int x_blk = tt * 2 + (int)rank;              // 128-token scale block
        for (int kt = 0; kt < nkt; ++kt, ++it) {
          const int s = (int)(it % (uint32_t)STAGES);
          if (it >= (uint32_t)STAGES &&
              !mbar_wait_bounded(&empty[s], ((it / STAGES) & 1) ^ 1, abort_v, p.err, 1u))
            break;
          uint8_t* st = smem + (size_t)s * STAGE;
          const uint32_t bar = full0 + (uint32_t)s * 8u;
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * STAGE);
          tma_load_2d_pair(st, &tmx, bar, kt * KT_BYTES, x_row);
          tma_load_2d_pair(st + A_BYTES, &tmw, bar, kt * KT_BYTES, w_row);
          // scale maps: rows of 128 bytes; a (block, stage) chunk is 2 KiB = 16 rows
          tma_load_2d_pair(st + A_BYTES + B_BYTES, &tsx, bar, 0, (x_blk * kb64 + kt * 4) * 4);
          tma_load_2d_pair(st + A_BYTES + B_BYTES + SFA_BYTES, &tsw, bar, 0, ((wp * 2) * kb64 + kt * 4) * 4);
          tma_load_2d_pair(st + A_BYTES + B_BYTES + SFA_BYTES + 4 * SF_BLOCK, &tsw, bar, 0,
                           ((wp * 2 + 1) * kb64 + kt * 4) * 4);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {  // ---------------- MMA issuer (leader CTA only) ----------------
      constexpr uint32_t idesc = idesc_mxf4nvf4_m256(BW);
      const uint32_t empty0_own = cl::mapa(&empty[0], 0), empty0_peer = cl::mapa(&empty[0], peer);
      const uint32_t accf_own = cl::mapa(accf, 0), accf_peer = cl::mapa(accf, peer);
      // the scale-factor copies of one stage (they touch only that stage's TMEM scale columns)
      auto copy_scales = [&](int s) {
        const uint32_t sfa_addr = smem_u32(smem + (size_t)s * STAGE) + A_BYTES + B_BYTES;
        const uint32_t sfb_addr = sfa_addr + SFA_BYTES;
        const uint32_t sf_col = tmem + ACC_COLS + (uint32_t)s * SF_COLS;
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          tmem_cp_32x128b_x4_pair(sf_col + 4 * kb, desc_sf(sfa_addr + kb * SF_BLOCK));
          tmem_cp_32x128b_x4_pair(sf_col + 16 + 8 * kb, desc_sf(sfb_addr + kb * SF_BLOCK));
          tmem_cp_32x128b_x4_pair(sf_col + 16 + 8 * kb + 4, desc_sf(sfb_addr + 4 * SF_BLOCK + kb * SF_BLOCK));
        }
      };
      uint32_t it = 0, lt = 0;
      for (int t = pair_id; t < tiles && !*abort_v; t += pairs, ++lt) {
        // The first stages' scale copies go in before the accumulator-empty wait: they overlap
        // the epilogue's drain of the previous tile instead of following it.
        const int pre = nkt < PRE_COPY ? nkt : PRE_COPY;
        bool failed = false;
        for (int j = 0; j < pre; ++j) {
          const uint32_t ij = it + (uint32_t)j;
          if (!mbar_wait_bounded(&full[ij % STAGES], (ij / STAGES) & 1, abort_v, p.err, 2u)) {
            failed = true;
            break;
          }
          tc_fence_after();
          copy_scales((int)(ij % STAGES));
        }
        if (!failed && lt > 0 && !mbar_wait_bounded_cluster(acce, (lt - 1) & 1, abort_v, p.err, 8u)) failed = true;
        tc_fence_after();
        for (int kt = 0; kt < nkt && !failed; ++kt, ++it) {
          const int s = (int)(it % (uint32_t)STAGES);
          if (kt >= pre) {
            if (!mbar_wait_bounded(&full[s], (it / STAGES) & 1, abort_v, p.err, 2u)) {
              failed = true;
              break;
            }
            tc_fence_after();
            copy_scales(s);
          }
          const uint32_t a_addr = smem_u32(smem + (size_t)s * STAGE);
          const uint32_t b_addr = a_addr + A_BYTES;
          const uint32_t sf_col = tmem + ACC_COLS + (uint32_t)s * SF_COLS;
#pragma unroll
          for (int kb = 0; kb < 4; ++kb)
            mma_mxf4nvf4_pair(tmem, desc_kmajor_sw128(a_addr + kb * 32), desc_kmajor_sw128(b_addr + kb * 32), idesc,
                              (kt | kb) != 0, sf_col + 4 * kb, sf_col + 16 + 8 * kb);
          tc_commit_pair(empty0_own + (uint32_t)s * 8u);
          tc_commit_pair(empty0_peer + (uint32_t)s * 8u);
        }
        tc_commit_pair(accf_own);  // also after a failure: drains the issued MMAs
        tc_commit_pair(accf_peer);
        if (failed) break;
      }
    }
    __syncwarp();
  } else {  // ---------------- epilogue (warps 2..9, both CTAs) ----------------
    pdl_wait();
    pdl_trigger();
    const int q = warp & 3;                 // TMEM lane quarter this warp may read
    const int h = (warp - 2) >> 2;          // column half: weight rows h*128 .. +127 of the tile
    const uint32_t acce_lead = cl::mapa(acce, 0);
    const float gw = __ldg(p.gw);
    const bool bf16 = p.out_dtype == ADA_DT_BF16;
    uint32_t lt = 0;
    for (int t = pair_id; t < tiles; t += pairs, ++lt) {
      const int wp = t % w_pairs, tt = t / w_pairs;
      const int m = tt * BT + (int)rank * 128 + q * 32 + lane;
      const float g = m < p.M ? p.gx[m] : 0.f;  // read before the wait, off the drain path
      const bool ok = mbar_wait_bounded(accf, lt & 1, abort_v, p.err, 4u) && !*abort_v;
      tc_fence_after();
      __syncwarp();
      uint32_t v[128];
      const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)h * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) tmem_ld16_nowait(lane_addr + 16 * c, v + 16 * c);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce_lead);  // the accumulator is free for the next tile
      if (!ok) break;
      if (m < p.M) {
        const float gsc = __fmul_rn(gw, g);
        const int n0 = wp * BW + h * 128;
        const uint4* bias8 = p.bias ? reinterpret_cast<const uint4*>(p.bias) + n0 / 8 : nullptr;
        uint4* yrow = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.y) + (int64_t)m * p.ldy + n0);
#pragma unroll
        for (int gi = 0; gi < 16; ++gi) {
          float b[8];
          if (bias8) {
            const uint4 u = __ldg(bias8 + gi);
            if (bf16) unpack8<__nv_bfloat16>(u, b); else unpack8<__half>(u, b);
          } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) b[k] = 0.f;
          }
          float o[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] = fmaf(__uint_as_float(v[gi * 8 + k]), gsc, 0.f) + b[k];
          yrow[gi] = bf16 ? pack8<__nv_bfloat16>(o) : pack8<__half>(o);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cl::cluster_sync();  // neither CTA leaves while the pair's MMAs or arrivals may still reach it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, TMEM_COLS);
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
// 2-D byte matrix [rows, inner_bytes] with row stride `stride` bytes; box = 128 bytes x box_rows, 128B swizzle.
static bool make_map(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows, uint64_t stride,
                     uint32_t box_rows) {
  const cuuint64_t dims[2] = {inner_bytes, rows};
  const cuuint64_t strides[1] = {stride};
  const cuuint32_t box[2] = {128, box_rows};
  return encode_bytes(map, base, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Token tile: the smallest of 16/32/64/128 covering m, capped so terms*bn <= 128.
static inline int block_n_for(int64_t m, int terms) {
  int cap = 128;
  while (cap > 16 && cap * terms > 128) cap >>= 1;
  int bn = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : 128;
  return bn < cap ? bn : cap;
}

constexpr size_t ERR_BYTES = 256;  // error word at offset 0 of every GEMM workspace

struct Plan {
  int terms, bn, m_tiles, m_pad, n_tiles, nkt, ks, rows_max, stages, tmem_cols;
  size_t smem;
  // persistent form (one split, more tiles than two per SM): pipeline and TMEM of it
  bool persistent;
  int p_stages, p_cols;
  size_t p_smem;
  // workspace of ada_nvfp4_linear (bytes, 256-aligned): [err][xq][sfx][gx]
  size_t off_xq, off_sfx, off_gx, total;
};

static inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }
static inline uint32_t pow2_cols(uint32_t c) {
  uint32_t r = 32;
  while (r < c) r <<= 1;
  return r;
}

// Two co-resident CTAs per SM when shared memory and TMEM allow (each CTA's MMA thread
// issues its own tcgen05 stream); else one CTA per SM with a deeper pipeline.
// No more stages than the K steps of the longest split (`max_units`): a pipeline deeper than the
// work only holds shared memory that the next kernel's CTAs could use.
// per_sm = 3: the plan needs three co-resident CTAs per SM (shared memory <= 74 KB, TMEM <= 128
// columns; only tiles compiled to the 96-register budget); -1 stages if that does not fit.
template <int BN, int T>
static void stages_for(int ks, int rows_max, int max_units, int& stages, uint32_t& cols, size_t& smem,
                       int per_sm = 2) {
  using C = Cfg<BN, T>;
  const size_t recv = C::recv_bytes(ks, rows_max);
  const int top = max_units < 2 ? 2 : max_units < MAX_STAGES ? max_units : MAX_STAGES;
  int s = 0;
  if (per_sm == 3) {
    for (int k = top; k >= 2 && BN * T <= 96; --k)
      if (C::smem_bytes(k, recv) <= 74 * 1024 && C::tmem_need(k) <= 128) { s = k; break; }
    stages = s ? s : -1;
    cols = s ? pow2_cols(C::tmem_need(s)) : 0;
    smem = C::smem_bytes(s, recv);
    return;
  }
  for (int k = top; k >= (top < 3 ? top : 3); --k)
    if (C::smem_bytes(k, recv) <= 113 * 1024 && C::tmem_need(k) <= 256) { s = k; break; }
  if (s == 0)
    for (int k = top; k >= 2; --k)
      if (C::smem_bytes(k, recv) <= 226 * 1024 && C::tmem_need(k) <= 512) { s = k; break; }
  stages = s;
  cols = s ? pow2_cols(C::tmem_need(s)) : 0;
  smem = C::smem_bytes(s, recv);
}

// Persistent form: one CTA per SM, two accumulators; the deepest pipeline that fits.
template <int BN, int T>
static void persistent_stages_for(int& stages, uint32_t& cols, size_t& smem) {
  using C = Cfg<BN, T>;
  int s = 0;
  for (int k = MAX_STAGES; k >= 2; --k) {
    const size_t sm = 1024 + (size_t)k * C::STAGE + C::CONST_SF + C::CTRL;
    if (sm <= 226 * 1024 && 2 * C::NB + k * C::SF_COLS + (C::BLOCK_SF ? 0 : 4) <= 512) { s = k; break; }
  }
  stages = s;
  cols = s ? pow2_cols(2 * C::NB + s * C::SF_COLS + (C::BLOCK_SF ? 0 : 4)) : 0;
  smem = 1024 + (size_t)s * C::STAGE + C::CONST_SF + C::CTRL;
}

#define ADA_FP4_CONFIGS(X) \
  X(16, 1) X(16, 2) X(16, 3) X(16, 4) X(16, 5) X(16, 6) X(16, 7) X(16, 8) \
  X(32, 1) X(32, 2) X(32, 3) X(32, 4) X(64, 1) X(64, 2) X(128, 1)

static void stages_dispatch(int bn, int t, int ks, int rows_max, int max_units, int& stages, uint32_t& cols,
                            size_t& smem, int per_sm = 2) {
#define ADA_SD(B, TT) \
  if (bn == B && t == TT) { stages_for<B, TT>(ks, rows_max, max_units, stages, cols, smem, per_sm); return; }
  ADA_FP4_CONFIGS(ADA_SD)
#undef ADA_SD
  stages = 0;
}

// Raise the kernel's dynamic shared memory limit to `smem` (never lowers it) and prefer the
// maximum shared-memory carveout.
template <int BN, int T>
static bool ensure_smem(size_t smem) {
  static std::atomic<size_t> configured[64];  // per device
  static std::mutex raise;                    // raises only: concurrent callers must not lower it
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (smem <= configured[dev].load(std::memory_order_acquire)) return true;
  std::lock_guard<std::mutex> hold(raise);
  if (smem <= configured[dev].load(std::memory_order_acquire)) return true;
  if (cudaFuncSetAttribute(gemm_kernel<BN, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return false;
  // The whole unified L1/shared array as shared memory, so two ~100 KB CTAs fit on one SM
  // (the default carveout leaves room for one).
  if (cudaFuncSetAttribute(gemm_kernel<BN, T>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    return false;
  configured[dev].store(smem, std::memory_order_release);
  return true;
}

// Stand-in for gemm_kernel in occupancy queries: same block size, register cap and dynamic
// shared memory, but no TMEM allocation.  The occupancy calculator assumes one CTA per SM for
// kernels that allocate TMEM, while the hardware co-schedules two of these CTAs per SM
// (measured), so cluster capacity is queried on this twin instead.
__global__ void __launch_bounds__(192, 2) occupancy_twin() {}

// Clusters of `ks` CTAs (with the shared memory the plan gives them) that fit on the GPU at
// once; 0 if unknown.  A split whose clusters do not all fit runs in two waves.
template <int BN, int T>
static int active_clusters(int ks, int per_sm = 2) {
  static std::atomic<int> cache[64][2][MAX_KS + 1];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || ks < 1 || ks > MAX_KS) return 0;
  std::atomic<int>& slot = cache[dev][per_sm == 3 ? 1 : 0][ks];
  const int known = slot.load(std::memory_order_relaxed);
  if (known) return known > 0 ? known : 0;
  int stages = 0;
  uint32_t cols = 0;
  size_t smem = 0;
  // deepest pipeline of the budget: a lower bound of the capacity
  stages_for<BN, T>(ks, (int)cdiv(BM, ks), MAX_STAGES, stages, cols, smem, per_sm);
  int n = 0;
  if (stages >= 2 &&
      cudaFuncSetAttribute(occupancy_twin, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) == cudaSuccess &&
      cudaFuncSetAttribute(occupancy_twin, cudaFuncAttributePreferredSharedMemoryCarveout,
                           (int)cudaSharedmemCarveoutMaxShared) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ks, 1, 1);
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ks;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, occupancy_twin, &cfg) != cudaSuccess) n = 0;
  }
  (void)cudaGetLastError();
  slot.store(n > 0 ? n : -1, std::memory_order_relaxed);
  return n;
}

static int active_clusters_dispatch(int bn, int t, int ks, int per_sm = 2) {
#define ADA_AC(B, TT) if (bn == B && t == TT) return active_clusters<B, TT>(ks, per_sm);
  ADA_FP4_CONFIGS(ADA_AC)
#undef ADA_AC
  return 0;
}

static int num_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (!n) {
    int v = 0;
    n = (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) ? v : 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// A plan of ks splits whose pipeline (with the cluster reduction buffer when `cluster`) fits
// three CTAs to an SM.
static bool fits_three(int bn, int terms, int64_t ks, int nkt, bool cluster = false) {
  int st = 0;
  uint32_t c = 0;
  size_t sm = 0;
  stages_dispatch(bn, terms, cluster ? (int)ks : 1, (int)cdiv(BM, ks), (int)cdiv(nkt, ks), st, c, sm, 3);
  return st >= 2;
}

// force_ks > 0 overrides the split-K factor (tests of the cluster reduction).
// parts: split-K partial planes are written out (no cluster reduction, any split works).
static int make_plan(int64_t m, int64_t n, int64_t k, int terms, int force_ks, Plan& P, bool parts = false,
                     int force_bn = 0) {
  if (m <= 0 || n <= 0 || k <= 0) return ADA_ERR_INVALID_ARG;
  if (terms < 1 || terms > q::MAX_TERMS) return ADA_ERR_INVALID_ARG;
  if (n % BM || k % KT) return ADA_ERR_UNSUPPORTED;
  if (m > (1 << 24) || n > (1 << 24) || k > (1 << 24)) return ADA_ERR_UNSUPPORTED;
  P.terms = terms;
  P.bn = force_bn ? force_bn : block_n_for(m, terms);
  P.m_tiles = (int)cdiv(m, P.bn);
  P.m_pad = P.m_tiles * P.bn;
  P.n_tiles = (int)(n / BM);
  P.nkt = (int)(k / KT);
  const int64_t tiles = (int64_t)P.n_tiles * P.m_tiles;
  if (tiles > 65535) return ADA_ERR_UNSUPPORTED;
  // Split-K factor: the largest ks <= 8 that divides the K steps evenly, leaves every CTA at
  // least 4 of them (shorter splits cost more in the cluster reduction than they gain), and
  // whose clusters (one per tile) all fit on the GPU in one wave, at most two CTAs per SM.
  int64_t ks = 1;
  bool three_per_sm = false;
  const int64_t ks_cap = P.nkt < MAX_KS ? P.nkt : MAX_KS;
  if (force_ks > 0) {
    ks = force_ks < ks_cap ? force_ks : ks_cap;
  } else if (parts) {
    // as many splits as keep every CTA resident in one wave: three per SM when the pipeline
    // fits three to an SM (spreads a projection with few tiles over more SMs), else two
    ks = (3 * (int64_t)num_sms()) / tiles;
    ks = ks < 1 ? 1 : ks > ks_cap ? ks_cap : ks;
    if (tiles * ks > 2 * (int64_t)num_sms() && !fits_three(P.bn, terms, ks, P.nkt)) {
      ks = (2 * (int64_t)num_sms()) / tiles;
      ks = ks < 1 ? 1 : ks > ks_cap ? ks_cap : ks;
    }
  } else {
    // two CTAs per SM, or three (74 KB pipeline) when that lets a larger split stay in one wave
    for (int64_t c = (P.nkt / 4 < ks_cap ? P.nkt / 4 : ks_cap); c >= 2; --c) {
      if (P.nkt % c) continue;
      if (tiles * c <= 2 * (int64_t)num_sms() && tiles <= active_clusters_dispatch(P.bn, terms, (int)c)) {
        ks = c;
        break;
      }
      if (tiles * c <= 3 * (int64_t)num_sms() && fits_three(P.bn, terms, c, P.nkt, true) &&
          tiles <= active_clusters_dispatch(P.bn, terms, (int)c, 3)) {
        ks = c;
        three_per_sm = true;
        break;
      }
    }
  }
  P.ks = (int)ks;
  P.rows_max = (int)cdiv(BM, ks);
  // three CTAs to an SM whenever the grid outgrows two per SM and no cluster reduction buffer is
  // needed: partial planes, or a single split (the grouped MoE GEMM)
  if (!three_per_sm)
    three_per_sm = (parts || ks == 1) && tiles * ks > 2 * (int64_t)num_sms() && fits_three(P.bn, terms, ks, P.nkt);
  uint32_t cols = 0;
  stages_dispatch(P.bn, terms, parts ? 1 : P.ks, P.rows_max, (int)cdiv(P.nkt, ks), P.stages, cols, P.smem,
                  three_per_sm ? 3 : 2);
  if (P.stages < 2) return ADA_ERR_UNSUPPORTED;
  P.tmem_cols = (int)cols;
  P.persistent = false;
  P.p_stages = 0;
  if (!parts && ks == 1 && tiles > 2 * (int64_t)num_sms()) {
    uint32_t pc = 0;
#define ADA_PS(B, TT) if (P.bn == B && terms == TT) persistent_stages_for<B, TT>(P.p_stages, pc, P.p_smem);
    ADA_FP4_CONFIGS(ADA_PS)
#undef ADA_PS
    P.p_cols = (int)pc;
    P.persistent = P.p_stages >= 2;
  }
  size_t off = ERR_BYTES;
  P.off_xq = off;
  off = al256(off + (size_t)terms * P.m_pad * (size_t)(k / 2));
  P.off_sfx = off;
  if (terms == 1) off = al256(off + (size_t)P.m_tiles * (size_t)(k / 64) * 512);
  P.off_gx = off;
  off = al256(off + (size_t)P.m_pad * 4);
  P.total = off;
  return ADA_OK;
}

// ---- CTA-pair launch ------------------------------------------------------------------
static std::atomic<bool> g_pair_gemm{true};  // ada_set_pair_gemm

static inline bool a16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// Scale-factor bytes as rows of 128 bytes (a 2 KiB chunk = one box of 16 rows), no swizzle.
static bool make_sf_map(CUtensorMap* map, const void* base, uint64_t bytes) {
  if (!a16(base) || bytes % 2048) return false;
  const cuuint64_t dims[2] = {128, bytes / 128};
  const cuuint64_t strides[1] = {128};
  const cuuint32_t box[2] = {128, 16};
  return encode_bytes(map, base, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Pairs of CTAs that are resident at once (one CTA per SM; 0 if the query fails).
static int pair_capacity() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const int known = cache[dev].load(std::memory_order_relaxed);
  if (known) return known > 0 ? known : 0;
  int n = 0;
  if (cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pair::SMEM) ==
      cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(pair::THREADS, 1, 1);
    cfg.dynamicSmemBytes = pair::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel, &cfg) != cudaSuccess) n = 0;
  }
  (void)cudaGetLastError();
  cache[dev] = n > 0 ? n : -1;
  return n;
}

// The pair kernel covers the dense W4A4 GEMM with 256-row weight tiles and 16-byte output rows;
// everything else (row-scaled terms, grouped, tensor-parallel, partial planes) stays on the
// one-CTA kernels.
static bool pair_eligible(const GemmParams& gp) {
  return g_pair_gemm && !gp.part && !gp.tile_expert && !gp.row_map && gp.world <= 1 && gp.sfx && gp.N % pair::BW == 0 &&
         gp.ldy % 8 == 0 && a16(gp.y) && (!gp.bias || a16(gp.bias)) && gp.nkt >= 1;
}

// Launches the pair kernel; returns ADA_ERR_UNSUPPORTED (nothing launched) when its maps or
// residency cannot be had, so the caller falls back to the one-CTA persistent kernel.
static int launch_pair(const CUtensorMap& tmw, const CUtensorMap& tmx, const GemmParams& gp, const Plan& P,
                       cudaStream_t st) {
  CUtensorMap tsw, tsx;
  if (!make_sf_map(&tsw, gp.sfw, (uint64_t)gp.N * (uint64_t)gp.K / 16)) return ADA_ERR_UNSUPPORTED;
  if (!make_sf_map(&tsx, gp.sfx, (uint64_t)P.m_tiles * (uint64_t)(gp.K / 64) * 512)) return ADA_ERR_UNSUPPORTED;
  const int cap = pair_capacity();
  if (cap < 1) return ADA_ERR_UNSUPPORTED;
  const int64_t tiles = (int64_t)(gp.N / pair::BW) * cdiv(gp.M, pair::BT);
  const int64_t pairs = tiles < cap ? tiles : cap;
  (void)ada::launch_kc(gemm_pair_kernel, dim3((unsigned)(2 * pairs)), dim3(pair::THREADS), pair::SMEM, st, 2, tmw,
                       tmx, tsw, tsx, gp);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

template <int BN, int T>
static int launch_gemm(const CUtensorMap& tmw, const CUtensorMap& tmx, const GemmParams& gp, const Plan& P,
                       cudaStream_t st) {
  if constexpr (BN == 128 && T == 1) {
    if (P.persistent && pair_eligible(gp)) {
      const int rc = launch_pair(tmw, tmx, gp, P, st);
      if (rc != ADA_ERR_UNSUPPORTED) return rc;
    }
  }
  if (P.persistent && !gp.part) {  // prefill-size dense GEMM, or the grouped MoE GEMM
    static std::atomic<size_t> configured[64];
    static std::mutex raise;  // raises only: concurrent callers must not lower the limit
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ADA_ERR_CUDA;
    if (P.p_smem > configured[dev].load(std::memory_order_acquire)) {
      std::lock_guard<std::mutex> hold(raise);
      if (P.p_smem > configured[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(gemm_persistent_kernel<BN, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)P.p_smem) != cudaSuccess)
          return ADA_ERR_CUDA;
        configured[dev].store(P.p_smem, std::memory_order_release);
      }
    }
    GemmParams pp = gp;
    pp.stages = P.p_stages;
    pp.tmem_cols = P.p_cols;
    const int64_t tiles = (int64_t)P.n_tiles * P.m_tiles;
    const unsigned grid = (unsigned)(tiles < num_sms() ? tiles : num_sms());
    (void)ada::launch_k(gemm_persistent_kernel<BN, T>, dim3(grid), dim3(192), P.p_smem, st, tmw, tmx, pp);
    ADA_CHECK_LAUNCH();
    return ADA_OK;
  }
  auto kern = gemm_kernel<BN, T>;
  if (!ensure_smem<BN, T>(P.smem)) return ADA_ERR_CUDA;
  const dim3 grid((unsigned)P.ks, (unsigned)(P.n_tiles * P.m_tiles));
  if (P.ks > 1 && !gp.part)
    (void)ada::launch_kc(kern, grid, dim3(192), P.smem, st, P.ks, tmw, tmx, gp);
  else
    (void)ada::launch_k(kern, grid, dim3(192), P.smem, st, tmw, tmx, gp);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}

static int dispatch_gemm(const CUtensorMap& tmw, const CUtensorMap& tmx, const GemmParams& gp, const Plan& P,
                         cudaStream_t st) {
#define ADA_G(B, TT) if (P.bn == B && P.terms == TT) return launch_gemm<B, TT>(tmw, tmx, gp, P, st);
  ADA_FP4_CONFIGS(ADA_G)
#undef ADA_G
  return ADA_ERR_UNSUPPORTED;
}

static int run_gemm(const Plan& P, const uint8_t* xq, const uint8_t* sfx, const float* gx, int m, int n, int k,
                    const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w, const float* w_scale_2,
                    const void* bias, void* y, int y_dtype, int64_t ldy, unsigned int* err, cudaStream_t st,
                    float* part = nullptr, int64_t part_plane = 0, int64_t part_ld = 0, int world = 1, int tp_rank = 0,
                    unsigned long long* const* inboxes = nullptr, const unsigned int* epoch = nullptr,
                    unsigned int tag_mul = 0, unsigned int tag_add = 0, const int* tile_expert = nullptr,
                    const int* row_map = nullptr, int64_t w_rows = 0, const uint8_t* const* pf = nullptr,
                    const int64_t* pf_bytes = nullptr) {
  CUtensorMap tmw, tmx;
  if (!make_map(&tmw, w_packed, (uint64_t)(k / 2), (uint64_t)(w_rows ? w_rows : n), (uint64_t)ldw, BM))
    return ADA_ERR_CUDA;
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
  gp.err = err;
  gp.part = part;
  gp.part_plane = part_plane;
  gp.part_ld = (int)part_ld;
  gp.M = m;
  gp.N = n;
  gp.K = k;
  gp.ldy = (int)ldy;
  gp.n_tiles = P.n_tiles;
  gp.nkt = P.nkt;
  gp.stages = P.stages;
  gp.tmem_cols = P.tmem_cols;
  gp.out_dtype = y_dtype;
  gp.ks = P.ks;
  gp.rows_max = P.rows_max;
  gp.world = world;
  gp.tp_rank = tp_rank;
  for (int d = 0; d < MAX_PEERS; ++d) gp.inbox[d] = d < world && inboxes ? inboxes[d] : nullptr;
  gp.epoch = epoch;
  gp.tag_mul = tag_mul;
  gp.tag_add = tag_add;
  gp.tile_expert = tile_expert;
  gp.row_map = row_map;
  gp.m_tiles_max = P.m_tiles;
  for (int r = 0; r < 2; ++r) {
    gp.pf[r] = pf ? pf[r] : nullptr;
    gp.pf_bytes[r] = pf && pf[r] ? pf_bytes[r] : 0;
  }
  return dispatch_gemm(tmw, tmx, gp, P, st);
}

// ---- grouped (MoE) GEMM routing ------------------------------------------------------
// One CTA: rows are counted per expert, every expert gets whole 16-row operand tiles (a prefix
// sum over experts), tile_expert[t] names the expert of tile t (-1: unused), row_map[s] the
// input row of operand row s (-1: padding).  Rows keep no particular order inside an expert:
// each output row depends on its own input row only.  An expert id outside [0, experts) sets
// the workspace error word (its row is not computed).
constexpr int GROUP_BN = 16;
constexpr unsigned int ERR_EXPERT_ID = 0x60;

// Expert parallelism: ids in [expert_base, expert_base + experts) are this rank's experts (local
// index id - expert_base); with strict == 0 every other id is another rank's and its row is
// skipped (output row untouched), with strict == 1 it is an error.
// dest[r]: the operand row of input row r (-1: another rank's expert), for the gathering quantiser.
__global__ void __launch_bounds__(1024) route_kernel(const int32_t* __restrict__ ids, int m, int experts, int t_max,
                                                     int* tile_expert, int* row_map, int* dest, unsigned int* err,
                                                     int expert_base, int strict) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int route_smem[];
  int* cnt = route_smem;        // rows per expert
  int* base = cnt + experts;    // first tile of the expert
  int* fill = base + experts;   // rows placed so far
  for (int e = threadIdx.x; e < experts; e += blockDim.x) cnt[e] = fill[e] = 0;
  for (int t = threadIdx.x; t < t_max; t += blockDim.x) tile_expert[t] = -1;
  for (int r = threadIdx.x; r < t_max * GROUP_BN; r += blockDim.x) row_map[r] = -1;
  __syncthreads();
  for (int r = threadIdx.x; r < m; r += blockDim.x) {
    const int e = __ldg(ids + r) - expert_base;
    if (e >= 0 && e < experts)
      atomicAdd(&cnt[e], 1);
    else if (strict)
      atomicOr(err, ERR_EXPERT_ID);
  }
  __syncthreads();
  {  // tiles per expert, exclusive prefix sum: each thread sums a run of up to 4 experts, then a
     // scan over the warps' totals (experts <= 4096 = 4 x 1024 threads)
    __shared__ int warp_tot[32];
    const int per = (experts + 1023) / 1024;
    const int e0 = threadIdx.x * per;
    int local = 0;
    for (int e = e0; e < e0 + per && e < experts; ++e) local += (cnt[e] + GROUP_BN - 1) / GROUP_BN;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int inc = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    if (lane == 31) warp_tot[wid] = inc;
    __syncthreads();
    if (wid == 0) {
      int t = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += v;
      }
      warp_tot[lane] = t;  // inclusive totals of warps 0..lane
    }
    __syncthreads();
    int run = inc - local + (wid > 0 ? warp_tot[wid - 1] : 0);
    for (int e = e0; e < e0 + per && e < experts; ++e) {
      base[e] = run;
      run += (cnt[e] + GROUP_BN - 1) / GROUP_BN;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < experts; e += blockDim.x)
    for (int t = 0; t < (cnt[e] + GROUP_BN - 1) / GROUP_BN; ++t) tile_expert[base[e] + t] = e;
  for (int r = threadIdx.x; r < m; r += blockDim.x) {
    const int e = __ldg(ids + r) - expert_base;
    if (e < 0 || e >= experts) {
      dest[r] = -1;
      continue;
    }
    const int pos = base[e] * GROUP_BN + atomicAdd(&fill[e], 1);
    row_map[pos] = r;
    dest[r] = pos;
  }
}

// Operand tiles a grouped call can need: every expert's partial tile plus the full ones.
inline int64_t group_tiles(int64_t m, int64_t experts) { return cdiv(m, GROUP_BN) + (experts < m ? experts : m); }

}  // namespace fp4

namespace fused {
int launch_act_quant(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t m_pad, const q::QuantDst& dst,
                     cudaStream_t st, const int* dest, int row_div);
int gated_act_quant_impl(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t rows, int32_t inter, int act,
                         int dtype, int terms, int block_n, uint8_t* xq, uint8_t* sfx, float* gx, void* stream,
                         const PartIn& pin, const int* dest);
}
}  // namespace ada

using namespace ada;

extern "C" int ada_set_pair_gemm(int enable) {
  const int prev = fp4::g_pair_gemm.exchange(enable != 0) ? 1 : 0;
  return prev;
}

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
  (void)ada::launch_k(fp4::prepack_kernel, dim3((unsigned)blocks), dim3(128), 0,
                      reinterpret_cast<cudaStream_t>(stream), scale, scale_is_fp16, ld_scale, (int)n, (int)k, sf_out);
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
  if (ldx < k || ldy < n || ldw < k / 2 || force_ksplit < 0) return ADA_ERR_INVALID_ARG;
  fp4::Plan P;
  int rc = fp4::make_plan(m, n, k, terms, force_ksplit, P);
  if (rc != ADA_OK) return rc;
  if (workspace_bytes < P.total) return ADA_ERR_WORKSPACE;
  if (((uintptr_t)x & 15) || (ldx & 7) || ((uintptr_t)w_packed & 15) || (ldw & 15) || ((uintptr_t)sf_w & 15) ||
      ((uintptr_t)workspace & 255))
    return ADA_ERR_ALIGNMENT;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const q::QuantDst dst{ws + P.off_xq, ws + P.off_sfx, reinterpret_cast<float*>(ws + P.off_gx), terms, P.bn, (int)k};
  rc = fused::launch_act_quant(x, x_dtype, ldx, m, P.m_pad, dst, st, nullptr, 1);
  if (rc != ADA_OK) return rc;
  return fp4::run_gemm(P, dst.xq, dst.sfx, dst.gx, (int)m, (int)n, (int)k, w_packed, ldw, sf_w, w_scale_2, bias, y,
                       y_dtype, ldy, reinterpret_cast<unsigned int*>(ws), st);
}

// Grouped plan: 16-row operand tiles, one per (expert, 16 rows), no K split.
static int grouped_plan(int64_t m, int64_t n, int64_t k, int terms, int64_t experts, fp4::Plan& P, size_t& off_route,
                        size_t& total) {
  if (m <= 0 || experts <= 0 || experts > 4096) return ADA_ERR_INVALID_ARG;
  if (terms * fp4::GROUP_BN > 128) return ADA_ERR_UNSUPPORTED;
  const int64_t t_max = fp4::group_tiles(m, experts);
  const int rc = fp4::make_plan(t_max * fp4::GROUP_BN, n, k, terms, 1, P, false, fp4::GROUP_BN);
  if (rc != ADA_OK) return rc;
  off_route = (P.total + 255) & ~(size_t)255;
  total = off_route + (size_t)(1 + t_max + t_max * fp4::GROUP_BN + m) * sizeof(int);
  return ADA_OK;
}

extern "C" size_t ada_nvfp4_linear_grouped_workspace_size(int64_t m, int64_t n, int64_t k, int terms,
                                                          int32_t num_experts) {
  fp4::Plan P;
  size_t off = 0, total = 0;
  return grouped_plan(m, n, k, terms, num_experts, P, off, total) == ADA_OK ? total : 0;
}

static int linear_grouped_impl(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k,
                               const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w, const float* w_scale_2,
                               int32_t num_experts, int64_t n, const int32_t* expert_ids, void* y, int y_dtype,
                               int64_t ldy, int terms, void* workspace, size_t workspace_bytes, void* stream,
                               int32_t expert_base, int strict) {
  if (m == 0) return ADA_OK;
  if (!x || !w_packed || !sf_w || !w_scale_2 || !expert_ids || !y || !workspace) return ADA_ERR_INVALID_ARG;
  if ((x_dtype != ADA_DT_BF16 && x_dtype != ADA_DT_F16) || (y_dtype != ADA_DT_BF16 && y_dtype != ADA_DT_F16))
    return ADA_ERR_INVALID_ARG;
  if (ldx < k || ldy < n || ldw < k / 2) return ADA_ERR_INVALID_ARG;
  if ((int64_t)num_experts * n > (1 << 24)) return ADA_ERR_UNSUPPORTED;
  fp4::Plan P;
  size_t off_route = 0, total = 0;
  int rc = grouped_plan(m, n, k, terms, num_experts, P, off_route, total);
  if (rc != ADA_OK) return rc;
  if (workspace_bytes < total) return ADA_ERR_WORKSPACE;
  if (((uintptr_t)x & 15) || (ldx & 7) || ((uintptr_t)w_packed & 15) || (ldw & 15) || ((uintptr_t)sf_w & 15) ||
      ((uintptr_t)workspace & 255) || ((uintptr_t)expert_ids & 3))
    return ADA_ERR_ALIGNMENT;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int t_max = P.m_tiles;
  int* tile_expert = reinterpret_cast<int*>(ws + off_route) + 1;
  int* row_map = tile_expert + t_max;
  int* dest = row_map + t_max * fp4::GROUP_BN;
  unsigned int* err = reinterpret_cast<unsigned int*>(ws);
  const size_t rsmem = (size_t)3 * num_experts * sizeof(int);
  if (rsmem > 48 * 1024 &&
      cudaFuncSetAttribute(fp4::route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsmem) != cudaSuccess)
    return ADA_ERR_CUDA;
  (void)launch_k(fp4::route_kernel, dim3(1), dim3(1024), rsmem, st, expert_ids, (int)m, (int)num_experts, t_max,
                 tile_expert, row_map, dest, err, (int)expert_base, strict);
  ADA_CHECK_LAUNCH();
  const q::QuantDst dst{ws + P.off_xq, ws + P.off_sfx, reinterpret_cast<float*>(ws + P.off_gx), terms, P.bn, (int)k};
  rc = fused::launch_act_quant(x, x_dtype, ldx, m, P.m_pad, dst, st, dest, 1);
  if (rc != ADA_OK) return rc;
  // the stacked weight matrix [num_experts * n, k / 2]: expert e's tile j is 128-row block e * (n / 128) + j
  return fp4::run_gemm(P, dst.xq, dst.sfx, dst.gx, (int)m, (int)n, (int)k, w_packed, ldw, sf_w, w_scale_2, nullptr, y,
                       y_dtype, ldy, err, st, nullptr, 0, 0, 1, 0, nullptr, nullptr, 0, 0, tile_expert, row_map,
                       (int64_t)num_experts * n);
}

extern "C" int ada_nvfp4_linear_grouped(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k,
                                        const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                                        const float* w_scale_2, int32_t num_experts, int64_t n,
                                        const int32_t* expert_ids, void* y, int y_dtype, int64_t ldy, int terms,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  return linear_grouped_impl(x, x_dtype, ldx, m, k, w_packed, ldw, sf_w, w_scale_2, num_experts, n, expert_ids, y,
                             y_dtype, ldy, terms, workspace, workspace_bytes, stream, 0, 1);
}

extern "C" int ada_nvfp4_linear_grouped_ep(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k,
                                           const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                                           const float* w_scale_2, int32_t num_experts, int32_t expert_base,
                                           int64_t n, const int32_t* expert_ids, void* y, int y_dtype, int64_t ldy,
                                           int terms, void* workspace, size_t workspace_bytes, void* stream) {
  if (expert_base < 0) return ADA_ERR_INVALID_ARG;
  return linear_grouped_impl(x, x_dtype, ldx, m, k, w_packed, ldw, sf_w, w_scale_2, num_experts, n, expert_ids, y,
                             y_dtype, ldy, terms, workspace, workspace_bytes, stream, expert_base, 0);
}

// ---- the expert MLP of a MoE block in one call ----------------------------------------
// Layout of its workspace (every region 256-byte aligned): [error word][routing: one int, tile
// experts, operand row map, destination of each input row][gate_up operand: codes, scales, row
// scales][gate_up output h, the model dtype][down operand: codes, scales, row scales].
struct ExpertsLayout {
  fp4::Plan gu, dn;
  size_t off_route, off_xq1, off_sfx1, off_gx1, off_h, off_xq2, off_sfx2, off_gx2, total;
};
static size_t al256z(size_t v) { return (v + 255) & ~(size_t)255; }
static int experts_layout(int64_t m, int64_t hidden, int64_t inter, int terms, int64_t experts, ExpertsLayout& L) {
  size_t o1 = 0, t1 = 0, o2 = 0, t2 = 0;
  int rc = grouped_plan(m, 2 * inter, hidden, terms, experts, L.gu, o1, t1);
  if (rc != ADA_OK) return rc;
  rc = grouped_plan(m, hidden, inter, terms, experts, L.dn, o2, t2);
  if (rc != ADA_OK) return rc;
  const int64_t t_max = L.gu.m_tiles, m_pad = L.gu.m_pad;
  size_t off = fp4::ERR_BYTES;
  L.off_route = off;
  off = al256z(off + (size_t)(1 + t_max + t_max * fp4::GROUP_BN + m) * sizeof(int));
  L.off_xq1 = off;
  off = al256z(off + (size_t)terms * m_pad * (size_t)(hidden / 2));
  L.off_sfx1 = off;
  if (terms == 1) off = al256z(off + (size_t)t_max * (size_t)(hidden / 64) * 512);
  L.off_gx1 = off;
  off = al256z(off + (size_t)m_pad * 4);
  L.off_h = off;
  off = al256z(off + (size_t)m * (size_t)(2 * inter) * 2);
  L.off_xq2 = off;
  off = al256z(off + (size_t)terms * m_pad * (size_t)(inter / 2));
  L.off_sfx2 = off;
  if (terms == 1) off = al256z(off + (size_t)t_max * (size_t)(inter / 64) * 512);
  L.off_gx2 = off;
  off = al256z(off + (size_t)m_pad * 4);
  L.total = off;
  return ADA_OK;
}

extern "C" size_t ada_moe_experts_workspace_size(int64_t tokens, int32_t topk, int64_t hidden, int64_t inter,
                                                 int terms, int32_t num_experts) {
  if (tokens <= 0 || topk <= 0) return 0;
  ExpertsLayout L;
  return experts_layout(tokens * topk, hidden, inter, terms, num_experts, L) == ADA_OK ? L.total : 0;
}

extern "C" int ada_moe_experts(const void* x, int x_dtype, int64_t ldx, int64_t tokens, int32_t topk,
                               const int32_t* expert_ids, int32_t num_experts, int32_t expert_base, int32_t all_local,
                               const uint8_t* w_gate_up, int64_t ld_gate_up, const uint8_t* sf_gate_up,
                               const float* scale2_gate_up, const uint8_t* w_down, int64_t ld_down,
                               const uint8_t* sf_down, const float* scale2_down, int64_t inter, int64_t hidden,
                               int act, void* y, int64_t ldy, int terms, void* workspace, size_t workspace_bytes,
                               void* stream) {
  if (tokens == 0) return ADA_OK;
  if (tokens < 0 || topk <= 0 || num_experts <= 0 || expert_base < 0 || (act != 0 && act != 1))
    return ADA_ERR_INVALID_ARG;
  if (!x || !expert_ids || !w_gate_up || !sf_gate_up || !scale2_gate_up || !w_down || !sf_down || !scale2_down || !y ||
      !workspace)
    return ADA_ERR_INVALID_ARG;
  if (x_dtype != ADA_DT_BF16 && x_dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (ldx < hidden || ldy < hidden || ld_gate_up < hidden / 2 || ld_down < inter / 2) return ADA_ERR_INVALID_ARG;
  if ((int64_t)num_experts * 2 * inter > (1 << 24) || tokens * topk > (1 << 24)) return ADA_ERR_UNSUPPORTED;
  const int64_t m = tokens * topk;
  ExpertsLayout L;
  int rc = experts_layout(m, hidden, inter, terms, num_experts, L);
  if (rc != ADA_OK) return rc;
  if (workspace_bytes < L.total) return ADA_ERR_WORKSPACE;
  if (((uintptr_t)x & 15) || (ldx & 7) || ((uintptr_t)y & 15) || (ldy & 7) || ((uintptr_t)w_gate_up & 15) ||
      (ld_gate_up & 15) || ((uintptr_t)w_down & 15) || (ld_down & 15) || ((uintptr_t)sf_gate_up & 15) ||
      ((uintptr_t)sf_down & 15) || ((uintptr_t)workspace & 255) || ((uintptr_t)expert_ids & 3))
    return ADA_ERR_ALIGNMENT;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned int* err = reinterpret_cast<unsigned int*>(ws);
  const int t_max = L.gu.m_tiles;
  int* tile_expert = reinterpret_cast<int*>(ws + L.off_route) + 1;
  int* row_map = tile_expert + t_max;
  int* dest = row_map + t_max * fp4::GROUP_BN;
  // one routing for both projections: 16-row tiles of each local expert's rows
  const size_t rsmem = (size_t)3 * num_experts * sizeof(int);
  if (rsmem > 48 * 1024 &&
      cudaFuncSetAttribute(fp4::route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsmem) != cudaSuccess)
    return ADA_ERR_CUDA;
  (void)launch_k(fp4::route_kernel, dim3(1), dim3(1024), rsmem, st, expert_ids, (int)m, (int)num_experts, t_max,
                 tile_expert, row_map, dest, err, (int)expert_base, all_local ? 1 : 0);
  ADA_CHECK_LAUNCH();
  // gate_up operand: routed row r reads token r / topk's row of x (the gather) and lands in its
  // expert's tile
  const q::QuantDst d1{ws + L.off_xq1, ws + L.off_sfx1, reinterpret_cast<float*>(ws + L.off_gx1), terms,
                       fp4::GROUP_BN, (int)hidden};
  rc = fused::launch_act_quant(x, x_dtype, ldx, m, L.gu.m_pad, d1, st, dest, topk);
  if (rc != ADA_OK) return rc;
  void* h = ws + L.off_h;
  rc = fp4::run_gemm(L.gu, d1.xq, d1.sfx, d1.gx, (int)m, (int)(2 * inter), (int)hidden, w_gate_up, ld_gate_up,
                     sf_gate_up, scale2_gate_up, nullptr, h, x_dtype, 2 * inter, err, st, nullptr, 0, 0, 1, 0, nullptr,
                     nullptr, 0, 0, tile_expert, row_map, (int64_t)num_experts * 2 * inter);
  if (rc != ADA_OK) return rc;
  // act(gate) * up of each routed row, quantised straight into the down projection's operand
  const q::QuantDst d2{ws + L.off_xq2, ws + L.off_sfx2, reinterpret_cast<float*>(ws + L.off_gx2), terms,
                       fp4::GROUP_BN, (int)inter};
  rc = fused::gated_act_quant_impl(h, 2 * inter, nullptr, 0, m, (int32_t)inter, act, x_dtype, terms, fp4::GROUP_BN,
                                   d2.xq, d2.sfx, d2.gx, stream, PartIn{nullptr, 0, 0, 0}, dest);
  if (rc != ADA_OK) return rc;
  return fp4::run_gemm(L.dn, d2.xq, d2.sfx, d2.gx, (int)m, (int)hidden, (int)inter, w_down, ld_down, sf_down,
                       scale2_down, nullptr, y, x_dtype, ldy, err, st, nullptr, 0, 0, 1, 0, nullptr, nullptr, 0, 0,
                       tile_expert, row_map, (int64_t)num_experts * hidden);
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
  if (m <= 0 || k <= 0 || !x || !xq || !gx) return ADA_ERR_INVALID_ARG;
  if (x_dtype != ADA_DT_BF16 && x_dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (ldx < k) return ADA_ERR_INVALID_ARG;
  if (k % 256) return ADA_ERR_UNSUPPORTED;
  if (!q::dst_ok(terms, block_n, (int)k) || (terms == 1 && !sfx)) return ADA_ERR_INVALID_ARG;
  if (((uintptr_t)x & 15) || (ldx & 7) || ((uintptr_t)xq & 15) || ((uintptr_t)gx & 3)) return ADA_ERR_ALIGNMENT;
  const int64_t m_pad = cdiv(m, block_n) * block_n;
  const q::QuantDst dst{xq, sfx, gx, terms, block_n, (int)k};
  return fused::launch_act_quant(x, x_dtype, ldx, m, m_pad, dst, reinterpret_cast<cudaStream_t>(stream), nullptr, 1);
}

extern "C" int ada_nvfp4_workspace_status(const void* workspace, int64_t m, int64_t n, int64_t k, int terms,
                                          unsigned int* status_out, void* stream) {
  (void)m;
  (void)n;
  (void)k;
  (void)terms;
  if (!workspace || !status_out) return ADA_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(status_out, workspace, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return ADA_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return ADA_ERR_CUDA;
  return ADA_OK;
}

extern "C" int ada_nvfp4_block_n(int64_t m, int terms) {
  if (m <= 0 || terms < 1 || terms > q::MAX_TERMS) return 0;
  return fp4::block_n_for(m, terms);
}

extern "C" size_t ada_nvfp4_gemm_workspace_size(int64_t m, int64_t n, int64_t k, int terms) {
  fp4::Plan P;
  if (fp4::make_plan(m, n, k, terms, 0, P) != ADA_OK) return 0;
  return fp4::ERR_BYTES;
}

extern "C" int ada_nvfp4_gemm(const uint8_t* xq, const uint8_t* sfx, const float* gx, int64_t m, int terms,
                              int block_n, const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                              const float* w_scale_2, int64_t n, int64_t k, const void* bias, void* y, int y_dtype,
                              int64_t ldy, int force_ksplit, void* workspace, size_t workspace_bytes, void* stream) {
  if (m == 0) return ADA_OK;
  if (!xq || !gx || !w_packed || !sf_w || !w_scale_2 || !y || !workspace) return ADA_ERR_INVALID_ARG;
  if (terms == 1 && !sfx) return ADA_ERR_INVALID_ARG;
  if (y_dtype != ADA_DT_BF16 && y_dtype != ADA_DT_F16) return ADA_ERR_INVALID_ARG;
  if (ldy < n || ldw < k / 2 || force_ksplit < 0) return ADA_ERR_INVALID_ARG;
  fp4::Plan P;
  int rc = fp4::make_plan(m, n, k, terms, force_ksplit, P);
  if (rc != ADA_OK) return rc;
  if (block_n != P.bn) return ADA_ERR_INVALID_ARG;
  if (workspace_bytes < fp4::ERR_BYTES) return ADA_ERR_WORKSPACE;
  if (((uintptr_t)xq & 15) || (sfx && ((uintptr_t)sfx & 15)) || ((uintptr_t)w_packed & 15) || (ldw & 15) ||
      ((uintptr_t)sf_w & 15) || ((uintptr_t)workspace & 255))
    return ADA_ERR_ALIGNMENT;
  return fp4::run_gemm(P, xq, sfx, gx, (int)m, (int)n, (int)k, w_packed, ldw, sf_w, w_scale_2, bias, y, y_dtype, ldy,
                       reinterpret_cast<unsigned int*>(workspace), reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ada_nvfp4_gemm_splits(int64_t m, int64_t n, int64_t k, int terms) {
  fp4::Plan P;
  if (fp4::make_plan(m, n, k, terms, 0, P, true) != ADA_OK) return 0;
  return P.ks;
}

static bool pf_ok(const void* p, size_t bytes) { return !p || (((uintptr_t)p & 15) == 0 && (bytes & 15) == 0); }

extern "C" int ada_nvfp4_gemm_partials_pf(const uint8_t* xq, const uint8_t* sfx, const float* gx, int64_t m,
                                          int terms, int block_n, const uint8_t* w_packed, int64_t ldw,
                                          const uint8_t* sf_w, const float* w_scale_2, int64_t n, int64_t k,
                                          float* parts, int64_t part_ld, int64_t part_plane, int nplanes,
                                          const void* next_w, size_t next_w_bytes, const void* next_sf,
                                          size_t next_sf_bytes, void* workspace, size_t workspace_bytes,
                                          void* stream) {
  if (m == 0) return ADA_OK;
  if (!xq || !gx || !w_packed || !sf_w || !w_scale_2 || !parts || !workspace) return ADA_ERR_INVALID_ARG;
  if (terms == 1 && !sfx) return ADA_ERR_INVALID_ARG;
  if (ldw < k / 2 || part_ld < n || part_plane < m * part_ld || nplanes < 1) return ADA_ERR_INVALID_ARG;
  if (part_ld > 0x7fffffff) return ADA_ERR_UNSUPPORTED;
  if (!pf_ok(next_w, next_w_bytes) || !pf_ok(next_sf, next_sf_bytes)) return ADA_ERR_ALIGNMENT;
  fp4::Plan P;
  int rc = fp4::make_plan(m, n, k, terms, nplanes, P, true);
  if (rc != ADA_OK) return rc;
  if (block_n != P.bn || P.ks != nplanes) return ADA_ERR_INVALID_ARG;
  if (workspace_bytes < fp4::ERR_BYTES) return ADA_ERR_WORKSPACE;
  if (((uintptr_t)xq & 15) || (sfx && ((uintptr_t)sfx & 15)) || ((uintptr_t)w_packed & 15) || (ldw & 15) ||
      ((uintptr_t)sf_w & 15) || ((uintptr_t)workspace & 255) || ((uintptr_t)parts & 3))
    return ADA_ERR_ALIGNMENT;
  const uint8_t* pf[2] = {reinterpret_cast<const uint8_t*>(next_w), reinterpret_cast<const uint8_t*>(next_sf)};
  const int64_t pfb[2] = {(int64_t)next_w_bytes, (int64_t)next_sf_bytes};
  return fp4::run_gemm(P, xq, sfx, gx, (int)m, (int)n, (int)k, w_packed, ldw, sf_w, w_scale_2, nullptr, nullptr,
                       ADA_DT_BF16, n, reinterpret_cast<unsigned int*>(workspace), reinterpret_cast<cudaStream_t>(stream),
                       parts, part_plane, part_ld, 1, 0, nullptr, nullptr, 0, 0, nullptr, nullptr, 0, pf, pfb);
}

extern "C" int ada_nvfp4_gemm_partials(const uint8_t* xq, const uint8_t* sfx, const float* gx, int64_t m, int terms,
                                       int block_n, const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                                       const float* w_scale_2, int64_t n, int64_t k, float* parts, int64_t part_ld,
                                       int64_t part_plane, int nplanes, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  if (m == 0) return ADA_OK;
  if (!xq || !gx || !w_packed || !sf_w || !w_scale_2 || !parts || !workspace) return ADA_ERR_INVALID_ARG;
  if (terms == 1 && !sfx) return ADA_ERR_INVALID_ARG;
  if (ldw < k / 2 || part_ld < n || part_plane < m * part_ld || nplanes < 1) return ADA_ERR_INVALID_ARG;
  if (part_ld > 0x7fffffff) return ADA_ERR_UNSUPPORTED;
  fp4::Plan P;
  int rc = fp4::make_plan(m, n, k, terms, nplanes, P, true);
  if (rc != ADA_OK) return rc;
  if (block_n != P.bn || P.ks != nplanes) return ADA_ERR_INVALID_ARG;
  if (workspace_bytes < fp4::ERR_BYTES) return ADA_ERR_WORKSPACE;
  if (((uintptr_t)xq & 15) || (sfx && ((uintptr_t)sfx & 15)) || ((uintptr_t)w_packed & 15) || (ldw & 15) ||
      ((uintptr_t)sf_w & 15) || ((uintptr_t)workspace & 255) || ((uintptr_t)parts & 3))
    return ADA_ERR_ALIGNMENT;
  return fp4::run_gemm(P, xq, sfx, gx, (int)m, (int)n, (int)k, w_packed, ldw, sf_w, w_scale_2, nullptr, nullptr,
                       ADA_DT_BF16, n, reinterpret_cast<unsigned int*>(workspace), reinterpret_cast<cudaStream_t>(stream),
                       parts, part_plane, part_ld);
}

extern "C" int ada_nvfp4_gemm_partials_peer(const uint8_t* xq, const uint8_t* sfx, const float* gx, int64_t m,
                                            int terms, int block_n, const uint8_t* w_packed, int64_t ldw,
                                            const uint8_t* sf_w, const float* w_scale_2, int64_t n, int64_t k,
                                            int64_t part_ld, int64_t part_plane, int nplanes, int32_t world,
                                            int32_t tp_rank, void* const* inboxes, const uint32_t* epoch,
                                            uint32_t tag_mul, uint32_t tag_add, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  if (m == 0) return ADA_OK;
  if (world < 2 || world > fp4::MAX_PEERS || tp_rank < 0 || tp_rank >= world || !inboxes || !epoch)
    return ADA_ERR_INVALID_ARG;
  for (int d = 0; d < world; ++d)
    if (!inboxes[d] || ((uintptr_t)inboxes[d] & 15)) return ADA_ERR_INVALID_ARG;
  if (((uintptr_t)epoch & 3)) return ADA_ERR_ALIGNMENT;
  if (!xq || !gx || !w_packed || !sf_w || !w_scale_2 || !workspace) return ADA_ERR_INVALID_ARG;
  if (terms == 1 && !sfx) return ADA_ERR_INVALID_ARG;
  if (ldw < k / 2 || part_ld < n || part_plane < m * part_ld || nplanes < 1) return ADA_ERR_INVALID_ARG;
  if (part_ld > 0x7fffffff) return ADA_ERR_UNSUPPORTED;
  fp4::Plan P;
  int rc = fp4::make_plan(m, n, k, terms, nplanes, P, true);
  if (rc != ADA_OK) return rc;
  if (block_n != P.bn || P.ks != nplanes) return ADA_ERR_INVALID_ARG;
  if (workspace_bytes < fp4::ERR_BYTES) return ADA_ERR_WORKSPACE;
  if (((uintptr_t)xq & 15) || (sfx && ((uintptr_t)sfx & 15)) || ((uintptr_t)w_packed & 15) || (ldw & 15) ||
      ((uintptr_t)sf_w & 15) || ((uintptr_t)workspace & 255))
    return ADA_ERR_ALIGNMENT;
  unsigned long long* boxes[fp4::MAX_PEERS];
  for (int d = 0; d < world; ++d) boxes[d] = reinterpret_cast<unsigned long long*>(inboxes[d]);
  return fp4::run_gemm(P, xq, sfx, gx, (int)m, (int)n, (int)k, w_packed, ldw, sf_w, w_scale_2, nullptr, nullptr,
                       ADA_DT_BF16, n, reinterpret_cast<unsigned int*>(workspace), reinterpret_cast<cudaStream_t>(stream),
                       reinterpret_cast<float*>(boxes[tp_rank]), part_plane, part_ld, world, tp_rank, boxes, epoch,
                       tag_mul, tag_add);
}

extern "C" int ada_nvfp4_gemm_ctas(int64_t m, int64_t n, int64_t k, int terms, int nplanes) {
  fp4::Plan P;
  if (fp4::make_plan(m, n, k, terms, nplanes, P, true) != ADA_OK) return -1;
  return P.ks * P.n_tiles * P.m_tiles;
}
