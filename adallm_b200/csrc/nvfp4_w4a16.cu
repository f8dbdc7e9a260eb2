// NVFP4 linear with the reference's W4A16 arithmetic at prefill size, on SM pairs.
//
// The reference's nvfp4_linear (adallm/ops/nvfp4_gemm.py:58-136, :460-564) dequantises the e2m1
// weights to fp16 (lut[code] * block scale * global scale) and multiplies them with the
// activations cast to fp16, accumulating in fp32.  At prefill size this is a tensor-core problem,
// and the block-scaled FP4 MMA (gemm_kernel / gemm_pair_kernel) needs the activations quantised
// to e2m1 terms; here the activations stay fp16 and the weights are widened instead:
//
//   * the activations (cast to fp16 once when they arrive as bf16, as the reference casts them)
//     are the MMA's A operand: 256 token rows per CTA pair, 128 staged by each CTA (TMA, 128-byte
//     swizzle);
//   * each CTA stages the packed e2m1 bytes and e4m3 block scales of its 128 of the tile's 256
//     weight rows (TMA + bulk copy), and converter warps widen them in shared memory to fp16
//     (lut[code] * block scale is exact in fp16) in the swizzled K-major layout the MMA reads;
//   * one tcgen05.mma.cta_group::2.kind::f16 of M 256 x N 256 x K 16 per 16-wide K step, fp32
//     accumulators in TMEM, two of them (2 x 256 columns) so the epilogue of tile i overlaps the
//     MMAs of tile i + 1; the epilogue multiplies by the global scale (fp32, not rounded into the
//     weights as the reference's fp16 dequantisation does), adds the bias and stores 16-byte rows.
//
// Protocol (CTA rank 0 of the pair leads; no multicast anywhere):
//   full[s]  (each):   this CTA's activation, packed-weight and scale loads of stage s landed.
//   ready[s] (rank 0): one converter group of each CTA wrote stage s's fp16 weights (8 arrivals).
//   empty[s] (each):   the leader's MMA thread commits to both CTAs once stage s is read.
//   accf[b]  (each):   accumulator b complete (committed to both CTAs).
//   acce[b]  (rank 0): accumulator b drained by the 8 epilogue warps of both CTAs (16 arrivals).
// Every wait is bounded (2 s); a timeout sets an error bit in the workspace and the CTA drains
// and exits.
#include "cluster.cuh"
#include "sm100.cuh"

namespace ada {
namespace w16 {

using namespace sm100;

constexpr int BT = 256;                        // tokens per tile (MMA M, 128 per CTA)
constexpr int BW = 256;                        // weight rows per tile (MMA N, 128 per CTA)
constexpr int KS = 64;                         // K elements per stage
constexpr uint32_t A_BYTES = 128 * KS * 2;     // this CTA's token rows, fp16, swizzled (16 KiB)
constexpr uint32_t B_BYTES = 128 * KS * 2;     // this CTA's weight rows widened to fp16 (16 KiB)
constexpr uint32_t W_BYTES = 128 * KS / 2;     // their packed e2m1 bytes (4 KiB)
constexpr uint32_t S_BYTES = 512;              // their e4m3 scales of this 64-wide K block
constexpr uint32_t LOAD_BYTES = A_BYTES + W_BYTES + S_BYTES;
constexpr uint32_t STAGE = 38 * 1024;          // A | B | W | S, padded to keep A and B 1 KiB aligned
constexpr int STAGES = 5;
constexpr uint32_t TMEM_COLS = 512;            // two 256-column accumulators
#ifndef ADA_W16_CONV_GROUPS
#define ADA_W16_CONV_GROUPS 2
#endif
constexpr int CONV_GROUPS = ADA_W16_CONV_GROUPS;  // converter groups taking the stages in turn
constexpr int CONV_WARPS = 4 * CONV_GROUPS;       // four warps (one thread per weight row) a group
constexpr int EPI_WARPS = 8;                   // two per TMEM lane quarter, 128 columns each
constexpr int EPI_WARP0 = 2 + CONV_WARPS;
constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE + 1024;
constexpr uint32_t ERR_EMPTY = 1u, ERR_READY = 2u, ERR_ACCF = 4u, ERR_ACCE = 8u, ERR_FULL = 0x80u;
static_assert(A_BYTES + B_BYTES + W_BYTES + S_BYTES <= STAGE && STAGE % 1024 == 0, "stage layout");
static_assert(SMEM <= 232448, "shared memory per CTA");
// kind::f16: fp32 D (bit 4), fp16 A and B (formats 0), both K-major, N 256, M 256
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BW >> 3) << 17) | ((uint32_t)(BT >> 4) << 24);

struct Params {
  const uint8_t* sfw;  // prepacked scales [N/128][K/64][512]
  const float* gw;     // global weight scale (device scalar)
  const void* bias;    // [N] (out dtype) or null
  void* y;             // [M, ldy]
  unsigned int* err;
  int M, N, K, ldy, out_dtype;
};

__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %3, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %4, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(accumulate), "r"(IDESC)
      : "memory");
}

// Eight e2m1 codes (element 0 in the low nibble) -> their values as four f16x2 (low half = even
// element), one conversion instruction per code pair.
__device__ __forceinline__ void e2m1x8_to_f16x8_cvt(uint32_t codes, uint32_t* h) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(codes));
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_w4a16_pair_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                           const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ctrl = smem + (size_t)STAGES * STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
  uint64_t* ready = full + STAGES;
  uint64_t* empty = ready + STAGES;
  uint64_t* accf = empty + STAGES;  // [2]
  uint64_t* acce = accf + 2;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_v = abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cl::ctarank() & 1u, peer = rank ^ 1u;
  const int w_pairs = p.N / BW;
  const int tiles = w_pairs * ((p.M + BT - 1) / BT);
  const int pair_id = (int)(blockIdx.x >> 1), pairs = (int)(gridDim.x >> 1);
  const int kb64 = p.K / 64;
  const int nks = p.K / KS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 2 * 4);  // one group's four warps in each CTA
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 2 * EPI_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmx);
    prefetch_tmap(&tmw);
  }
  tc_fence_before();
  cl::cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any pair traffic
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---------------- producer (both CTAs) ----------------
      pdl_wait();
      uint32_t it = 0;
      for (int t = pair_id; t < tiles && !*abort_v; t += pairs) {
        const int wp = t % w_pairs, tt = t / w_pairs;
        const int x_row = tt * BT + (int)rank * 128;
        const int w_blk = wp * 2 + (int)rank;  // this CTA's 128-row weight block
        for (int kt = 0; kt < nks; ++kt, ++it) {
          const int s = (int)(it % (uint32_t)STAGES);
          if (it >= (uint32_t)STAGES &&
              !mbar_wait_bounded(&empty[s], ((it / STAGES) & 1) ^ 1, abort_v, p.err, ERR_EMPTY))
            break;
          uint8_t* st = smem + (size_t)s * STAGE;
          mbar_arrive_expect_tx(&full[s], LOAD_BYTES);
          tma_load_2d(st, &tmx, &full[s], kt * KS * 2, x_row);
          tma_load_2d(st + A_BYTES + B_BYTES, &tmw, &full[s], kt * (KS / 2), w_blk * 128);
          bulk_load(st + A_BYTES + B_BYTES + W_BYTES, p.sfw + ((size_t)w_blk * kb64 + kt) * 512, S_BYTES, &full[s]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {  // ---------------- MMA issuer (leader CTA only) ----------------
      const uint32_t empty0_own = cl::mapa(&empty[0], 0), empty0_peer = cl::mapa(&empty[0], peer);
      const uint32_t accf0_own = cl::mapa(&accf[0], 0), accf0_peer = cl::mapa(&accf[0], peer);
      uint32_t it = 0, lt = 0;
      for (int t = pair_id; t < tiles && !*abort_v; t += pairs, ++lt) {
        const uint32_t b = lt & 1, use = lt >> 1;
        if (use > 0 && !mbar_wait_bounded_cluster(&acce[b], (use - 1) & 1, abort_v, p.err, ERR_ACCE)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * (uint32_t)BW;
        bool failed = false;
        for (int kt = 0; kt < nks; ++kt, ++it) {
          const int s = (int)(it % (uint32_t)STAGES);
          if (!mbar_wait_bounded_cluster(&ready[s], (it / STAGES) & 1, abort_v, p.err, ERR_READY)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + (size_t)s * STAGE);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < KS / 16; ++kk)
            mma_f16_pair(acc, desc_kmajor_sw128(a_addr + kk * 32), desc_kmajor_sw128(b_addr + kk * 32),
                         (kt | kk) != 0);
          tc_commit_pair(empty0_own + (uint32_t)s * 8u);
          tc_commit_pair(empty0_peer + (uint32_t)s * 8u);
        }
        tc_commit_pair(accf0_own + b * 8u);  // also after a failure: drains the issued MMAs
        tc_commit_pair(accf0_peer + b * 8u);
        if (failed) break;
      }
    }
    __syncwarp();
  } else if (warp < EPI_WARP0) {  // ---------------- converters (both CTAs) ----------------
    // CONV_GROUPS groups of four warps take the stages in turn (group g the stages it with
    // it % CONV_GROUPS == g), so one group's wait, fence and arrive overlap the next group's work.
    // Thread r of a group widens weight row r of this CTA's 128: 64 e2m1 codes x their 4 block
    // scales -> 64 fp16 values, the row's eight 16-byte chunks in the swizzled K-major tile
    // (chunk c of row r at 16 * (c ^ (r % 8)) within the row's 128 bytes; 8-row atoms 1 KiB apart)
    const int i = threadIdx.x - 64;
    const int r = i & 127, grp = i >> 7;
    const uint32_t ready0_lead = cl::mapa(&ready[0], 0);
    uint32_t it = 0;
    bool ok = true;
    for (int t = pair_id; t < tiles && ok; t += pairs) {
      for (int kt = 0; kt < nks; ++kt, ++it) {
        if ((int)(it % (uint32_t)CONV_GROUPS) != grp) continue;
        const int s = (int)(it % (uint32_t)STAGES);
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (it / STAGES) & 1, abort_v, p.err, ERR_FULL))) {
          ok = false;
          break;
        }
        uint8_t* st = smem + (size_t)s * STAGE;
        const uint4* wrow = reinterpret_cast<const uint4*>(st + A_BYTES + B_BYTES + r * (KS / 2));
        const uint4 w0 = wrow[0], w1 = wrow[1];
        const uint32_t sc = *reinterpret_cast<const uint32_t*>(st + A_BYTES + B_BYTES + W_BYTES + (r & 31) * 16 +
                                                               (r >> 5) * 4);
        const uint32_t s01 = e4m3x2_to_f16x2((uint16_t)(sc & 0xFFFFu)), s23 = e4m3x2_to_f16x2((uint16_t)(sc >> 16));
        const __half2 sh[4] = {__half2half2(__low2half(*reinterpret_cast<const __half2*>(&s01))),
                               __half2half2(__high2half(*reinterpret_cast<const __half2*>(&s01))),
                               __half2half2(__low2half(*reinterpret_cast<const __half2*>(&s23))),
                               __half2half2(__high2half(*reinterpret_cast<const __half2*>(&s23)))};
        const uint32_t codes[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint8_t* brow = st + A_BYTES + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t h[4];
          e2m1x8_to_f16x8_cvt(codes[c], h);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __half2 v = __hmul2(*reinterpret_cast<const __half2*>(&h[j]), sh[c >> 1]);
            h[j] = *reinterpret_cast<const uint32_t*>(&v);
          }
          *reinterpret_cast<uint4*>(brow + ((c ^ (r & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
        }
        // the tile stays in this CTA's shared memory, where this CTA's half of the pair MMA reads
        // it: the async-proxy fence and a CTA-scope release order the writes before the arrival
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive_remote_cta(ready0_lead + (uint32_t)s * 8u);
      }
    }
    __syncwarp();
  } else {  // ---------------- epilogue (8 warps, both CTAs) ----------------
    pdl_wait();
    pdl_trigger();
    const int q = warp & 3;                   // TMEM lane quarter this warp may read
    const int h = (warp - EPI_WARP0) >> 2;    // column half: weight rows h*128 .. +127 of the tile
    const uint32_t acce0_lead = cl::mapa(&acce[0], 0);
    const float gw = __ldg(p.gw);
    const bool bf16 = p.out_dtype == ADA_DT_BF16;
    uint32_t lt = 0;
    for (int t = pair_id; t < tiles; t += pairs, ++lt) {
      const int wp = t % w_pairs, tt = t / w_pairs;
      const uint32_t b = lt & 1, use = lt >> 1;
      const int m = tt * BT + (int)rank * 128 + q * 32 + lane;
      const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&accf[b], use & 1, abort_v, p.err, ERR_ACCF) && !*abort_v);
      tc_fence_after();
      __syncwarp();
      const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + b * (uint32_t)BW + (uint32_t)h * 128;
      const int n0 = wp * BW + h * 128;
      const uint4* bias8 = p.bias ? reinterpret_cast<const uint4*>(p.bias) + n0 / 8 : nullptr;
      uint4* yrow = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.y) + (int64_t)m * p.ldy + n0);
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {  // 16 columns at a time
        uint32_t v[16];
        tmem_ld16_nowait(lane_addr + 16 * c, v);
        tmem_wait_ld();
        if (ok && m < p.M) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            float bb[8];
            if (bias8) {
              const uint4 u = __ldg(bias8 + 2 * c + g);
              if (bf16) unpack8<__nv_bfloat16>(u, bb); else unpack8<__half>(u, bb);
            } else {
#pragma unroll
              for (int k = 0; k < 8; ++k) bb[k] = 0.f;
            }
            float o[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) o[k] = fmaf(__uint_as_float(v[8 * g + k]), gw, 0.f) + bb[k];
            yrow[2 * c + g] = bf16 ? pack8<__nv_bfloat16>(o) : pack8<__half>(o);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce0_lead + b * 8u);  // accumulator b free for tile lt + 2
      if (!ok) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  cl::cluster_sync();  // neither CTA leaves while the pair's MMAs or arrivals may still reach it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, TMEM_COLS);
}

// bf16 activations -> fp16 rows (the reference's kernel casts its x tile to fp16,
// adallm/ops/nvfp4_gemm.py:100-105), 8 a thread.
__global__ void __launch_bounds__(256) to_f16_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int64_t m,
                                                     int64_t k, __half* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int64_t per_row = k / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m * per_row;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row, c = (i % per_row) * 8;
    float f[8];
    unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(x + r * ldx + c), f);
    *reinterpret_cast<uint4*>(out + r * k + c) = pack8<__half>(f);
  }
}

static bool make_map(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows, uint64_t stride,
                     uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
  const cuuint64_t dims[2] = {inner_bytes, rows};
  const cuuint64_t strides[1] = {stride};
  const cuuint32_t box[2] = {box_inner, box_rows};
  return encode_bytes(map, base, 2, dims, strides, box, swz);
}

static int pair_capacity() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const int known = cache[dev].load(std::memory_order_relaxed);
  if (known) return known > 0 ? known : 0;
  int n = 0;
  if (cudaFuncSetAttribute(gemm_w4a16_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM) ==
      cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_w4a16_pair_kernel, &cfg) != cudaSuccess) n = 0;
  }
  (void)cudaGetLastError();
  cache[dev] = n > 0 ? n : -1;
  return n;
}

}  // namespace w16
}  // namespace ada

using namespace ada;

static inline bool a16p(const void* p) { return ((uintptr_t)p & 15u) == 0; }

extern "C" size_t ada_nvfp4_linear_w4a16_workspace_size(int64_t m, int64_t k) {
  if (m <= 0 || k <= 0) return 0;
  return 256 + (size_t)m * (size_t)k * 2;
}

extern "C" int ada_nvfp4_linear_w4a16(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k,
                                      const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w, const float* w_scale_2,
                                      int64_t n, const void* bias, void* y, int y_dtype, int64_t ldy, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  if (m == 0) return ADA_OK;
  if (m < 0 || !x || !w_packed || !sf_w || !w_scale_2 || !y || !workspace) return ADA_ERR_INVALID_ARG;
  if ((x_dtype != ADA_DT_BF16 && x_dtype != ADA_DT_F16) || (y_dtype != ADA_DT_BF16 && y_dtype != ADA_DT_F16))
    return ADA_ERR_INVALID_ARG;
  if (ldx < k || ldy < n || ldw < k / 2) return ADA_ERR_INVALID_ARG;
  if (n % w16::BW || k % w16::KS || m > (1 << 24) || n > (1 << 24) || k > (1 << 24)) return ADA_ERR_UNSUPPORTED;
  // one pair may walk every tile: its K-step counter (uint32, stage parities modulo 5 stages)
  // and the tile index (int) must not wrap
  if ((n / w16::BW) * cdiv(m, (int64_t)w16::BT) * (k / w16::KS) >= (int64_t(1) << 31)) return ADA_ERR_UNSUPPORTED;
  if (workspace_bytes < ada_nvfp4_linear_w4a16_workspace_size(m, k)) return ADA_ERR_WORKSPACE;
  if (!a16p(x) || (ldx & 7) || !a16p(y) || (ldy & 7) || (bias && !a16p(bias)) || !a16p(w_packed) || (ldw & 15) ||
      !a16p(sf_w) || ((uintptr_t)workspace & 255))
    return ADA_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  const void* x16 = x;
  int64_t ld16 = ldx;
  if (x_dtype == ADA_DT_BF16) {  // the reference's x.to(fp16), into the workspace
    __half* out = reinterpret_cast<__half*>(ws + 256);
    const int64_t work = m * (k / 8);
    const unsigned blocks = (unsigned)std::min<int64_t>((work + 255) / 256, 148 * 16);
    (void)launch_k(w16::to_f16_kernel, dim3(blocks), dim3(256), 0, st, (const __nv_bfloat16*)x, ldx, m, k, out);
    ADA_CHECK_LAUNCH();
    x16 = out;
    ld16 = k;
  }
  CUtensorMap tmx, tmw;
  if (!w16::make_map(&tmx, x16, (uint64_t)k * 2, (uint64_t)m, (uint64_t)ld16 * 2, 128, 128,
                     CU_TENSOR_MAP_SWIZZLE_128B))
    return ADA_ERR_CUDA;
  if (!w16::make_map(&tmw, w_packed, (uint64_t)k / 2, (uint64_t)n, (uint64_t)ldw, w16::KS / 2, 128,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
    return ADA_ERR_CUDA;
  const int cap = w16::pair_capacity();
  if (cap < 1) return ADA_ERR_CUDA;
  w16::Params p;
  p.sfw = sf_w;
  p.gw = w_scale_2;
  p.bias = bias;
  p.y = y;
  p.err = reinterpret_cast<unsigned int*>(ws);
  p.M = (int)m;
  p.N = (int)n;
  p.K = (int)k;
  p.ldy = (int)ldy;
  p.out_dtype = y_dtype;
  const int64_t tiles = (n / w16::BW) * cdiv(m, w16::BT);
  const int64_t pairs = tiles < cap ? tiles : cap;
  (void)launch_kc(w16::gemm_w4a16_pair_kernel, dim3((unsigned)(2 * pairs)), dim3(w16::THREADS), w16::SMEM, st, 2,
                  tmx, tmw, p);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}
