// Vocabulary projection (lm_head) with the greedy pick fused into its epilogue, on the
// 5th-generation tensor cores (sm_100a).
//
// Reference: ParallelLMHead.forward (adallm/ops/embed_head.py:56-66) computes
// logits = F.linear(x, W) in bf16 (fp32 accumulation, bf16 result) over this rank's vocabulary
// shard, and greedy decoding takes the first maximum of those bf16 logits (torch.argmax).
//
// Decode shape: x bf16 [M <= 64 tokens, K], W bf16 [V, K] (V ~ 150k-260k rows): a weight stream
// (1.24 GB for Qwen3-8B), so the kernel is HBM-bound and built like the persistent NVFP4 GEMM:
// one CTA per SM walks 128-row vocabulary tiles; warp 0 streams W tiles [128 x 64] and the token
// tile [NB x 64] by TMA into a ring of stages (the first stages of W before the programmatic-launch
// wait, as W never depends on the previous kernel), warp 1 issues tcgen05.mma kind::f16 (bf16
// operands, M 128 = vocabulary rows, N = NB tokens, fp32 accumulators in TMEM, two of them so the
// epilogue of tile i overlaps the MMAs of tile i + 1), warps 2..5 read the accumulator rows
// (tcgen05.ld), round them to bf16 (optionally storing the logits), and reduce each token's
// (value, row) maximum over the tile -- ties to the lower row.  A second tiny kernel reduces the
// per-tile maxima of each token (in tile order, ties to the lower row), which reproduces
// torch.argmax over the bf16 logits.
#include "common.cuh"
#include "sm100.cuh"

namespace ada {
namespace lmh {

using namespace sm100;

constexpr int BM = 128;            // vocabulary rows per tile (MMA M, TMEM lanes)
constexpr int KT = 64;             // bf16 K elements per stage: one 128-byte swizzle row
constexpr int A_BYTES = BM * 128;  // 16 KB of W per stage
constexpr int MAX_NB = 64;         // tokens per call (MMA N, a multiple of 16)
constexpr int STAGES = 8;
constexpr size_t ERR_BYTES = 256;  // error word at offset 0 of the workspace
constexpr unsigned int ERR_STAGE = 1u, ERR_FULL = 2u, ERR_ACC = 4u, ERR_ACCE = 8u;  // bounded waits that ran out

struct Params {
  int M, V, K, n_tiles, nkt;
  __nv_bfloat16* logits;  // [M][ldl] or null
  int64_t ldl;
  float* part_val;        // [n_tiles][NB] per-tile maximum of each token
  int* part_idx;          // [n_tiles][NB] its row
  unsigned int* err;
};

template <int NB>
struct Cfg {
  static constexpr int B_BYTES = NB * 128;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * NB <= 32 ? 32 : 2 * NB <= 64 ? 64 : 128;
  // bf16 A and B (formats 1), fp32 D, both K-major, M 128, N NB
  static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NB >> 3) << 17) |
                                    ((uint32_t)(BM >> 4) << 24);
  // ring, the per-warp maxima [2][4][NB] (value, row), flags [2][4], barriers, TMEM slot, abort flag
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE + 2 * 4 * NB * 8 + 32 + 512;
};

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// (v, i) replaces (bv, bi) when larger, or equal with a lower row (torch.argmax: first maximum).
__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

template <int NB>
__global__ void __launch_bounds__(192, 1)
    lm_head_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx, const Params p) {
  using C = Cfg<NB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sval = reinterpret_cast<float*>(smem + (size_t)STAGES * C::STAGE);  // [2][4][NB]
  int* sidx = reinterpret_cast<int*>(sval + 2 * 4 * NB);                     // [2][4][NB]
  int* sok = sidx + 2 * 4 * NB;                                              // [2][4] per-warp accumulator ok
  uint64_t* full = reinterpret_cast<uint64_t*>(sok + 8);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;  // [2] accumulator b complete
  uint64_t* acce = accf + 2;        // [2] accumulator b drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_v = abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = p.n_tiles, nkt = p.nkt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
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
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
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
      // W never depends on the previous kernel: the first STAGES tiles of it are requested
      // before the programmatic-launch wait, the token tiles after it.
      const int first_total = ((tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * nkt;
      const int pre = first_total < STAGES ? first_total : STAGES;
      for (int i = 0; i < pre; ++i) {
        const int t = (int)blockIdx.x + (i / nkt) * (int)gridDim.x, kt = i % nkt;
        mbar_expect_tx(&full[i], A_BYTES);
        tma_load_2d(smem + (size_t)i * C::STAGE, &tmw, &full[i], kt * 128, t * BM);
      }
      pdl_wait();
      uint32_t it = 0;
      for (int t = blockIdx.x; t < tiles && !*abort_v; t += gridDim.x) {
        bool stop = false;
        for (int kt = 0; kt < nkt; ++kt, ++it) {
          const int s = (int)(it % (uint32_t)STAGES);
          uint8_t* st = smem + (size_t)s * C::STAGE;
          if (it >= (uint32_t)STAGES) {
            if (!mbar_wait_bounded(&empty[s], ((it / STAGES) & 1) ^ 1, abort_v, p.err, ERR_STAGE)) {
              stop = true;
              break;
            }
            mbar_expect_tx(&full[s], A_BYTES);
            tma_load_2d(st, &tmw, &full[s], kt * 128, t * BM);
          }
          mbar_arrive_expect_tx(&full[s], C::B_BYTES);
          tma_load_2d(st + A_BYTES, &tmx, &full[s], kt * 128, 0);
        }
        if (stop) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer ----------------
      uint32_t it = 0, lt = 0;
      for (int t = blockIdx.x; t < tiles && !*abort_v; t += gridDim.x, ++lt) {
        const uint32_t b = lt & 1, use = lt >> 1;
        if (use > 0 && !mbar_wait_bounded(&acce[b], (use - 1) & 1, abort_v, p.err, ERR_ACCE)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * NB;
        bool failed = false;
        for (int kt = 0; kt < nkt; ++kt, ++it) {
          const int s = (int)(it % (uint32_t)STAGES);
          if (!mbar_wait_bounded(&full[s], (it / STAGES) & 1, abort_v, p.err, ERR_FULL)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + (size_t)s * C::STAGE);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < KT / 16; ++kk)  // 16 bf16 = 32 bytes of the 128-byte row per MMA
            mma_bf16(acc, desc_kmajor_sw128(a_addr + kk * 32), desc_kmajor_sw128(b_addr + kk * 32), C::IDESC,
                     (kt | kk) != 0);
          tc_commit(&empty[s]);
        }
        tc_commit(&accf[b]);  // also after a failure: drains the issued MMAs
        if (failed) break;
      }
    }
    __syncwarp();
  } else {  // ---------------- epilogue (warps 2..5: TMEM lane quarter = warp % 4) ----------------
    pdl_wait();     // outputs of the previous step are no longer read past here
    pdl_trigger();  // let the cross-tile reduction get resident
    const int q = warp & 3;
    const int et = threadIdx.x - 64;
    const int r = q * 32 + lane;
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++lt) {
      const uint32_t b = lt & 1, use = lt >> 1;
      const bool ok_warp =
          __all_sync(0xffffffffu, mbar_wait_bounded(&accf[b], use & 1, abort_v, p.err, ERR_ACC) && !*abort_v);
      tc_fence_after();
      const int n = t * BM + r;
      const bool row_ok = n < p.V;
      const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + b * NB;
      float* sv = sval + (b * 4 + q) * NB;
      int* si = sidx + (b * 4 + q) * NB;
#pragma unroll 1
      for (int c = 0; c < NB; c += 16) {
        float v[16];
        tmem_ld16(lane_addr + c, v);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const __nv_bfloat16 lb = __float2bfloat16_rn(v[k]);
          const int m = c + k;
          if (ok_warp && row_ok && p.logits && m < p.M) p.logits[(int64_t)m * p.ldl + n] = lb;
          float bv = row_ok ? __bfloat162float(lb) : -INFINITY;
          int bi = row_ok ? n : 0x7fffffff;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            better(bv, bi, ov, oi);
          }
          if (lane == 0) {
            sv[m] = bv;
            si[m] = bi;
          }
        }
      }
      if (lane == 0) sok[b * 4 + q] = ok_warp ? 1 : 0;
      tc_fence_before();
      epi_bar();  // every lane has read accumulator b; the warps' maxima and flags are in shared memory
      // one decision for all four warps, so they leave the loop together (the named barrier above
      // must be reached by all 128 epilogue threads the same number of times)
      const bool ok = sok[b * 4] && sok[b * 4 + 1] && sok[b * 4 + 2] && sok[b * 4 + 3];
      if (et == 0) mbar_arrive_plain(&acce[b]);
      if (et < NB) {  // token et: the four warps' maxima, combined; ties go to the lower row
        float bv = sval[(b * 4) * NB + et];
        int bi = sidx[(b * 4) * NB + et];
        for (int w = 1; w < 4; ++w) better(bv, bi, sval[(b * 4 + w) * NB + et], sidx[(b * 4 + w) * NB + et]);
        p.part_val[(int64_t)t * NB + et] = ok ? bv : __int_as_float(0x7fc00000);
        p.part_idx[(int64_t)t * NB + et] = bi;
      }
      if (!ok) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// One warp per token: the maximum over the tiles in tile order (ties to the lower row).
__global__ void __launch_bounds__(32) lm_head_pick_kernel(const float* __restrict__ pv, const int* __restrict__ pi,
                                                          int tiles, int nb, int64_t idx_base, int64_t* out_idx,
                                                          float* out_val) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = threadIdx.x; t < tiles; t += 32) better(bv, bi, pv[(int64_t)t * nb + m], pi[(int64_t)t * nb + m]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  if (threadIdx.x == 0) {
    if (out_idx) out_idx[m] = (bi == 0x7fffffff ? 0 : bi) + idx_base;
    if (out_val) out_val[m] = bv;
  }
}

static int nb_for(int64_t m) { return m <= 16 ? 16 : m <= 32 ? 32 : m <= 48 ? 48 : 64; }

template <int NB>
static bool smem_ready() {
  static std::atomic<bool> done[64];  // function attributes are per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (done[dev]) return true;
  if (cudaFuncSetAttribute(lm_head_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg<NB>::SMEM) !=
      cudaSuccess)
    return false;
  done[dev] = true;
  return true;
}

}  // namespace lmh
}  // namespace ada

using namespace ada;

extern "C" size_t ada_lm_head_workspace_size(int64_t m, int64_t vocab) {
  if (m <= 0 || m > lmh::MAX_NB || vocab <= 0) return 0;
  const int64_t tiles = (vocab + lmh::BM - 1) / lmh::BM;
  return lmh::ERR_BYTES + (size_t)tiles * lmh::nb_for(m) * (sizeof(float) + sizeof(int));
}

extern "C" int ada_lm_head_argmax(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw,
                                  int64_t vocab, int64_t idx_base, void* logits, int64_t ldl, int64_t* out_idx,
                                  float* out_val, void* workspace, size_t workspace_bytes, void* stream) {
  if (m < 0 || k <= 0 || vocab <= 0) return ADA_ERR_INVALID_ARG;
  if (m == 0) return ADA_OK;
  if (!x || !w || !workspace || (!logits && !out_idx && !out_val)) return ADA_ERR_INVALID_ARG;
  if (m > lmh::MAX_NB || k % lmh::KT || vocab > 0x7fffff00LL) return ADA_ERR_UNSUPPORTED;
  if (ldx < k || ldw < k || (logits && ldl < vocab)) return ADA_ERR_INVALID_ARG;
  if (((uintptr_t)x & 15) || ((uintptr_t)w & 15) || (ldx & 7) || (ldw & 7)) return ADA_ERR_ALIGNMENT;
  if (((uintptr_t)workspace & 255)) return ADA_ERR_ALIGNMENT;
  if (workspace_bytes < ada_lm_head_workspace_size(m, vocab)) return ADA_ERR_WORKSPACE;
  const int nb = lmh::nb_for(m);
  lmh::Params P;
  P.M = (int)m;
  P.V = (int)vocab;
  P.K = (int)k;
  P.n_tiles = (int)((vocab + lmh::BM - 1) / lmh::BM);
  P.nkt = (int)(k / lmh::KT);
  P.logits = reinterpret_cast<__nv_bfloat16*>(logits);
  P.ldl = ldl;
  P.err = reinterpret_cast<unsigned int*>(workspace);
  P.part_val = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + lmh::ERR_BYTES);
  P.part_idx = reinterpret_cast<int*>(P.part_val + (size_t)P.n_tiles * nb);

  // W [vocab][k] and x [m][k] as byte tensors; boxes of 128 bytes (64 bf16) x 128 rows / x NB rows.
  // Rows past the tensor (the last vocabulary tile, the token padding) are filled with zeros.
  CUtensorMap tmw, tmx;
  const cuuint64_t wd[2] = {(cuuint64_t)k * 2, (cuuint64_t)vocab}, ws_[1] = {(cuuint64_t)ldw * 2};
  const cuuint32_t wb[2] = {128, (cuuint32_t)lmh::BM};
  const cuuint64_t xd[2] = {(cuuint64_t)k * 2, (cuuint64_t)m}, xs[1] = {(cuuint64_t)ldx * 2};
  const cuuint32_t xb[2] = {128, (cuuint32_t)nb};
  if (!sm100::encode_bytes(&tmw, w, 2, wd, ws_, wb, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !sm100::encode_bytes(&tmx, x, 2, xd, xs, xb, CU_TENSOR_MAP_SWIZZLE_128B))
    return ADA_ERR_CUDA;

  static std::atomic<int> sms[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ADA_ERR_CUDA;
  int n_sm = sms[dev].load(std::memory_order_relaxed);
  if (!n_sm) {
    if (cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n_sm <= 0)
      return ADA_ERR_CUDA;
    sms[dev].store(n_sm, std::memory_order_relaxed);
  }
  const unsigned grid = (unsigned)(P.n_tiles < n_sm ? P.n_tiles : n_sm);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define ADA_LMH(NB_)                                                                                         \
  do {                                                                                                       \
    if (!lmh::smem_ready<NB_>()) return ADA_ERR_CUDA;                                                        \
    (void)ada::launch_k(lmh::lm_head_kernel<NB_>, dim3(grid), dim3(192), lmh::Cfg<NB_>::SMEM, st, tmw, tmx, P); \
  } while (0)
  switch (nb) {
    case 16: ADA_LMH(16); break;
    case 32: ADA_LMH(32); break;
    case 48: ADA_LMH(48); break;
    default: ADA_LMH(64); break;
  }
#undef ADA_LMH
  ADA_CHECK_LAUNCH();
  if (out_idx || out_val) {
    (void)ada::launch_k(lmh::lm_head_pick_kernel, dim3((unsigned)m), dim3(32), 0, st, (const float*)P.part_val,
                        (const int*)P.part_idx, P.n_tiles, nb, idx_base, out_idx, out_val);
    ADA_CHECK_LAUNCH();
  }
  return ADA_OK;
}
