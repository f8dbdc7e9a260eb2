// Causal prefill attention over the FP8 paged KV cache for B200 (sm_100a).
//
// Replaces the prefix-cache prefill branch of Attention.forward (reference
// adallm/ops/attention.py:335-358): there the e4m3 pages of every sequence are first gathered
// and widened to a contiguous fp16 K/V copy (_gather_kv_from_blocks, :254-286) and then passed
// to flash_attn_varlen_func(causal=True, window_size=(W, 0)).  Here the kernel reads the e4m3
// pages in place through the block table, so the gather copy (2 x 2 bytes per cached element
// written and read again) disappears.
//
// Semantics (flash-attn's published varlen rules, as the reference calls it): sequence b has
// len_q = cu_seqlens_q[b+1] - cu_seqlens_q[b] new query tokens and len_k = cu_seqlens_k[b+1] -
// cu_seqlens_k[b] keys (cached prefix + new tokens, all already stored in the pages); the causal
// mask is aligned to the bottom right, so query i (0-based within the new tokens) sees keys
// j <= i + len_k - len_q, and with a sliding window W > 0 only keys j >= i + len_k - len_q - W
// (W + 1 keys).  q is rounded to fp16, K/V widened from e4m3 to fp16, scores and softmax
// statistics in fp32, probabilities rounded to fp16 for P.V, fp32 accumulation.  A row with no
// visible key is written as zeros.
//
// Work split and roles: see the tcgen05 section below.  One CTA per (256-row query block, KV
// head, sequence); the 256 rows are (token, head) pairs of the GQA group, head fastest, so
// 256 / group consecutive query tokens share every K/V block the CTA loads (each e4m3 byte is
// read once per query block, not once per head).  S = Q . K^T and O += P . V run on the
// 5th-generation tensor cores (tcgen05.mma kind::f16, f16 operands staged in shared memory,
// fp32 accumulators in TMEM); the e4m3 pages arrive by TMA (4-D tensor map over
// [pages][page][Hkv][128] bytes) and are widened to f16 operand tiles in shared memory.
// Query blocks are dealt last-first so the longest causal rows start first.
#include "common.cuh"
#include "sm100.cuh"

namespace ada {
namespace pf {

constexpr int D = 128;
constexpr int TILE = 16;
constexpr int TILE_BYTES = TILE * D;       // 16 keys x 128 e4m3 bytes
constexpr float LOG2E = 1.4426950408889634f;
constexpr unsigned int ERR_TILE_WAIT = 0x70;

struct Params {
  const void* q;
  int64_t q_st, q_sh;  // token, head strides (elements)
  void* out;
  int64_t o_st, o_sh;
  const int32_t* bt;
  int64_t bt_stride;
  int64_t num_pages;  // block ids outside [0, num_pages) are holes (masked)
  int32_t max_pages;
  const int32_t* cu_q;
  const int32_t* cu_k;
  int32_t group, qt, page, window;
  float scale_log2;  // softmax scale * k_scale * log2(e)
  float v_scale;
  unsigned int* err;  // optional error word (bounded waits that ran out)
};

// Key range [lo, hi) visible to query token t (0-based among the new tokens).
__device__ __forceinline__ void key_range(const Params& P, int t, int off, int len_k, int& lo, int& hi) {
  hi = min(len_k, t + off + 1);
  lo = P.window > 0 ? max(0, t + off - P.window) : 0;
}

// ======================= tensor-core (tcgen05) form =======================
// One CTA per (256-row query block, KV head, sequence): two 128-row query tiles (the 128 rows
// of a tile are the TMEM lanes) share every K/V block the CTA loads and widens.
// Roles (14 warps):
//   warp 0       producer: walks the block table (entries held in the warp's lanes 8 blocks
//                ahead), lane 0 TMA-loads the e4m3 K and V rows of each 64-key block (four
//                16-key page tiles) into a staging ring;
//   warp 1       MMA issuer (lane 0) and TMEM owner: per block and tile t, S_t = Q_t . K^T
//                (M 128, N 64, kind::f16) into one of tile t's two TMEM S buffers, then
//                O_t += P_t . V (M 128, N 128) into tile t's TMEM O;
//   warps 2-5    converters: the query rows bf16/fp16 -> f16 once, then per block the staged
//                e4m3 K and V -> f16 operand tiles (128-byte swizzled; K read K-major, V
//                MN-major, so neither needs a transpose);
//   warps 6-9    softmax of tile 0, warps 10-13 softmax of tile 1: thread = row; reads its 64
//                scores with tcgen05.ld, masks, one online-softmax step, rescales its O row in
//                TMEM when its reference max moved (after the previous P.V completed), writes
//                its f16 probabilities as the A tile of the next P.V; finally normalises and
//                stores its O row.
// S of block j + 1 is computed while the softmax warpgroups work on block j, and each tile's
// P.V runs while its warpgroup works on the next block; the two warpgroups (two warps per
// scheduler) hide each other's latency.  Every wait is bounded (2 s) and ends the CTA's loops
// through a shared abort flag.
//
// Barriers (phase k of a barrier = its k-th completion; block j, tile t):
//   e_full[j % NSTG]   producer arrive.expect_tx + TMA bytes -> converters   (phase j / NSTG)
//   e_empty[j % NSTG]  4 converter warps -> producer, slot reusable           (phase j / NSTG)
//   kv_full[j % NKV]   4 converter warps -> MMA (and softmax, page flags)     (phase j / NKV)
//   kv_empty[j % NKV]  commit after both tiles' P.V of block j -> converters (phase j / NKV)
//   s_full[t][j % 2]   commit after S_{t,j} -> softmax warpgroup t            (phase j / 2)
//   p_full[t]          4 softmax warps of tile t -> MMA, P tile written       (phase j)
//   o_done[t]          commit after P.V of tile t, block j -> softmax t       (phase j)
//   q_ready            4 converter warps -> MMA, Q tiles written              (phase 0)
//   fin                commit after the last MMA -> teardown                  (phase 0)
// A barrier can run at most one phase ahead of any waiter: each refill of a slot waits for the
// consumer's release of the previous use (e_empty, kv_empty; S buffers by p_full, the single P
// tile by o_done of the previous block).
namespace tc {
constexpr int NT = 2;    // 128-row query tiles per CTA, one softmax warpgroup each, sharing every K/V block
constexpr int BM = 128;  // rows per tile = TMEM lanes
constexpr int BN = 64;
constexpr int NSTG = 2;
constexpr int NKV = 3;  // f16 K/V operand slots: the converters run up to NKV - 1 blocks ahead of P.V
constexpr int NCONV = 4;
constexpr int NSOFT = 4;  // warps per softmax warpgroup
constexpr int THREADS = (2 + NCONV + NT * NSOFT) * 32;
constexpr int Q_OFF = 0;                        // f16 Q, NT x [2 d-halves][128 rows][128 B]
constexpr int KF_OFF = Q_OFF + NT * 32768;      // f16 K, NKV slots x [2 d-halves][64 keys][128 B]
constexpr int VF_OFF = KF_OFF + NKV * 16384;    // f16 V, NKV slots x [2 d-halves][64 keys][128 B]
constexpr int P_OFF = VF_OFF + NKV * 16384;     // f16 P, NT x [128 rows][64 keys = 128 B]
constexpr int E_OFF = P_OFF + NT * 16384;       // e4m3 staging, NSTG x (4 K page tiles + 4 V page tiles)
constexpr int E_BYTES = 2 * 4 * TILE_BYTES;
constexpr int BAR_OFF = E_OFF + NSTG * E_BYTES;
constexpr int NBAR = 2 * NSTG + 2 * NKV + 4 * NT + 2;
constexpr int FLAG_OFF = BAR_OFF + NBAR * 8;  // page-tile flags: e_ok[NSTG], kv_ok[NKV] (bit i: tile i loaded)
constexpr int SMEM = 1024 + FLAG_OFF + (NSTG + NKV) * 4 + 16;
constexpr uint32_t TMEM_COLS = 512;  // O of tile t at [128 t, +128); S buffer b of tile t at 256 + 128 t + 64 b
constexpr float RESCALE_LOG2 = 8.f;  // move a row's reference max only when it grew by more than this
constexpr uint32_t S_COL = 256;
static_assert(SMEM <= 232448, "shared memory per CTA");
// instruction descriptors, kind::f16: D f32 (bit 4), A/B f16, M 128; P.V reads B (V) MN-major (bit 16)
constexpr uint32_t IDESC_S = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
constexpr uint32_t IDESC_PV = (1u << 4) | (1u << 16) | ((uint32_t)(D >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 16 consecutive fp32 columns of this thread's TMEM lane; the values are valid after tmem_wait_ld.
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Wait for this thread's tcgen05.ld, then pin the 16 registers after the wait (an empty volatile
// asm that redefines them), so no use of them is scheduled before it.
__device__ __forceinline__ void tmem_wait_ld16(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]));
}
__device__ __forceinline__ void tmem_pin16(uint32_t* r) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// try_wait with a suspend-time hint: the thread sleeps until the phase completes (or the hint
// runs out) instead of spinning, so waiting roles leave the issue slots to the working ones.
__device__ __forceinline__ bool try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(sm100::smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Bounded wait (2 s): gives up when another role aborted, or sets the abort flag and the error
// code when the phase never completes.
__device__ __forceinline__ bool wait_b(uint64_t* bar, uint32_t parity, volatile int* abort_v, unsigned int* err) {
  if (try_wait_sleep(bar, parity)) return true;
  const uint64_t t0 = sm100::globaltimer();
  for (;;) {
    if (try_wait_sleep(bar, parity)) return true;
    if (*abort_v) return false;
    if (sm100::globaltimer() - t0 > 2000000000ull) {
      *abort_v = 1;
      if (err) atomicOr(err, ERR_TILE_WAIT);
      return false;
    }
  }
}

// Block-table entry of the 16-key tile starting at key0 of sequence b (-1 past the keys any
// row of the block can see); tile_page turns it into the page id, or -1 for a hole.
__device__ __forceinline__ int tile_entry(const Params& P, int b, int key0, int k_end) {
  if (key0 >= k_end) return -1;
  return __ldg(P.bt + (int64_t)b * P.bt_stride + key0 / P.page);
}
__device__ __forceinline__ int tile_page(const Params& P, int entry) {
  return (entry < 0 || entry >= P.num_pages) ? -1 : entry;
}

// 16 e4m3 -> 16 f16 (two 16-byte chunks, element order kept).
__device__ __forceinline__ void cvt16(const uint4& e, uint4& lo, uint4& hi) {
  lo.x = e4m3x2_to_f16x2((uint16_t)(e.x & 0xFFFFu));
  lo.y = e4m3x2_to_f16x2((uint16_t)(e.x >> 16));
  lo.z = e4m3x2_to_f16x2((uint16_t)(e.y & 0xFFFFu));
  lo.w = e4m3x2_to_f16x2((uint16_t)(e.y >> 16));
  hi.x = e4m3x2_to_f16x2((uint16_t)(e.z & 0xFFFFu));
  hi.y = e4m3x2_to_f16x2((uint16_t)(e.z >> 16));
  hi.z = e4m3x2_to_f16x2((uint16_t)(e.w & 0xFFFFu));
  hi.w = e4m3x2_to_f16x2((uint16_t)(e.w >> 16));
}

template <typename TQ, typename TO>
__global__ void __launch_bounds__(THREADS, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, Params P) {
  using namespace sm100;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, kvh = blockIdx.y;
  const int qblk = gridDim.x - 1 - blockIdx.x;  // longest causal rows first

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = base + Q_OFF;
  uint8_t* kf = base + KF_OFF;
  uint8_t* vf = base + VF_OFF;
  uint8_t* ps = base + P_OFF;
  uint8_t* es = base + E_OFF;
  uint64_t* e_full = reinterpret_cast<uint64_t*>(base + BAR_OFF);
  uint64_t* e_empty = e_full + NSTG;
  uint64_t* kv_full = e_empty + NSTG;
  uint64_t* kv_empty = kv_full + NKV;
  uint64_t* s_full = kv_empty + NKV;  // [NT][2]
  uint64_t* p_full = s_full + 2 * NT;  // [NT]
  uint64_t* o_done = p_full + NT;      // [NT]
  uint64_t* q_ready = o_done + NT;
  uint64_t* fin = q_ready + 1;
  int* e_ok = reinterpret_cast<int*>(base + FLAG_OFF);
  int* kv_ok = e_ok + NSTG;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kv_ok + NKV);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_v = abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTG; ++s) {
      mbar_init(&e_full[s], 1);
      mbar_init(&e_empty[s], NCONV);
    }
    for (int i = 0; i < NKV; ++i) {
      mbar_init(&kv_full[i], NCONV);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2 * NT; ++i) mbar_init(&s_full[i], 1);
    for (int t = 0; t < NT; ++t) {
      mbar_init(&p_full[t], NSOFT);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(q_ready, NCONV);
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // q, the cache pages and the metadata come from earlier kernels
  pdl_trigger();

  const int q_begin = __ldg(P.cu_q + b);
  const int len_q = __ldg(P.cu_q + b + 1) - q_begin;
  const int len_k = __ldg(P.cu_k + b + 1) - __ldg(P.cu_k + b);
  const int t0 = qblk * P.qt;
  const bool active = t0 < len_q;
  const int off = len_k - len_q;
  int nblk = 0, kb0 = 0, k_end = 0;
  if (active) {
    const int t_last = min(t0 + P.qt, len_q) - 1;
    int k_lo, k_hi, dlo, dhi;
    key_range(P, t0, off, len_k, k_lo, dhi);
    key_range(P, t_last, off, len_k, dlo, k_hi);
    k_end = min(k_hi, P.max_pages * P.page);
    kb0 = (k_lo / BN) * BN;
    nblk = k_end > k_lo ? (k_end - kb0 + BN - 1) / BN : 0;
  }

  if (warp == 0) {  // ---------------- producer ----------------
    // The warp holds the block-table entries of 8 blocks (32 page tiles, one per lane) and the
    // next 8 in flight, so no table load is waited for in the per-block path; lane 0 issues.
    auto entry = [&](int t) { return tile_entry(P, b, kb0 + TILE * t, k_end); };
    int cur = nblk > 0 ? entry(lane) : -1;
    int nxt = nblk > 8 ? entry(32 + lane) : -1;
    int issued = 0;
    for (int j = 0; j < nblk; ++j) {
      if (j > 0 && (j & 7) == 0) {
        cur = nxt;
        nxt = j + 8 < nblk ? entry(32 * (j / 8 + 1) + lane) : -1;
      }
      int blk[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) blk[i] = tile_page(P, __shfl_sync(0xffffffffu, cur, 4 * (j & 7) + i));
      const int s = j % NSTG;
      int go = 1;
      if (lane == 0) go = !*abort_v && (j < NSTG || wait_b(&e_empty[s], ((j / NSTG) - 1) & 1, abort_v, P.err));
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      if (lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        uint32_t bytes = 0;
        int mask = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          bytes += blk[i] >= 0 ? 2 * TILE_BYTES : 0;
          mask |= (blk[i] >= 0 ? 1 : 0) << i;
        }
        e_ok[s] = mask;  // published by the arrive below (release), read after the phase completes
        mbar_arrive_expect_tx(&e_full[s], bytes);
        uint8_t* st = es + s * E_BYTES;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (blk[i] < 0) continue;
          const int key0 = kb0 + j * BN + TILE * i;
          const int row0 = key0 - (key0 / P.page) * P.page;
          tma_load_4d(st + i * TILE_BYTES, &tmk, &e_full[s], 0, kvh, row0, blk[i]);
          tma_load_4d(st + (4 + i) * TILE_BYTES, &tmv, &e_full[s], 0, kvh, row0, blk[i]);
        }
      }
      issued = j + 1;
    }
    if (lane == 0) {
      // leave no copy in flight when the CTA ends: wait (bounded) for the last use of each slot
      for (int j = issued > NSTG ? issued - NSTG : 0; j < issued; ++j) {
        const int s = j % NSTG;
        uint32_t spins = 0;
        const uint64_t t_start = globaltimer();
        while (!mbar_try_wait(&e_full[s], (j / NSTG) & 1)) {
          if ((++spins & 63u) == 0 && globaltimer() - t_start > 2000000000ull) {
            if (P.err) atomicOr(P.err, ERR_TILE_WAIT);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {  // ---------------- MMA issuer ----------------
    if (lane == 0 && nblk > 0) {
      const uint32_t q_addr = smem_u32(qs), k_addr = smem_u32(kf), v_addr = smem_u32(vf), p_addr = smem_u32(ps);
      auto issue_s = [&](int j) {  // S_{t,j} = Q_t . K_j^T (K slot j % NKV) into S buffer j % 2 of tile t
        const uint32_t kb = (uint32_t)(j % NKV);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const uint32_t d = tmem + S_COL + 128u * (uint32_t)t + BN * (uint32_t)(j & 1);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t hoff = (uint32_t)t * 32768u + (uint32_t)(kk / 4) * 16384u + (uint32_t)(kk % 4) * 32u;
            const uint32_t koff = kb * 16384u + (uint32_t)(kk / 4) * 8192u + (uint32_t)(kk % 4) * 32u;
            mma_f16(d, desc_kmajor_sw128(q_addr + hoff), desc_kmajor_sw128(k_addr + koff), IDESC_S, kk > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[2 * t + (j & 1)]);
        }
      };
      bool ok = wait_b(q_ready, 0, abort_v, P.err) && wait_b(&kv_full[0], 0, abort_v, P.err);
      if (ok) {
        tc_fence_after();
        issue_s(0);
      }
      for (int j = 0; ok && j < nblk; ++j) {
        if (j + 1 < nblk) {
          if (!wait_b(&kv_full[(j + 1) % NKV], ((j + 1) / NKV) & 1, abort_v, P.err)) break;
          tc_fence_after();
          issue_s(j + 1);
        }
        const uint32_t kb = (uint32_t)(j % NKV);
        bool pv_ok = true;
        for (int t = 0; t < NT && pv_ok; ++t) {  // O_t += P_{t,j} . V_j, 16 keys per MMA
          if (!wait_b(&p_full[t], j & 1, abort_v, P.err)) {
            pv_ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t pd = desc_kmajor_sw128(p_addr + (uint32_t)t * 16384u + (uint32_t)kk * 32u);
            // V MN-major: d-halves 8 KB apart (leading), 8-key groups 1 KB apart (stride)
            const uint64_t vd = smem_desc(v_addr + kb * 16384u + (uint32_t)kk * 16u * 128u, 8192, 1024, SWZ_128B);
            mma_f16(tmem + 128u * (uint32_t)t, pd, vd, IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&o_done[t]);
        }
        if (!pv_ok) break;
        tc_commit(&kv_empty[kb]);
      }
      // every MMA issued above has completed before the teardown
      tc_commit(fin);
      uint32_t spins = 0;
      const uint64_t t_start = globaltimer();
      while (!mbar_try_wait(fin, 0)) {
        if ((++spins & 63u) == 0 && globaltimer() - t_start > 2000000000ull) {
          if (P.err) atomicOr(P.err, ERR_TILE_WAIT);
          break;
        }
      }
    }
  } else if (warp < 2 + NCONV) {  // ---------------- converters ----------------
    const int ct = threadIdx.x - 64;  // 0..127
    if (active) {
      // query rows -> f16 Q tiles: CTA row R = (token t0 + R / group, head R % group of KV head
      // kvh) is row R % 128 of tile R / 128
      for (int R = ct; R < NT * BM; R += NCONV * 32) {
        const int r = R % BM;
        const int tok = t0 + R / P.group;
        const bool ok = R < P.qt * P.group && tok < len_q;
        const TQ* qp = reinterpret_cast<const TQ*>(P.q) + (int64_t)(q_begin + tok) * P.q_st +
                       (int64_t)(kvh * P.group + R % P.group) * P.q_sh;
        uint8_t* qt = qs + (R / BM) * 32768;
#pragma unroll 4
        for (int c = 0; c < 16; ++c) {  // 8 elements per chunk
          uint4 h = make_uint4(0, 0, 0, 0);
          if (ok) {
            float f[8];
            unpack8<TQ>(*reinterpret_cast<const uint4*>(qp + 8 * c), f);
            h.x = pack_half2(f[0], f[1]);
            h.y = pack_half2(f[2], f[3]);
            h.z = pack_half2(f[4], f[5]);
            h.w = pack_half2(f[6], f[7]);
          }
          const int half = c >> 3, ch = c & 7;
          *reinterpret_cast<uint4*>(qt + half * 16384 + r * 128 + ((ch ^ (r & 7)) << 4)) = h;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_plain(q_ready);
    }
    for (int j = 0; j < nblk; ++j) {
      const int s = j % NSTG, kb = j % NKV;
      if (!wait_b(&e_full[s], (j / NSTG) & 1, abort_v, P.err)) break;
      if (j >= NKV && !wait_b(&kv_empty[kb], ((j / NKV) - 1) & 1, abort_v, P.err)) break;
      const uint8_t* st = es + s * E_BYTES;
      const int mask = e_ok[s];
      int blk_ok[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) blk_ok[i] = (mask >> i) & 1;
      // 64 keys x 8 chunks of 16 e4m3 per operand: 4 units per thread for K, 4 for V
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int unit = ct + 128 * u;
        const int key = unit >> 3, ch = unit & 7;
        const int sub = key >> 4, row = key & 15;
        const int half = ch >> 2;
        const int c0 = ((ch & 3) * 2) ^ (key & 7), c1 = ((ch & 3) * 2 + 1) ^ (key & 7);
        const bool kok = blk_ok[sub] != 0;
        const bool vok = kok & (kb0 + j * BN + key < len_k);
        const uint4 z = make_uint4(0, 0, 0, 0);
        // the staging slot is always in bounds: load, then select (no branch per unit)
        uint4 ke = *reinterpret_cast<const uint4*>(st + sub * TILE_BYTES + row * 128 + ((ch ^ (row & 7)) << 4));
        uint4 ve = *reinterpret_cast<const uint4*>(st + (4 + sub) * TILE_BYTES + row * 128 + ((ch ^ (row & 7)) << 4));
        if (!kok) ke = z;
        if (!vok) ve = z;
        uint4 lo, hi;
        cvt16(ke, lo, hi);
        uint8_t* kd = kf + kb * 16384 + half * 8192 + key * 128;  // slot kb of NKV
        *reinterpret_cast<uint4*>(kd + (c0 << 4)) = lo;
        *reinterpret_cast<uint4*>(kd + (c1 << 4)) = hi;
        cvt16(ve, lo, hi);
        uint8_t* vd = vf + kb * 16384 + half * 8192 + key * 128;
        *reinterpret_cast<uint4*>(vd + (c0 << 4)) = lo;
        *reinterpret_cast<uint4*>(vd + (c1 << 4)) = hi;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        if (warp == 2) kv_ok[kb] = mask;  // for the softmax, published by this lane's arrive
        mbar_arrive_plain(&kv_full[kb]);
        mbar_arrive_plain(&e_empty[s]);
      }
    }
  } else {  // ---------------- softmax + epilogue: warpgroup t, thread = row r of tile t ----------------
    const int t = (warp - 2 - NCONV) / NSOFT;
    const int q4 = warp & 3;  // TMEM lane quarter this warp may access
    const int r = 32 * q4 + lane;
    const int R = t * BM + r;  // row of the CTA
    const uint32_t trow = tmem + ((uint32_t)(32 * q4) << 16);
    const uint32_t o_col = 128u * (uint32_t)t, s_col = S_COL + 128u * (uint32_t)t;
    const int tok = t0 + R / P.group;
    const bool valid = active && R < P.qt * P.group && tok < len_q;
    int lo = 0, hi = 0;
    if (valid) key_range(P, tok, off, len_k, lo, hi);
    float m = -INFINITY, l = 0.f;
    bool failed = false;
    for (int j = 0; j < nblk; ++j) {
      const int sb = j & 1;
      // warp-uniform outcome: the tcgen05.ld / st below are warp-collective
      if (!__all_sync(0xffffffffu, wait_b(&s_full[2 * t + sb], (j >> 1) & 1, abort_v, P.err))) {
        failed = true;
        break;
      }
      tc_fence_after();
      uint32_t sr[64];
#pragma unroll
      for (int i = 0; i < 4; ++i) tmem_ld16_async(trow + s_col + BN * sb + 16 * i, sr + 16 * i);
      tmem_wait_ld16(sr);
      tmem_pin16(sr + 16);
      tmem_pin16(sr + 32);
      tmem_pin16(sr + 48);
      const int key_base = kb0 + j * BN;
      // the page flags the converters stored with K/V slot j % NKV: S_j was computed from that
      // slot, so its kv_full phase is complete (this wait returns at once and orders the read)
      if (!__all_sync(0xffffffffu, wait_b(&kv_full[j % NKV], (j / NKV) & 1, abort_v, P.err))) {
        failed = true;
        break;
      }
      const int blk_ok = kv_ok[j % NKV];
      // visible columns i of this block: [a, e) and a loaded page tile; a warp-uniform branch
      // takes the unmasked form for blocks every row sees whole, and the mask is built with
      // non-short-circuit operators (selects, no per-element branches)
      const int a = lo - key_base, e = hi - key_base;
      // raw scores (masked: -inf); the softmax scale (> 0) is applied inside the exponent's FFMA
      float x[64];
      if (__all_sync(0xffffffffu, blk_ok == 15 && a <= 0 && e >= BN)) {
#pragma unroll
        for (int i = 0; i < 64; ++i) x[i] = __uint_as_float(sr[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const bool vis = (i >= a) & (i < e) & (((blk_ok >> (i >> 4)) & 1) != 0);
          x[i] = vis ? __uint_as_float(sr[i]) : -INFINITY;
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; i += 4) {
        mx0 = fmaxf(mx0, x[i]);
        mx1 = fmaxf(mx1, x[i + 1]);
        mx2 = fmaxf(mx2, x[i + 2]);
        mx3 = fmaxf(mx3, x[i + 3]);
      }
      const float c = P.scale_log2;
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * c;
      // The running max is the reference point of this row's O and l.  It is moved (and O, l
      // rescaled by alpha) only when the block's max exceeds it by more than 2^RESCALE_LOG2, so
      // the probabilities stay <= 2^8 (exact in fp16's range) and O / l is unchanged: the same
      // reference point scales numerator and denominator.
      float alpha = 1.f;
      if (mx > m + RESCALE_LOG2 || (m == -INFINITY && mx != -INFINITY)) {
        alpha = fast_exp2(m - mx);  // 0 when the row had no visible key yet
        m = mx;
      }
      const float sub = m != -INFINITY ? m : 0.f;
      float ps0 = 0.f, ps1 = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = fast_exp2(fmaf(x[2 * i], c, -sub)), p1 = fast_exp2(fmaf(x[2 * i + 1], c, -sub));
        ps0 += p0;  // fp32 probabilities feed the row sum, fp16 ones feed P.V
        ps1 += p1;
        pk[i] = pack_half2(p0, p1);
      }
      l = l * alpha + (ps0 + ps1);
      if (j > 0) {  // P.V of the previous block has completed: O is stable, the P tile is free
        if (!__all_sync(0xffffffffu, wait_b(&o_done[t], (j - 1) & 1, abort_v, P.err))) {
          failed = true;
          break;
        }
        tc_fence_after();
        // warp-uniform rescale decision (tcgen05.ld / st are warp-collective)
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            uint32_t o[16];
            tmem_ld16_async(trow + o_col + 16 * c, o);
            tmem_wait_ld16(o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st16(trow + o_col + 16 * c, o);
          }
          tmem_wait_st();
        }
      }
      // probabilities as the A tile of P.V: row r, 64 keys = 128 B, 128-byte swizzle
      uint8_t* prow = ps + t * 16384 + r * 128;  // one P tile per query tile: P.V of block j - 1 has completed
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_plain(&p_full[t]);
    }
    // ---- epilogue: O row / l -> out (dims 0..127 of head kvh * group + r % group)
    if (!failed && nblk > 0) {
      failed = !__all_sync(0xffffffffu, wait_b(&o_done[t], (nblk - 1) & 1, abort_v, P.err));
      tc_fence_after();
    }
    failed = __any_sync(0xffffffffu, failed || *abort_v != 0);
    const float inv = (valid && l > 0.f && !failed) ? P.v_scale / l : 0.f;
    TO* op = reinterpret_cast<TO*>(P.out) + (int64_t)(q_begin + tok) * P.o_st +
             (int64_t)(kvh * P.group + R % P.group) * P.o_sh;
#pragma unroll 1
    for (int c = 0; c < D / 16; ++c) {
      uint32_t o[16];
      if (nblk > 0 && !failed) {
        tmem_ld16_async(trow + o_col + 16 * c, o);
        tmem_wait_ld16(o);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = 0u;
      }
      if (valid) {
        float f[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(o[i]) * inv;
        *reinterpret_cast<uint4*>(op + 16 * c) = pack8<TO>(f);
        *reinterpret_cast<uint4*>(op + 16 * c + 8) = pack8<TO>(f + 8);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

template <typename TQ, typename TO>
inline bool tc_smem_ready() {
  static std::atomic<bool> done[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (done[dev]) return true;
  if (cudaFuncSetAttribute(prefill_tc_kernel<TQ, TO>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) !=
      cudaSuccess)
    return false;
  done[dev] = true;
  return true;
}
}  // namespace tc

}  // namespace pf
}  // namespace ada

using namespace ada;

extern "C" int ada_fp8_paged_prefill(const void* q, int q_dtype, int64_t q_stride_t, int64_t q_stride_h,
                                     const uint8_t* k_cache, const uint8_t* v_cache, int64_t kv_stride_page,
                                     int64_t kv_stride_tok, int64_t kv_stride_head, int64_t num_pages,
                                     const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                                     const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t batch,
                                     int32_t max_seqlen_q, int32_t num_heads, int32_t num_kv_heads,
                                     int32_t head_dim, int32_t page_size, float scale, float k_scale,
                                     float v_scale, int32_t window, void* out, int out_dtype, int64_t out_stride_t,
                                     int64_t out_stride_h, unsigned int* err, void* stream) {
  if (batch < 0 || max_seqlen_q < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_pages <= 0 || page_size <= 0)
    return ADA_ERR_INVALID_ARG;
  if (batch == 0 || max_seqlen_q == 0) return ADA_OK;
  if (!q || !k_cache || !v_cache || !block_tables || !cu_seqlens_q || !cu_seqlens_k || !out)
    return ADA_ERR_INVALID_ARG;
  if ((q_dtype != ADA_DT_BF16 && q_dtype != ADA_DT_F16) || (out_dtype != ADA_DT_BF16 && out_dtype != ADA_DT_F16))
    return ADA_ERR_INVALID_ARG;
  if (head_dim != pf::D) return ADA_ERR_UNSUPPORTED;
  if (num_heads % num_kv_heads != 0) return ADA_ERR_INVALID_ARG;
  const int group = num_heads / num_kv_heads;
  if (group > pf::tc::NT * pf::tc::BM) return ADA_ERR_UNSUPPORTED;
  if (page_size % pf::TILE != 0) return ADA_ERR_UNSUPPORTED;
  if (window < 0 || bt_stride < max_pages || num_pages <= 0) return ADA_ERR_INVALID_ARG;
  if (!(scale * k_scale > 0.f)) return ADA_ERR_INVALID_ARG;  // the row max is taken on unscaled scores
  if ((int64_t)max_pages * page_size > (1LL << 30)) return ADA_ERR_UNSUPPORTED;
  if (((uintptr_t)k_cache | (uintptr_t)v_cache) & 15) return ADA_ERR_ALIGNMENT;
  if ((kv_stride_page | kv_stride_tok | kv_stride_head) & 15) return ADA_ERR_ALIGNMENT;
  if (((uintptr_t)q & 15) || (q_stride_t & 7) || (q_stride_h & 7)) return ADA_ERR_ALIGNMENT;
  if (((uintptr_t)out & 15) || (out_stride_t & 7) || (out_stride_h & 7)) return ADA_ERR_ALIGNMENT;
  if (((uintptr_t)err & 3)) return ADA_ERR_ALIGNMENT;

  pf::Params P;
  P.q = q;
  P.q_st = q_stride_t;
  P.q_sh = q_stride_h;
  P.out = out;
  P.o_st = out_stride_t;
  P.o_sh = out_stride_h;
  P.bt = block_tables;
  P.bt_stride = bt_stride;
  P.num_pages = num_pages;
  P.max_pages = max_pages;
  P.cu_q = cu_seqlens_q;
  P.cu_k = cu_seqlens_k;
  P.group = group;
  P.qt = pf::tc::NT * pf::tc::BM / group;
  P.page = page_size;
  P.window = window;
  P.scale_log2 = scale * k_scale * pf::LOG2E;
  P.v_scale = v_scale;
  P.err = err;

  CUtensorMap tmk, tmv;
  const cuuint64_t dims[4] = {(cuuint64_t)head_dim, (cuuint64_t)num_kv_heads, (cuuint64_t)page_size,
                              (cuuint64_t)num_pages};
  const cuuint64_t strides[3] = {(cuuint64_t)kv_stride_head, (cuuint64_t)kv_stride_tok, (cuuint64_t)kv_stride_page};
  const cuuint32_t box[4] = {(cuuint32_t)head_dim, 1, (cuuint32_t)pf::TILE, 1};
  if (!sm100::encode_bytes(&tmk, k_cache, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !sm100::encode_bytes(&tmv, v_cache, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
    return ADA_ERR_CUDA;

  const int64_t qblocks = cdiv(max_seqlen_q, P.qt);
  if (qblocks > 0x7fffffff || num_kv_heads > 65535 || batch > 65535) return ADA_ERR_UNSUPPORTED;
  const dim3 grid((unsigned)qblocks, (unsigned)num_kv_heads, (unsigned)batch);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define ADA_PF(TQ, TO)                                                                                        \
  do {                                                                                                        \
    if (!pf::tc::tc_smem_ready<TQ, TO>()) return ADA_ERR_CUDA;                                                \
    (void)ada::launch_k(pf::tc::prefill_tc_kernel<TQ, TO>, grid, dim3(pf::tc::THREADS), pf::tc::SMEM, st, tmk, tmv, \
                        P);                                                                                   \
  } while (0)
  if (q_dtype == ADA_DT_BF16) {
    if (out_dtype == ADA_DT_BF16) ADA_PF(__nv_bfloat16, __nv_bfloat16); else ADA_PF(__nv_bfloat16, __half);
  } else {
    if (out_dtype == ADA_DT_BF16) ADA_PF(__half, __nv_bfloat16); else ADA_PF(__half, __half);
  }
#undef ADA_PF
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}
