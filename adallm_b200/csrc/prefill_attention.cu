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
// Work split.  One CTA per (64-row query block, KV head, sequence): the 64 rows are
// (token, head) pairs of the GQA group, head fastest, so QT = 64 / group consecutive query
// tokens share every K/V tile the CTA loads (each e4m3 byte is read once per query block, not
// once per head).  Warp 4 is the producer: one lane walks the block table and issues TMA loads
// of 16-token K and V tiles (4-D tensor map over [pages][page][Hkv][128] bytes, 128-byte
// swizzle) into a ring of stages; warps 0-3 each own 16 rows and run the flash-attention
// recurrence with mma.sync m16n8k16 (f16 in, f32 accumulate): S = Q . K^T (rows x 16 keys),
// online softmax on the S fragments, O += P . V with P taken straight from the S fragments.
// Query blocks are dealt last-first so the longest causal rows start first.
//
// Fragment layouts.  For Q . K^T the head dimension is permuted (identically for Q and K, so
// the dot product is unchanged) so that thread (g, c) reads bytes [32c, 32c+32) of keys g and
// g+8; for P . V the output dimension is permuted so that thread (g, c) reads bytes
// [16g, 16g+16) of keys 2c, 2c+1, 2c+8, 2c+9 and ends up holding dims [32c, 32c+32) of its
// rows: 16-byte shared-memory reads, conflict-free through the swizzle, and 64-byte row stores.
#include "common.cuh"
#include "sm100.cuh"

namespace ada {
namespace pf {

constexpr int D = 128;
constexpr int TILE = 16;
constexpr int TILE_BYTES = TILE * D;       // 16 keys x 128 e4m3 bytes
constexpr int STAGE_BYTES = 2 * TILE_BYTES;  // K tile, V tile
constexpr int STAGES = 8;
constexpr int KB = 4;                      // tiles per online-softmax step (64 keys)
constexpr int ROWS = 64;                   // (token, head) rows per CTA
constexpr int MMA_WARPS = 4;
constexpr int THREADS = (MMA_WARPS + 1) * 32;
constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 2 * STAGES * 8 + STAGES * 4 + 16;
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

__device__ __forceinline__ uint4 tile_ld16(const uint8_t* tile, int row, int chunk) {
  return *reinterpret_cast<const uint4*>(tile + row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Key range [lo, hi) visible to query token t (0-based among the new tokens).
__device__ __forceinline__ void key_range(const Params& P, int t, int off, int len_k, int& lo, int& hi) {
  hi = min(len_k, t + off + 1);
  lo = P.window > 0 ? max(0, t + off - P.window) : 0;
}

// Q rows g and g+8 of this warp, dims [32c, 32c+32), as the A operand of the score MMA:
// qa[4s + 0/1] = row g / g+8, dims 32c+4s+{0,1}; qa[4s + 2/3] = row g / g+8, dims 32c+4s+{2,3}.
template <typename TQ>
__device__ __forceinline__ void load_q(const Params& P, const TQ* q0, bool ok0, const TQ* q8, bool ok8,
                                       uint32_t* qa) {
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const TQ* qp = half ? q8 : q0;
    const bool ok = half ? ok8 : ok0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float f[8];
      if (ok) {
        unpack8<TQ>(*reinterpret_cast<const uint4*>(qp + 8 * i), f);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = 0.f;
      }
      // dims 32c + 8i + e: k-steps s = 2i (e 0..3) and 2i+1 (e 4..7)
      qa[4 * (2 * i) + half] = pack_half2(f[0], f[1]);
      qa[4 * (2 * i) + 2 + half] = pack_half2(f[2], f[3]);
      qa[4 * (2 * i + 1) + half] = pack_half2(f[4], f[5]);
      qa[4 * (2 * i + 1) + 2 + half] = pack_half2(f[6], f[7]);
    }
  }
}

template <typename TQ, typename TO>
__global__ void __launch_bounds__(THREADS, 2)
    prefill_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, Params P) {
  using namespace sm100;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, kvh = blockIdx.y;
  const int qblk = gridDim.x - 1 - blockIdx.x;  // longest causal rows first

  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  int* slot_ok = reinterpret_cast<int*>(empty + STAGES);
  int* abort_flag = slot_ok + STAGES;
  volatile int* abort_v = abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], MMA_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // q, the cache pages and the metadata come from earlier kernels
  pdl_trigger();

  const int q_begin = __ldg(P.cu_q + b);
  const int len_q = __ldg(P.cu_q + b + 1) - q_begin;
  const int len_k = __ldg(P.cu_k + b + 1) - __ldg(P.cu_k + b);
  const int t0 = qblk * P.qt;  // first query token of the block
  if (t0 >= len_q) return;     // CTA-uniform, before any wait or load
  const int t_last = min(t0 + P.qt, len_q) - 1;
  const int off = len_k - len_q;
  // keys any row of the block can see; the table reaches max_pages * page keys at most
  int k_lo, k_hi, dummy_lo, dummy_hi;
  key_range(P, t0, off, len_k, k_lo, dummy_hi);
  key_range(P, t_last, off, len_k, dummy_lo, k_hi);
  k_hi = min(k_hi, P.max_pages * P.page);
  const int kt0 = k_lo / TILE;
  const int ntiles = k_hi > k_lo ? (k_hi + TILE - 1) / TILE - kt0 : 0;

  if (warp == MMA_WARPS) {  // ---------------- producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < ntiles && !*abort_v; ++i) {
        const int s = i % STAGES;
        if (i >= STAGES && !mbar_wait_bounded(&empty[s], ((i / STAGES) - 1) & 1, abort_v, P.err, ERR_TILE_WAIT))
          break;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const int key0 = (kt0 + i) * TILE;
        const int page_idx = key0 / P.page;
        int blk = __ldg(P.bt + (int64_t)b * P.bt_stride + page_idx);
        if (blk < 0 || blk >= P.num_pages) blk = -1;
        slot_ok[s] = blk >= 0;
        if (blk >= 0) {
          uint8_t* st = ring + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          tma_load_4d(st, &tmk, &full[s], 0, kvh, key0 - page_idx * P.page, blk);
          tma_load_4d(st + TILE_BYTES, &tmv, &full[s], 0, kvh, key0 - page_idx * P.page, blk);
        } else {
          mbar_arrive_plain(&full[s]);  // a hole in the block table: nothing to load
        }
        issued = i + 1;
      }
      // leave no copy in flight when the CTA ends: wait (bounded) for the last use of each slot
      for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i) {
        const int s = i % STAGES;
        uint32_t spins = 0;
        const uint64_t t_start = globaltimer();
        while (!mbar_try_wait(&full[s], (i / STAGES) & 1)) {
          if ((++spins & 63u) == 0 && globaltimer() - t_start > 2000000000ull) {
            if (P.err) atomicOr(P.err, ERR_TILE_WAIT);
            break;
          }
        }
      }
    }
    return;
  }

  // ---------------- consumers: warps 0..3, rows 16 * warp + {g, g + 8} ----------------
  const int g = lane >> 2, c = lane & 3;
  const int r0 = 16 * warp + g, r8 = r0 + 8;
  const int used = P.qt * P.group;  // rows past this are padding
  const int tok0 = t0 + r0 / P.group, tok8 = t0 + r8 / P.group;
  const bool ok0 = r0 < used && tok0 < len_q, ok8 = r8 < used && tok8 < len_q;
  const int h0 = kvh * P.group + r0 % P.group, h8 = kvh * P.group + r8 % P.group;
  int lo0, hi0, lo8, hi8;
  key_range(P, tok0, off, len_k, lo0, hi0);
  key_range(P, tok8, off, len_k, lo8, hi8);
  if (!ok0) hi0 = lo0;  // padding rows see nothing
  if (!ok8) hi8 = lo8;

  const TQ* qbase = reinterpret_cast<const TQ*>(P.q);
  uint32_t qa[32];
  load_q<TQ>(P, qbase + (int64_t)(q_begin + tok0) * P.q_st + (int64_t)h0 * P.q_sh + 32 * c, ok0,
             qbase + (int64_t)(q_begin + tok8) * P.q_st + (int64_t)h8 * P.q_sh + 32 * c, ok8, qa);

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m8 = -INFINITY, l0 = 0.f, l8 = 0.f;
  const uint4 z = make_uint4(0, 0, 0, 0);

  bool failed = false;
  for (int i0 = 0; i0 < ntiles && !failed; i0 += KB) {
    // ---- S = Q . K^T over KB tiles (64 keys): tile u, n-block j covers keys key0(u) + 8j .. +8
    float sc[KB][2][4];
    bool blk_ok[KB];
#pragma unroll
    for (int u = 0; u < KB; ++u) {
      sc[u][0][0] = sc[u][0][1] = sc[u][0][2] = sc[u][0][3] = 0.f;
      sc[u][1][0] = sc[u][1][1] = sc[u][1][2] = sc[u][1][3] = 0.f;
      blk_ok[u] = false;
      const int i = i0 + u;
      if (i >= ntiles) continue;  // warp-uniform
      const int s = i % STAGES;
      // a wait that ran out marks the step failed; its (stale) tile is computed and discarded
      if (!failed && !mbar_wait_bounded(&full[s], (i / STAGES) & 1, abort_v, P.err, ERR_TILE_WAIT)) failed = true;
      blk_ok[u] = slot_ok[s] != 0;
      const uint8_t* kt = ring + s * STAGE_BYTES;
      uint4 kg[2], kg8[2];
      kg[0] = tile_ld16(kt, g, 2 * c);
      kg[1] = tile_ld16(kt, g, 2 * c + 1);
      kg8[0] = tile_ld16(kt, g + 8, 2 * c);
      kg8[1] = tile_ld16(kt, g + 8, 2 * c + 1);
      const uint32_t* kw = reinterpret_cast<const uint32_t*>(kg);
      const uint32_t* kw8 = reinterpret_cast<const uint32_t*>(kg8);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t b0[2], b1[2];
        b0[0] = e4m3x2_to_f16x2((uint16_t)(kw[ks] & 0xFFFFu));
        b0[1] = e4m3x2_to_f16x2((uint16_t)(kw[ks] >> 16));
        b1[0] = e4m3x2_to_f16x2((uint16_t)(kw8[ks] & 0xFFFFu));
        b1[1] = e4m3x2_to_f16x2((uint16_t)(kw8[ks] >> 16));
        mma_16816_f16(sc[u][0], &qa[4 * ks], b0);
        mma_16816_f16(sc[u][1], &qa[4 * ks], b1);
      }
    }
    if (failed) break;

    // ---- masks, one online-softmax step for the 64 keys (rows g: [..][0..1], rows g+8: [..][2..3])
    float mx0 = -INFINITY, mx8 = -INFINITY;
#pragma unroll
    for (int u = 0; u < KB; ++u) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = (kt0 + i0 + u) * TILE + 8 * j + 2 * c + e;
          sc[u][j][e] = (blk_ok[u] && key >= lo0 && key < hi0) ? sc[u][j][e] * P.scale_log2 : -INFINITY;
          sc[u][j][2 + e] = (blk_ok[u] && key >= lo8 && key < hi8) ? sc[u][j][2 + e] * P.scale_log2 : -INFINITY;
          mx0 = fmaxf(mx0, sc[u][j][e]);
          mx8 = fmaxf(mx8, sc[u][j][2 + e]);
        }
      }
    }
#pragma unroll
    for (int sh = 1; sh < 4; sh <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
      mx8 = fmaxf(mx8, __shfl_xor_sync(0xffffffffu, mx8, sh));
    }
    const float mn0 = fmaxf(m0, mx0), mn8 = fmaxf(m8, mx8);
    const float al0 = mn0 != -INFINITY ? fast_exp2(m0 - mn0) : 1.f;
    const float al8 = mn8 != -INFINITY ? fast_exp2(m8 - mn8) : 1.f;
    const float sub0 = mn0 != -INFINITY ? mn0 : 0.f;  // exp2(-inf - 0) = 0 for a row with nothing yet
    const float sub8 = mn8 != -INFINITY ? mn8 : 0.f;
    m0 = mn0;
    m8 = mn8;
    float ps0 = 0.f, ps8 = 0.f;
    uint32_t pa[KB][4];
#pragma unroll
    for (int u = 0; u < KB; ++u) {
      float p[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        p[j][0] = fast_exp2(sc[u][j][0] - sub0);
        p[j][1] = fast_exp2(sc[u][j][1] - sub0);
        p[j][2] = fast_exp2(sc[u][j][2] - sub8);
        p[j][3] = fast_exp2(sc[u][j][3] - sub8);
      }
      // fp32 probabilities feed the row sums, fp16 ones feed P.V; the S accumulator layout is
      // the A-operand layout of P . V (keys 2c.. in a0/a1, 2c+8.. in a2/a3)
      ps0 += (p[0][0] + p[0][1]) + (p[1][0] + p[1][1]);
      ps8 += (p[0][2] + p[0][3]) + (p[1][2] + p[1][3]);
      pa[u][0] = pack_half2(p[0][0], p[0][1]);
      pa[u][1] = pack_half2(p[0][2], p[0][3]);
      pa[u][2] = pack_half2(p[1][0], p[1][1]);
      pa[u][3] = pack_half2(p[1][2], p[1][3]);
    }
    l0 = l0 * al0 + ps0;
    l8 = l8 * al8 + ps8;
#pragma unroll
    for (int nb = 0; nb < 16; ++nb) {
      o[nb][0] *= al0;
      o[nb][1] *= al0;
      o[nb][2] *= al8;
      o[nb][3] *= al8;
    }

    // ---- O += P . V, tile by tile; keys past len_k and holes may hold stale bytes (NaN in
    // e4m3): their V rows are zeroed
#pragma unroll
    for (int u = 0; u < KB; ++u) {
      const int i = i0 + u;
      if (i >= ntiles) continue;  // warp-uniform
      const int s = i % STAGES;
      const uint8_t* vt = ring + s * STAGE_BYTES + TILE_BYTES;
      const int key0 = (kt0 + i) * TILE;
      uint4 vv[4];
      const int vk[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
#pragma unroll
      for (int e = 0; e < 4; ++e) vv[e] = (blk_ok[u] && key0 + vk[e] < len_k) ? tile_ld16(vt, vk[e], g) : z;
      const uint32_t* v0 = reinterpret_cast<const uint32_t*>(&vv[0]);
      const uint32_t* v1 = reinterpret_cast<const uint32_t*>(&vv[1]);
      const uint32_t* v8 = reinterpret_cast<const uint32_t*>(&vv[2]);
      const uint32_t* v9 = reinterpret_cast<const uint32_t*>(&vv[3]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t sel = half ? 0x7362u : 0x5140u;
          const uint32_t w01 = prmt(v0[j], v1[j], sel);  // dims 16g + 4j + 2half + {0, 1}, keys 2c, 2c+1
          const uint32_t w89 = prmt(v8[j], v9[j], sel);  // same dims, keys 2c+8, 2c+9
          uint32_t bv[2];
          bv[0] = e4m3x2_to_f16x2((uint16_t)(w01 & 0xFFFFu));
          bv[1] = e4m3x2_to_f16x2((uint16_t)(w89 & 0xFFFFu));
          mma_16816_f16(o[4 * j + 2 * half], pa[u], bv);
          bv[0] = e4m3x2_to_f16x2((uint16_t)(w01 >> 16));
          bv[1] = e4m3x2_to_f16x2((uint16_t)(w89 >> 16));
          mma_16816_f16(o[4 * j + 2 * half + 1], pa[u], bv);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_plain(&empty[s]);  // this warp is done with the slot
    }
  }

  // ---- normalise and store: thread holds dims [32c, 32c+32) of rows g and g+8 ----
#pragma unroll
  for (int sh = 1; sh < 4; sh <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, sh);
    l8 += __shfl_xor_sync(0xffffffffu, l8, sh);
  }
  failed = failed || *abort_v != 0;
  const float inv0 = (l0 > 0.f && !failed) ? P.v_scale / l0 : 0.f;
  const float inv8 = (l8 > 0.f && !failed) ? P.v_scale / l8 : 0.f;
  TO* obase = reinterpret_cast<TO*>(P.out);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const bool ok = half ? ok8 : ok0;
    if (!ok) continue;
    const float inv = half ? inv8 : inv0;
    TO* op = obase + (int64_t)(q_begin + (half ? tok8 : tok0)) * P.o_st + (int64_t)(half ? h8 : h0) * P.o_sh + 32 * c;
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // dims 32c + 8i .. +8: i < 2 from o[.][0/2] (nb = 8i..), else o[.][1/3]
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int dd = 8 * i + e;  // 0..31
        const int nb = dd & 15;
        f[e] = o[nb][(dd >> 4) + 2 * half] * inv;
      }
      *reinterpret_cast<uint4*>(op + 8 * i) = pack8<TO>(f);
    }
  }
}

template <typename TQ, typename TO>
inline bool smem_ready() {
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (done[dev]) return true;
  if (cudaFuncSetAttribute(prefill_kernel<TQ, TO>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
    return false;
  done[dev] = true;
  return true;
}

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
  if (group > pf::ROWS) return ADA_ERR_UNSUPPORTED;
  if (page_size % pf::TILE != 0) return ADA_ERR_UNSUPPORTED;
  if (window < 0 || bt_stride < max_pages || num_pages <= 0) return ADA_ERR_INVALID_ARG;
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
  P.qt = pf::ROWS / group;
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
#define ADA_PF(TQ, TO)                                                                                  \
  do {                                                                                                  \
    if (!pf::smem_ready<TQ, TO>()) return ADA_ERR_CUDA;                                                 \
    (void)ada::launch_k(pf::prefill_kernel<TQ, TO>, grid, dim3(pf::THREADS), pf::SMEM, st, tmk, tmv, P); \
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
