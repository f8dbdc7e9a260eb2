// FP8 paged split-K decode attention for B200 (sm_100a).
//
// Replaces fp8_kv_decode_group_kernel (reference adallm/ops/attention.py:126-233).
// Same math: per (sequence, kv head) the Hq/Hkv query heads of the GQA group
// attend to tokens [start, ctx) of the paged e4m3 cache, with q rounded to
// fp16, K/V widened to fp16, fp32 scores and softmax statistics, fp16
// probabilities for P.V and fp32 accumulation.  Differences by design:
//   * split-K over the context (flash-decoding): each warp takes splits of 64-512 tokens of
//     one (sequence, kv head) -- the length chosen per launch so the work fits one wave of
//     the grid -- and writes an unnormalised partial (max, sum, O) to the workspace; a
//     reduction kernel merges the splits;
//   * the page walk is exact for any page size that is a multiple of 16
//     (the reference reads past a page for pages < 64);
//   * optional per-tensor k_scale / v_scale (1.0 reproduces the reference).
//
// Tile = 16 tokens of one page.  Each warp streams its split's tiles through its own ring of
// RING slots: lane 0 issues a TMA load (4-D tensor map over [pages][page][Hkv][D] bytes,
// 128-byte swizzle, one mbarrier per slot) of a tile's K and V rows, gathered page by page
// through the block table, and refills a slot as soon as the tile in it has been consumed.
// The warp computes S^T = K_tile . Q^T with mma.m16n8k16 (tokens on M,
// heads on N), an online softmax per head, and O^T += V_tile^T . P^T.  For the K operand
// the head dimension is permuted so that thread (g, c) needs bytes [32c, 32c+32) of tokens
// g and g+8 (the permutation is applied to Q identically); for the V operand the output
// dimension is permuted so thread (g, c) needs bytes [16g, 16g+16) of tokens 2c, 2c+1,
// 2c+8, 2c+9: 16-byte shared-memory reads, conflict-free through the swizzle.
#include "cluster.cuh"
#include "quant.cuh"
#include "sm100.cuh"

namespace ada {
namespace attn {

constexpr int D = 128;
constexpr int TILE = 16;
// Split length of the long-cache kernel, in tiles of 16 tokens: chosen per launch on the device
// (split_tiles_for) between CT_MIN and CT_MAX (one lane per tile holds the split's page ids).
constexpr int CT_MIN = 4;
constexpr int CT_MAX = 32;
constexpr int TILE_BYTES = TILE * D;  // one K (or V) tile: 16 rows x 128 bytes
constexpr float LOG2E = 1.4426950408889634f;

struct Params {
  const void* q;
  int64_t q_sb, q_sh;
  const uint8_t* k;
  const uint8_t* v;
  int64_t s_page, s_tok, s_head;
  int64_t num_pages;  // pool size: block ids outside [0, num_pages) are treated as holes
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* ctx;
  int32_t num_heads, group, page, window, max_splits, max_pages;
  float scale_log2;  // softmax scale * k_scale * log2(e)
  float v_scale;
  float* o_part;   // [B][Hq][max_splits][D]
  float* ml_part;  // [B][Hq][max_splits][2]   (max in log2 units, sum)
  // 1: context_lens, block_tables and every cached K/V row except each sequence's newest
  // position (ctx - 1) were written at least two kernels earlier on the stream, so the
  // short-cache kernel may read them (and start the TMA loads of those tiles) before its
  // programmatic-launch wait; q and the newest row are read after it.
  int early;
  int* split_tiles;  // workspace word: the split length the split kernel chose, for the merges
};

// Tokens beyond the block table's reach (ctx > max_pages * page) cannot be addressed and are
// dropped, so every index below stays inside the table and the workspace.
__device__ __forceinline__ int clamp_ctx(const Params& P, int ctx) {
  return min(ctx, P.max_pages * P.page);
}

// Tokens [start, ctx) of a sequence are attended (start > 0 with a sliding window); its splits of
// ct tiles begin at the tile-aligned start16.
__device__ __forceinline__ void seq_range(const Params& P, int ctx, int ct, int& start, int& start16, int& nsplit) {
  start = P.window > 0 ? max(ctx - P.window, 0) : 0;
  start16 = start & ~15;
  const int chunk = ct * TILE;
  nsplit = ctx > 0 ? min((ctx - start16 + chunk - 1) / chunk, P.max_splits) : 0;
}

// Warp-wide: work items (sequence, split of ct tiles, KV head) of the launch.
__device__ __forceinline__ int split_items(const Params& P, int batch, int num_kv_heads, int ct) {
  int n = 0;
  for (int b = (int)(threadIdx.x & 31); b < batch; b += 32) {
    int st, st16, ns;
    seq_range(P, clamp_ctx(P, __ldg(P.ctx + b)), ct, st, st16, ns);
    n += ns;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
  return n * num_kv_heads;
}
// Warp-wide: the split length of this launch -- the shortest split (most parallel work) whose
// items all fit in one wave of the grid's `warps`, found by bisection (items only fall as splits
// grow); CT_MAX when even that needs several waves.  A first wave of whole splits saturates HBM
// (a KV page's heads are read by neighbouring warps together), while the warps of a second,
// partial wave run alone, each latency-bound on its own ring.  Integer arithmetic on the
// context lengths only, so every warp gets the same answer.
__device__ __forceinline__ int split_tiles_for(const Params& P, int batch, int num_kv_heads, int warps) {
  const int lane = threadIdx.x & 31;
  if (batch <= 32) {  // one lane per candidate length; the sequences' tile counts read once
    int tiles = 0;
    if (lane < batch) {
      int st, st16, ns;
      const int ctx = clamp_ctx(P, __ldg(P.ctx + lane));
      seq_range(P, ctx, CT_MAX, st, st16, ns);
      tiles = ctx > 0 ? (ctx - st16 + TILE - 1) / TILE : 0;
    }
    // items(ct) >= total tiles x heads / ct: start at that bound and lengthen until one wave holds
    int total = tiles;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    const int64_t need = (int64_t)total * num_kv_heads;
    int ct = (int)max((int64_t)CT_MIN, (need + warps - 1) / warps);
    for (; ct < CT_MAX; ++ct) {
      int n = min((tiles + ct - 1) / ct, P.max_splits);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
      if ((int64_t)n * num_kv_heads <= warps) break;
    }
    return min(ct, CT_MAX);
  }
  if (split_items(P, batch, num_kv_heads, CT_MAX) > warps) return CT_MAX;
  int lo = CT_MIN, hi = CT_MAX;  // items(hi) <= warps
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (split_items(P, batch, num_kv_heads, mid) <= warps)
      hi = mid;
    else
      lo = mid + 1;
  }
  return lo;
}

// 16 bytes at (row, 16-byte chunk) of a 128-byte-swizzled tile (chunk index XOR row % 8).
__device__ __forceinline__ uint4 tile_ld16(const uint8_t* tile, int row, int chunk) {
  return *reinterpret_cast<const uint4*>(tile + row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Q operand (B of the score MMA) of the GQA group of KV head kvh: head g of the group,
// d in [32c, 32c+32), fp16 as the reference (attention.py:314-324).  qf[2s], qf[2s+1] = k-step s.
template <typename TQ>
__device__ __forceinline__ void load_q_frag(const Params& P, int b, int kvh, int g, int c, uint32_t* qf) {
  if (g < P.group) {
    const TQ* qp =
        reinterpret_cast<const TQ*>(P.q) + (int64_t)b * P.q_sb + (int64_t)(kvh * P.group + g) * P.q_sh + 32 * c;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float f[8];
      unpack8<TQ>(*reinterpret_cast<const uint4*>(qp + 8 * i), f);
      qf[4 * i + 0] = pack_half2(f[0], f[1]);
      qf[4 * i + 1] = pack_half2(f[2], f[3]);
      qf[4 * i + 2] = pack_half2(f[4], f[5]);
      qf[4 * i + 3] = pack_half2(f[6], f[7]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) qf[i] = 0u;
  }
}

// Online-softmax state of one warp over the tiles it has seen: O^T fragments (d = 16g + 2mt
// (+1), heads 2c / 2c+1) and per head pair the running max (log2 units) and sum.
struct WarpState {
  float acc[8][4];
  float m0, m1, l0, l1;
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
  }
};

// Fold one 16-token tile (K at kt, V at kt + TILE_BYTES, 128-byte swizzled) into the warp's
// state.  Tokens outside [lo, t1) or of a hole in the block table get probability 0.
__device__ __forceinline__ void attn_tile(const Params& P, const uint8_t* kt, bool blk_ok, int tt, int ctx, int lo,
                                          int t1, const uint32_t* qf, WarpState& st, __half (*p_s)[16], int g,
                                          int c) {
  const uint8_t* vt = kt + TILE_BYTES;
  uint4 k0[2], k8[2], vv[4];
  k0[0] = tile_ld16(kt, g, 2 * c);
  k0[1] = tile_ld16(kt, g, 2 * c + 1);
  k8[0] = tile_ld16(kt, g + 8, 2 * c);
  k8[1] = tile_ld16(kt, g + 8, 2 * c + 1);
  const int toks[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
  const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // Rows at or past ctx (and holes) may hold stale or uninitialised bytes (NaN in
    // e4m3); they get probability 0, so their V must be finite: zero them.
    vv[i] = (blk_ok && tt + toks[i] < ctx) ? tile_ld16(vt, toks[i], g) : z;
  }

  // ---- scores S^T[token][head] -------------------------------------------
  float sc[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t* kg = reinterpret_cast<const uint32_t*>(k0);
  const uint32_t* kg8 = reinterpret_cast<const uint32_t*>(k8);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    uint32_t a[4];
    a[0] = e4m3x2_to_f16x2((uint16_t)(kg[ks] & 0xFFFFu));
    a[1] = e4m3x2_to_f16x2((uint16_t)(kg8[ks] & 0xFFFFu));
    a[2] = e4m3x2_to_f16x2((uint16_t)(kg[ks] >> 16));
    a[3] = e4m3x2_to_f16x2((uint16_t)(kg8[ks] >> 16));
    mma_16816_f16(sc, a, &qf[2 * ks]);
  }
  const int tg = tt + g, tg8 = tt + g + 8;
  const bool vg = blk_ok && tg >= lo && tg < t1;
  const bool vg8 = blk_ok && tg8 >= lo && tg8 < t1;
  const float x0 = vg ? sc[0] * P.scale_log2 : -INFINITY;   // token g,   head 2c
  const float x1 = vg ? sc[1] * P.scale_log2 : -INFINITY;   // token g,   head 2c+1
  const float x2 = vg8 ? sc[2] * P.scale_log2 : -INFINITY;  // token g+8, head 2c
  const float x3 = vg8 ? sc[3] * P.scale_log2 : -INFINITY;  // token g+8, head 2c+1
  float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
  }
  const float mn0 = fmaxf(st.m0, mx0), mn1 = fmaxf(st.m1, mx1);
  float al0 = 1.f, al1 = 1.f, p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
  if (mn0 != -INFINITY) {
    al0 = fast_exp2(st.m0 - mn0);
    p0 = fast_exp2(x0 - mn0);
    p2 = fast_exp2(x2 - mn0);
  }
  if (mn1 != -INFINITY) {
    al1 = fast_exp2(st.m1 - mn1);
    p1 = fast_exp2(x1 - mn1);
    p3 = fast_exp2(x3 - mn1);
  }
  st.m0 = mn0;
  st.m1 = mn1;
  // fp32 probabilities feed the row sum, fp16 ones feed P.V (attention.py:219-223)
  const __half hp0 = __float2half_rn(p0), hp1 = __float2half_rn(p1);
  const __half hp2 = __float2half_rn(p2), hp3 = __float2half_rn(p3);
  st.l0 = st.l0 * al0 + (p0 + p2);
  st.l1 = st.l1 * al1 + (p1 + p3);
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    st.acc[mt][0] *= al0;
    st.acc[mt][1] *= al1;
    st.acc[mt][2] *= al0;
    st.acc[mt][3] *= al1;
  }
  // ---- transpose P through shared memory: P^T operand wants (token pairs, head g)
  p_s[2 * c][g] = hp0;
  p_s[2 * c + 1][g] = hp1;
  p_s[2 * c][g + 8] = hp2;
  p_s[2 * c + 1][g + 8] = hp3;
  __syncwarp();
  uint32_t bp[2];
  bp[0] = *reinterpret_cast<const uint32_t*>(&p_s[g][2 * c]);
  bp[1] = *reinterpret_cast<const uint32_t*>(&p_s[g][2 * c + 8]);
  __syncwarp();

  // ---- O^T[d][head] += V^T . P^T ----------------------------------------
  const uint32_t* v0 = reinterpret_cast<const uint32_t*>(&vv[0]);
  const uint32_t* v1 = reinterpret_cast<const uint32_t*>(&vv[1]);
  const uint32_t* v8 = reinterpret_cast<const uint32_t*>(&vv[2]);
  const uint32_t* v9 = reinterpret_cast<const uint32_t*>(&vv[3]);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t sel = half ? 0x7362u : 0x5140u;
      const uint32_t lo01 = prmt(v0[j], v1[j], sel);
      const uint32_t lo89 = prmt(v8[j], v9[j], sel);
      uint32_t a[4];
      a[0] = e4m3x2_to_f16x2((uint16_t)(lo01 & 0xFFFFu));
      a[1] = e4m3x2_to_f16x2((uint16_t)(lo01 >> 16));
      a[2] = e4m3x2_to_f16x2((uint16_t)(lo89 & 0xFFFFu));
      a[3] = e4m3x2_to_f16x2((uint16_t)(lo89 >> 16));
      mma_16816_f16(st.acc[2 * j + half], a, bp);
    }
  }
}

// One warp = one work item (sequence b, KV head, split) at a time: items are dealt to the
// grid's warps round-robin.  Each warp streams its item's tiles through its own ring of
// RING tile slots (K and V, 4 KB per tile): lane i looks up tile i's page, lane 0 issues the
// TMA loads RING tiles ahead of the tile being computed, and the warp writes the item's
// unnormalised partial (per head: O, max, sum) straight from its registers.
constexpr int RING = 4;
constexpr int SPLIT_WARPS = 4;
constexpr int SPLIT_SMEM_V3 = 1024 + SPLIT_WARPS * RING * 2 * TILE_BYTES + SPLIT_WARPS * RING * 8 + 64;

template <typename TQ>
__global__ void __launch_bounds__(SPLIT_WARPS * 32, 3)
    decode_split_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, Params P,
                        int num_kv_heads, int batch) {
  using namespace sm100;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int group = P.group;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring_base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = ring_base + warp * RING * 2 * TILE_BYTES;
  uint64_t* bar = reinterpret_cast<uint64_t*>(ring_base + SPLIT_WARPS * RING * 2 * TILE_BYTES) + warp * RING;
  int* abort_flag = reinterpret_cast<int*>(reinterpret_cast<uint64_t*>(ring_base + SPLIT_WARPS * RING * 2 * TILE_BYTES) +
                                           SPLIT_WARPS * RING);
  __shared__ __align__(16) __half p_s[SPLIT_WARPS][8][16];

  if (threadIdx.x == 0) *abort_flag = 0;
  if (lane < RING) mbar_init(&bar[lane], 1);
  fence_mbar_init();
  __syncthreads();
  // the split length depends on the context lengths only: with settled metadata (P.early) it is
  // worked out while the previous kernel finishes
  int ct = P.early ? split_tiles_for(P, batch, num_kv_heads, (int)gridDim.x * SPLIT_WARPS) : 0;
  pdl_wait();
  pdl_trigger();
  if (!P.early) ct = split_tiles_for(P, batch, num_kv_heads, (int)gridDim.x * SPLIT_WARPS);
  if (blockIdx.x == 0 && threadIdx.x == 0) *P.split_tiles = ct;  // after the wait: the last merge read it
  const int chunk = ct * TILE;
  uint32_t uses = 0;  // tiles this warp has put through its ring (slot = uses % RING, parity = (uses / RING) & 1)
  // Work items are the splits that hold tokens -- (sequence b, split s < nsplit(b), KV head) in
  // sequence-major order, KV head fastest so neighbouring warps (and CTAs) read the rows of the
  // same pages together -- dealt round-robin to the grid's warps, so every warp gets the same
  // number of live items whatever the spread of context lengths.
  int live = 0;
  for (int bb = lane; bb < batch; bb += 32) {
    int st_, st16_, ns_;
    seq_range(P, clamp_ctx(P, __ldg(P.ctx + bb)), ct, st_, st16_, ns_);
    live += ns_;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) live += __shfl_xor_sync(0xffffffffu, live, o);
  const int items = live * num_kv_heads;
  int cur_b = 0, cur_first = 0, cur_n = 0;  // sequence cur_b owns flat splits [cur_first, cur_first + cur_n)
  {
    int st_, st16_;
    if (batch > 0) seq_range(P, clamp_ctx(P, __ldg(P.ctx)), ct, st_, st16_, cur_n);
  }
  for (int item = blockIdx.x * SPLIT_WARPS + warp; item < items; item += gridDim.x * SPLIT_WARPS) {
    const int kvh = item % num_kv_heads;
    const int flat = item / num_kv_heads;
    while (flat >= cur_first + cur_n && cur_b + 1 < batch) {  // items only move forward: a running cursor
      cur_first += cur_n;
      ++cur_b;
      int st_, st16_;
      seq_range(P, clamp_ctx(P, __ldg(P.ctx + cur_b)), ct, st_, st16_, cur_n);
    }
    const int b = cur_b, s = flat - cur_first;
    const int ctx = clamp_ctx(P, __ldg(P.ctx + b));
    int start, start16, nsplit;
    seq_range(P, ctx, ct, start, start16, nsplit);
    if (s < 0 || s >= nsplit) continue;  // warp-uniform; cannot happen with a consistent cursor
    const int t0 = start16 + s * chunk;
    const int t1 = min(ctx, t0 + chunk);
    const int ntiles = (t1 - t0 + 15) >> 4;
    const int lo = max(start, t0);

    // lane i: page of tile i (lanes >= ntiles: unused)
    int my_block = -1, my_row0 = 0;
    if (lane < ntiles) {
      const int tt = t0 + TILE * lane;
      const int page_idx = tt / P.page;
      my_row0 = tt - page_idx * P.page;
      my_block = __ldg(P.bt + (int64_t)b * P.bt_stride + page_idx);
      if (my_block >= P.num_pages) my_block = -1;
    }
    auto issue = [&](int k, uint32_t use) {  // lane 0 only
      const int blk = __shfl_sync(0xffffffffu, my_block, k);
      const int row0 = __shfl_sync(0xffffffffu, my_row0, k);
      if (lane == 0) {
        const int slot = use % RING;
        uint64_t* bb = &bar[slot];
        if (blk >= 0) {
          mbar_arrive_expect_tx(bb, 2 * TILE_BYTES);
          tma_load_4d(ring + slot * 2 * TILE_BYTES, &tmk, bb, 0, kvh, row0, blk);
          tma_load_4d(ring + slot * 2 * TILE_BYTES + TILE_BYTES, &tmv, bb, 0, kvh, row0, blk);
        } else {
          mbar_arrive_plain(bb);  // a hole in the block table: nothing to load
        }
      }
    };
    for (int k = 0; k < RING && k < ntiles; ++k) issue(k, uses + k);

    uint32_t qf[16];
    load_q_frag<TQ>(P, b, kvh, g, c, qf);
    WarpState ws;
    ws.init();
    bool failed = false;

    for (int k = 0; k < ntiles; ++k) {
      const uint32_t use = uses + k;
      const int slot = use % RING;
      if (!mbar_wait_bounded(&bar[slot], (use / RING) & 1, abort_flag, nullptr, 0u)) {
        failed = true;
        break;
      }
      const bool blk_ok = __shfl_sync(0xffffffffu, my_block, k) >= 0;
      attn_tile(P, ring + slot * 2 * TILE_BYTES, blk_ok, t0 + TILE * k, ctx, lo, t1, qf, ws, p_s[warp], g, c);
      // every byte of the slot has been consumed by the MMAs above: refill it with tile k + RING
      __syncwarp();
      if (k + RING < ntiles) {
        if (lane == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(k + RING, use + RING);
      }
    }
    uses += ntiles;
    float m0 = ws.m0, m1 = ws.m1, l0 = ws.l0, l1 = ws.l1;
    if (failed) {  // a tile never arrived: poison this split's result and stop using the ring
      m0 = m1 = l0 = l1 = __int_as_float(0x7fc00000);
    }

    // ---- this item's partial, straight from the fragments ------------------------
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    const int64_t row0 = ((int64_t)b * P.num_heads + kvh * group + 2 * c) * P.max_splits + s;  // head 2c
    const int64_t row1 = row0 + P.max_splits;                                                  // head 2c+1
    if (2 * c < group) {
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int d = 16 * g + 2 * mt;
        *reinterpret_cast<float2*>(P.o_part + row0 * D + d) =
            make_float2(ws.acc[mt][0] * P.v_scale, ws.acc[mt][2] * P.v_scale);
      }
      if (g == 0) *reinterpret_cast<float2*>(P.ml_part + row0 * 2) = make_float2(m0, l0);
    }
    if (2 * c + 1 < group) {
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int d = 16 * g + 2 * mt;
        *reinterpret_cast<float2*>(P.o_part + row1 * D + d) =
            make_float2(ws.acc[mt][1] * P.v_scale, ws.acc[mt][3] * P.v_scale);
      }
      if (g == 0) *reinterpret_cast<float2*>(P.ml_part + row1 * 2) = make_float2(m1, l1);
    }
    if (failed) break;
  }
}

// ---- short caches: the whole decode attention of a token in one cluster ----------------
// When the cache holds at most FUSED_MAX_TOKENS tokens per sequence, the split/merge pair is
// replaced by one kernel: grid (Hkv, rows), cluster (Hkv, 1, 1) = one CTA per KV head of a
// token.  The 4 warps of a CTA take the token's tiles round-robin (each through its own TMA
// ring), merge their softmax states in shared memory and write the normalised heads of the
// group.  With a quantised output the cluster combines the token row's amax through DSMEM and
// every CTA quantises its heads' slice of the o_proj operand (quant.cuh).
constexpr int FUSED_MAX_TOKENS = 1024;
constexpr int FUSED_SMEM = 1024 + SPLIT_WARPS * RING * 2 * TILE_BYTES + SPLIT_WARPS * RING * 8 + 64;

template <typename TQ, typename TO>
__global__ void __launch_bounds__(SPLIT_WARPS * 32, 3)
    decode_fused_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, Params P,
                        TO* __restrict__ out, int batch, q::QuantDst dst, int quant) {
  using namespace sm100;
  __shared__ cl::Exchange xch;
  cl::cluster_start(&xch, 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int group = P.group;
  const int kvh = blockIdx.x, b = blockIdx.y;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring_base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = ring_base + warp * RING * 2 * TILE_BYTES;
  uint64_t* bar = reinterpret_cast<uint64_t*>(ring_base + SPLIT_WARPS * RING * 2 * TILE_BYTES) + warp * RING;
  int* abort_flag = reinterpret_cast<int*>(reinterpret_cast<uint64_t*>(ring_base + SPLIT_WARPS * RING * 2 * TILE_BYTES) +
                                           SPLIT_WARPS * RING);
  __shared__ __align__(16) __half p_s[SPLIT_WARPS][8][16];
  __shared__ float sm_m[SPLIT_WARPS][8], sm_l[SPLIT_WARPS][8];
  __shared__ float red[cl::MAX_WARPS];

  if (threadIdx.x == 0) *abort_flag = 0;
  if (lane < RING) mbar_init(&bar[lane], 1);
  fence_mbar_init();
  __syncthreads();
  if (!P.early) {
    pdl_wait();
    pdl_trigger();
  }

  const int o_begin = kvh * group * (D / 8), o_count = group * (D / 8);  // this CTA's octets of the row
  if (b >= batch) {  // padding row of the last token tile: zero operand, unit scale
    if (P.early) {
      pdl_wait();
      pdl_trigger();
    }
    if (quant) {
      for (int o = threadIdx.x; o < o_count; o += blockDim.x) q::zero_oct(dst, b, o_begin + o);
      if (kvh == 0 && threadIdx.x == 0) dst.gx[b] = 1.f;
    }
    cl::cluster_wait();
    return;
  }
  const int ctx = clamp_ctx(P, __ldg(P.ctx + b));
  int start, start16, nsplit;
  seq_range(P, ctx, CT_MAX, start, start16, nsplit);  // the tile range only
  const int t0 = start16, t1 = ctx;
  const int ntiles = ctx > t0 ? (t1 - t0 + 15) >> 4 : 0;
  const int nk = ntiles > warp ? (ntiles - warp + SPLIT_WARPS - 1) / SPLIT_WARPS : 0;  // this warp's tiles
  // lane j: page of this warp's j-th tile (tile warp + 4j)
  int my_block = -1, my_row0 = 0;
  if (lane < nk) {
    const int tt = t0 + TILE * (warp + SPLIT_WARPS * lane);
    const int page_idx = tt / P.page;
    my_row0 = tt - page_idx * P.page;
    my_block = __ldg(P.bt + (int64_t)b * P.bt_stride + page_idx);
    if (my_block >= P.num_pages) my_block = -1;
  }
  auto issue = [&](int k) {
    const int blk = __shfl_sync(0xffffffffu, my_block, k);
    const int row0 = __shfl_sync(0xffffffffu, my_row0, k);
    if (lane == 0) {
      const int slot = k % RING;
      uint64_t* bb = &bar[slot];
      if (blk >= 0) {
        mbar_arrive_expect_tx(bb, 2 * TILE_BYTES);
        tma_load_4d(ring + slot * 2 * TILE_BYTES, &tmk, bb, 0, kvh, row0, blk);
        tma_load_4d(ring + slot * 2 * TILE_BYTES + TILE_BYTES, &tmv, bb, 0, kvh, row0, blk);
      } else {
        mbar_arrive_plain(bb);
      }
    }
  };
  // early mode: the tile holding position ctx - 1 (this warp's tile `held`) waits for the
  // programmatic-launch dependency; the others are requested before it.
  const int held = (P.early && ntiles > 0 && (ntiles - 1) % SPLIT_WARPS == warp) ? (ntiles - 1) / SPLIT_WARPS : -1;
  for (int k = 0; k < RING && k < nk; ++k)
    if (k != held) issue(k);
  if (P.early) {
    pdl_wait();
    pdl_trigger();
    if (held >= 0 && held < RING) issue(held);
  }
  uint32_t qf[16];
  load_q_frag<TQ>(P, b, kvh, g, c, qf);
  WarpState ws;
  ws.init();
  bool failed = false;
  for (int k = 0; k < nk; ++k) {
    const int slot = k % RING;
    if (!mbar_wait_bounded(&bar[slot], (k / RING) & 1, abort_flag, nullptr, 0u)) {
      failed = true;
      break;
    }
    const bool blk_ok = __shfl_sync(0xffffffffu, my_block, k) >= 0;
    attn_tile(P, ring + slot * 2 * TILE_BYTES, blk_ok, t0 + TILE * (warp + SPLIT_WARPS * k), ctx, start, t1, qf, ws,
              p_s[warp], g, c);
    __syncwarp();
    if (k + RING < nk) {
      if (lane == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(k + RING);
    }
  }
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    ws.l0 += __shfl_xor_sync(0xffffffffu, ws.l0, o);
    ws.l1 += __shfl_xor_sync(0xffffffffu, ws.l1, o);
  }
  if (failed) *abort_flag = 1;
  __syncthreads();  // every warp is done with its ring: the ring memory is reused below
  float(*sm_o)[8][D] = reinterpret_cast<float(*)[8][D]>(ring_base);  // [warp][head][d]
  float* vals = reinterpret_cast<float*>(ring_base + SPLIT_WARPS * 8 * D * sizeof(float));  // [head][d]
  if (g == 0) {
    sm_m[warp][2 * c] = ws.m0;
    sm_m[warp][2 * c + 1] = ws.m1;
    sm_l[warp][2 * c] = ws.l0;
    sm_l[warp][2 * c + 1] = ws.l1;
  }
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const int d = 16 * g + 2 * mt;
    sm_o[warp][2 * c][d] = ws.acc[mt][0];
    sm_o[warp][2 * c + 1][d] = ws.acc[mt][1];
    sm_o[warp][2 * c][d + 1] = ws.acc[mt][2];
    sm_o[warp][2 * c + 1][d + 1] = ws.acc[mt][3];
  }
  __syncthreads();
  const bool bad = *abort_flag != 0;  // a tile never arrived: poison the token's output
  const int d = threadIdx.x;          // 128 threads == D
  float amax = 0.f;
  for (int h = 0; h < group; ++h) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < SPLIT_WARPS; ++w) M = fmaxf(M, sm_m[w][h]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < SPLIT_WARPS; ++w) {
        const float sw = fast_exp2(sm_m[w][h] - M);
        L += sm_l[w][h] * sw;
        O += sm_o[w][h][d] * sw;
      }
    }
    float v = L > 0.f ? (O * P.v_scale) / L : 0.f;
    if (bad) v = __int_as_float(0x7fc00000);
    v = to_f32(from_f32<TO>(v));
    if (out) out[((int64_t)b * P.num_heads + kvh * group + h) * D + d] = from_f32<TO>(v);
    vals[h * D + d] = v;
    amax = fmaxf(amax, fabsf(v));
  }
  cl::cluster_wait();  // all CTAs of the cluster run: their shared memory may be written
  if (!quant) return;
  const q::RowQ rq = q::make_rowq(cl::cluster_allreduce_x<cl::OpMax>(amax, red, &xch), dst.terms);
  if (kvh == 0 && threadIdx.x == 0) dst.gx[b] = rq.g[0];
  for (int o0 = 0; o0 < o_count; o0 += blockDim.x) {  // every lane calls quant_oct (terms == 1 pairs lanes)
    const int o = o0 + (int)threadIdx.x;
    float r[8];
    if (o < o_count) {
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] = vals[o * 8 + i];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] = 0.f;
    }
    q::quant_oct(dst, b, o_begin + (o < o_count ? o : 0), r, rq, o < o_count);
  }
}

template <typename TQ, typename TO>
inline bool fused_smem_ready() {
  static std::atomic<bool> done[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (done[dev]) return true;
  if (cudaFuncSetAttribute(decode_fused_kernel<TQ, TO>, cudaFuncAttributeMaxDynamicSharedMemorySize, FUSED_SMEM) !=
          cudaSuccess ||
      cudaFuncSetAttribute(decode_fused_kernel<TQ, TO>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    return false;
  done[dev] = true;
  return true;
}

// ---- split merge ------------------------------------------------------------------
// The (max, sum) statistics of the splits of heads [h0, h0 + nh) of sequence b are staged in
// shared memory: sw[hl * nsplit + s] = 2^(m_s - M) (the weight of split s), sl[hl] = the
// merged sum L.  One warp per head: lane-strided max and sum plus a fixed xor-shuffle tree,
// so every kernel that merges a head rounds identically.  All threads of the CTA call it.
__device__ __forceinline__ void merge_weights(const Params& P, int b, int h0, int nh, int nsplit, float* sw,
                                              float* sl) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int hl = warp; hl < nh; hl += nw) {
    const float* ml = P.ml_part + ((int64_t)b * P.num_heads + h0 + hl) * P.max_splits * 2;
    float M = -INFINITY;
    for (int s = lane; s < nsplit; s += 32) M = fmaxf(M, ml[2 * s]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    for (int s = lane; s < nsplit; s += 32) {
      const float w = M != -INFINITY ? fast_exp2(ml[2 * s] - M) : 0.f;
      sw[hl * nsplit + s] = w;
      L += ml[2 * s + 1] * w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) sl[hl] = L;
  }
  __syncthreads();
}

// Split-merge order shared by every merge kernel: A_j = sum over splits s = j, j+4, j+8, ...
// (ascending) of fmaf(o_part[s][d], w_s, .), O = ((A_0 + A_1) + A_2) + A_3, then O / L.
template <int N>
__device__ __forceinline__ void merge_partial(const Params& P, int b, int h, int d0, int nsplit, const float* w, int j,
                                              float* A) {
  const float* op = P.o_part + ((int64_t)b * P.num_heads + h) * P.max_splits * D + d0;
#pragma unroll
  for (int i = 0; i < N; ++i) A[i] = 0.f;
#pragma unroll 2
  for (int s = j; s < nsplit; s += 4) {
    const float ws = w[s];
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 f = *reinterpret_cast<const float4*>(op + (int64_t)s * D + i);
      A[i + 0] = fmaf(f.x, ws, A[i + 0]);
      A[i + 1] = fmaf(f.y, ws, A[i + 1]);
      A[i + 2] = fmaf(f.z, ws, A[i + 2]);
      A[i + 3] = fmaf(f.w, ws, A[i + 3]);
    }
  }
}
__device__ __forceinline__ float merge_finish(float a0, float a1, float a2, float a3, float L) {
  const float O = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
  return L > 0.f ? __fdiv_rn(O, L) : 0.f;
}

// All four interleaved partials in one thread (the fused merge+quant kernel).
template <int N>
__device__ __forceinline__ void merge_out(const Params& P, int b, int h, int d0, int nsplit, const float* w, float L,
                                          float* out) {
  float A[4][N];
#pragma unroll
  for (int j = 0; j < 4; ++j) merge_partial<N>(P, b, h, d0, nsplit, w, j, A[j]);
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = merge_finish(A[0][i], A[1][i], A[2][i], A[3][i], L);
}

// One CTA per (head, sequence): warp j accumulates the splits s = j (mod 4) for all 128 dims
// (4 per lane); thread t combines dim t.  Dynamic shared memory: nsplit floats.
template <typename TO>
__global__ void __launch_bounds__(128) decode_reduce_kernel(Params P, TO* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float merge_smem[];
  __shared__ float sl[1];
  __shared__ __align__(16) float part[4][D];
  const int h = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ctx = clamp_ctx(P, __ldg(P.ctx + b));
  int start, start16, nsplit;
  seq_range(P, ctx, *P.split_tiles, start, start16, nsplit);  // the split kernel's split length
  merge_weights(P, b, h, 1, nsplit, merge_smem, sl);
  float A[4];
  merge_partial<4>(P, b, h, 4 * lane, nsplit, merge_smem, warp, A);
  *reinterpret_cast<float4*>(&part[warp][4 * lane]) = make_float4(A[0], A[1], A[2], A[3]);
  __syncthreads();
  const int d = threadIdx.x;
  out[((int64_t)b * P.num_heads + h) * D + d] =
      from_f32<TO>(merge_finish(part[0][d], part[1][d], part[2][d], part[3][d], sl[0]));
}

// Split-K merge fused with the NVFP4 activation quantiser (quant.cuh): the token's
// [num_heads * 128] attention row is spread over a cluster of CTAs (grid (ctas, m_pad),
// cluster.cuh), each merging a contiguous slice of 16-element units; the merged row
// (rounded to the output dtype, as the unfused kernel writes it) is quantised as the
// operand of o_proj once the cluster has combined the row amax.  `out` may be null.
template <typename TO, int MAXU>
__global__ void __launch_bounds__(512) decode_reduce_quant_kernel(Params P, TO* __restrict__ out, int batch,
                                                                  q::QuantDst dst) {
  __shared__ float red[cl::MAX_WARPS];
  __shared__ cl::Exchange xch;
  cl::cluster_start(&xch, 1);
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.y;
  const int row_len = P.num_heads * D;
  const int o0 = cl::slice_octet(row_len >> 4, blockIdx.x, gridDim.x);
  const int o1 = cl::slice_octet(row_len >> 4, blockIdx.x + 1, gridDim.x);
  if (b >= batch) {
    for (int o = o0 + threadIdx.x; o < o1; o += blockDim.x) q::zero_oct(dst, b, o);
    if (blockIdx.x == 0 && threadIdx.x == 0) dst.gx[b] = 1.f;
    cl::cluster_wait();
    return;
  }
  const int ctx = clamp_ctx(P, __ldg(P.ctx + b));
  int start, start16, nsplit;
  seq_range(P, ctx, *P.split_tiles, start, start16, nsplit);
  extern __shared__ float merge_smem[];  // [heads of this slice][nsplit] weights, then [heads] sums
  const int h0 = (o0 * 8) / D, nh = ((o1 * 8 - 1) / D) - h0 + 1;
  float* sl = merge_smem + nh * nsplit;
  merge_weights(P, b, h0, nh, nsplit, merge_smem, sl);
  float v[MAXU][8];
  float amax = 0.f;
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int o = o0 + threadIdx.x + u * blockDim.x;
#pragma unroll
    for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
    if (o >= o1) continue;
    const int h = (o * 8) / D, d0 = (o * 8) % D;
    float r[8];
    merge_out<8>(P, b, h, d0, nsplit, merge_smem + (h - h0) * nsplit, sl[h - h0], r);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[u][i] = to_f32(from_f32<TO>(r[i]));
      amax = fmaxf(amax, fabsf(v[u][i]));
    }
    if (out) *reinterpret_cast<uint4*>(out + (int64_t)b * row_len + o * 8) = pack8<TO>(v[u]);
  }
  cl::cluster_wait();
  const q::RowQ rq = q::make_rowq(cl::cluster_allreduce_x<cl::OpMax>(amax, red, &xch), dst.terms);
  if (blockIdx.x == 0 && threadIdx.x == 0) dst.gx[b] = rq.g[0];
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int o = o0 + threadIdx.x + u * blockDim.x;
    q::quant_oct(dst, b, o < o1 ? o : 0, v[u], rq, o < o1);
  }
}

// Dynamic shared memory above 48 KB and the maximum shared carveout (three CTAs per SM),
// set once per device.
template <typename TQ>
inline bool split_smem_ready() {
  static std::atomic<bool> done[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (done[dev]) return true;
  if (cudaFuncSetAttribute(decode_split_kernel<TQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, SPLIT_SMEM_V3) !=
          cudaSuccess ||
      cudaFuncSetAttribute(decode_split_kernel<TQ>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    return false;
  done[dev] = true;
  return true;
}

inline int max_splits_for(int32_t max_pages, int32_t page) {
  const int64_t toks = (int64_t)max_pages * page;
  return (int)cdiv(toks + 15, CT_MIN * TILE);  // +15: the tile-aligned window start can add one tile
}
constexpr size_t SPLIT_WORD_BYTES = 256;  // the chosen split length, after the partials

}  // namespace attn
}  // namespace ada

using namespace ada;

extern "C" size_t ada_fp8_paged_decode_workspace_size(int32_t batch, int32_t num_heads, int32_t max_pages,
                                                      int32_t page_size, int32_t head_dim) {
  if (batch <= 0 || num_heads <= 0 || max_pages <= 0 || page_size <= 0 || head_dim <= 0) return 0;
  const int64_t S = attn::max_splits_for(max_pages, page_size);
  return (size_t)batch * num_heads * S * (head_dim + 2) * sizeof(float) + attn::SPLIT_WORD_BYTES;
}

static int paged_decode_impl(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                             const uint8_t* k_cache, const uint8_t* v_cache, int64_t kv_stride_page,
                             int64_t kv_stride_tok, int64_t kv_stride_head, int64_t num_pages,
                             const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                             const int32_t* context_lens, int32_t batch, int32_t num_heads, int32_t num_kv_heads,
                             int32_t head_dim, int32_t page_size, float scale, float k_scale, float v_scale,
                             int32_t window, void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                             void* stream, const q::QuantDst* qd, int32_t flags);

extern "C" int ada_fp8_paged_decode(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                                    const uint8_t* k_cache, const uint8_t* v_cache, int64_t kv_stride_page,
                                    int64_t kv_stride_tok, int64_t kv_stride_head, int64_t num_pages,
                                    const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                                    const int32_t* context_lens, int32_t batch, int32_t num_heads,
                                    int32_t num_kv_heads, int32_t head_dim, int32_t page_size, float scale,
                                    float k_scale, float v_scale, int32_t window, void* out, int out_dtype,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  if (!out) return ADA_ERR_INVALID_ARG;
  return paged_decode_impl(q, q_dtype, q_stride_b, q_stride_h, k_cache, v_cache, kv_stride_page, kv_stride_tok,
                           kv_stride_head, num_pages, block_tables, bt_stride, max_pages, context_lens, batch,
                           num_heads, num_kv_heads, head_dim, page_size, scale, k_scale, v_scale, window, out,
                           out_dtype, workspace, workspace_bytes, stream, nullptr, 0);
}

extern "C" int ada_fp8_paged_decode_quant_ex(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                                             const uint8_t* k_cache, const uint8_t* v_cache, int64_t kv_stride_page,
                                             int64_t kv_stride_tok, int64_t kv_stride_head, int64_t num_pages,
                                             const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                                             const int32_t* context_lens, int32_t batch, int32_t num_heads,
                                             int32_t num_kv_heads, int32_t head_dim, int32_t page_size, float scale,
                                             float k_scale, float v_scale, int32_t window, void* out, int out_dtype,
                                             int terms, int block_n, uint8_t* xq, uint8_t* sfx, float* gx,
                                             void* workspace, size_t workspace_bytes, int32_t flags, void* stream) {
  if (flags & ~ADA_ATTN_META_EARLY) return ADA_ERR_INVALID_ARG;
  const int row = num_heads * head_dim;
  if (row % 256) return ADA_ERR_UNSUPPORTED;
  if (!q::dst_ok(terms, block_n, row) || !xq || !gx || (terms == 1 && !sfx)) return ADA_ERR_INVALID_ARG;
  if (((uintptr_t)xq & 15) || ((uintptr_t)gx & 3)) return ADA_ERR_ALIGNMENT;
  const q::QuantDst qd{xq, sfx, gx, terms, block_n, row};
  return paged_decode_impl(q, q_dtype, q_stride_b, q_stride_h, k_cache, v_cache, kv_stride_page, kv_stride_tok,
                           kv_stride_head, num_pages, block_tables, bt_stride, max_pages, context_lens, batch,
                           num_heads, num_kv_heads, head_dim, page_size, scale, k_scale, v_scale, window, out,
                           out_dtype, workspace, workspace_bytes, stream, &qd, flags);
}

extern "C" int ada_fp8_paged_decode_quant(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                                          const uint8_t* k_cache, const uint8_t* v_cache, int64_t kv_stride_page,
                                          int64_t kv_stride_tok, int64_t kv_stride_head, int64_t num_pages,
                                          const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                                          const int32_t* context_lens, int32_t batch, int32_t num_heads,
                                          int32_t num_kv_heads, int32_t head_dim, int32_t page_size, float scale,
                                          float k_scale, float v_scale, int32_t window, void* out, int out_dtype,
                                          int terms, int block_n, uint8_t* xq, uint8_t* sfx, float* gx,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  return ada_fp8_paged_decode_quant_ex(q, q_dtype, q_stride_b, q_stride_h, k_cache, v_cache, kv_stride_page,
                                       kv_stride_tok, kv_stride_head, num_pages, block_tables, bt_stride, max_pages,
                                       context_lens, batch, num_heads, num_kv_heads, head_dim, page_size, scale,
                                       k_scale, v_scale, window, out, out_dtype, terms, block_n, xq, sfx, gx,
                                       workspace, workspace_bytes, 0, stream);
}

static int paged_decode_impl(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                             const uint8_t* k_cache, const uint8_t* v_cache, int64_t kv_stride_page,
                             int64_t kv_stride_tok, int64_t kv_stride_head, int64_t num_pages,
                             const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                             const int32_t* context_lens, int32_t batch, int32_t num_heads, int32_t num_kv_heads,
                             int32_t head_dim, int32_t page_size, float scale, float k_scale, float v_scale,
                             int32_t window, void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                             void* stream, const q::QuantDst* qd, int32_t flags) {
  if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_pages <= 0 || page_size <= 0) return ADA_ERR_INVALID_ARG;
  if (batch == 0) return ADA_OK;
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !workspace) return ADA_ERR_INVALID_ARG;
  if ((q_dtype != ADA_DT_BF16 && q_dtype != ADA_DT_F16) || (out_dtype != ADA_DT_BF16 && out_dtype != ADA_DT_F16))
    return ADA_ERR_INVALID_ARG;
  if (head_dim != attn::D) return ADA_ERR_UNSUPPORTED;
  if (num_heads % num_kv_heads != 0) return ADA_ERR_INVALID_ARG;
  const int group = num_heads / num_kv_heads;
  if (group > 8) return ADA_ERR_UNSUPPORTED;
  if (page_size % 16 != 0) return ADA_ERR_UNSUPPORTED;
  if (window < 0 || bt_stride < max_pages || num_pages <= 0) return ADA_ERR_INVALID_ARG;
  // 16-byte gathers: every cache row start and the q rows must be 16-byte aligned
  if (((uintptr_t)k_cache | (uintptr_t)v_cache) & 15) return ADA_ERR_ALIGNMENT;
  if ((kv_stride_page | kv_stride_tok | kv_stride_head) & 15) return ADA_ERR_ALIGNMENT;
  if (((uintptr_t)q & 15) || (q_stride_b & 7) || (q_stride_h & 7)) return ADA_ERR_ALIGNMENT;
  const size_t need = ada_fp8_paged_decode_workspace_size(batch, num_heads, max_pages, page_size, head_dim);
  if (workspace_bytes < need) return ADA_ERR_WORKSPACE;

  attn::Params P;
  P.q = q;
  P.q_sb = q_stride_b;
  P.q_sh = q_stride_h;
  P.k = k_cache;
  P.v = v_cache;
  P.s_page = kv_stride_page;
  P.s_tok = kv_stride_tok;
  P.s_head = kv_stride_head;
  P.num_pages = num_pages;
  P.bt = block_tables;
  P.bt_stride = bt_stride;
  P.ctx = context_lens;
  P.num_heads = num_heads;
  P.group = group;
  P.page = page_size;
  P.window = window;
  P.max_splits = attn::max_splits_for(max_pages, page_size);
  P.max_pages = max_pages;
  P.scale_log2 = scale * k_scale * attn::LOG2E;
  P.v_scale = v_scale;
  P.o_part = reinterpret_cast<float*>(workspace);
  P.ml_part = P.o_part + (size_t)batch * num_heads * P.max_splits * attn::D;
  P.split_tiles = reinterpret_cast<int*>(P.ml_part + (size_t)batch * num_heads * P.max_splits * 2);
  P.early = (flags & ADA_ATTN_META_EARLY) ? 1 : 0;

  // K / V caches as 4-D byte tensors [num_pages][page][Hkv][D] -> TMA box of 16 rows x 128 B
  CUtensorMap tmk, tmv;
  const cuuint64_t dims[4] = {(cuuint64_t)head_dim, (cuuint64_t)num_kv_heads, (cuuint64_t)page_size,
                              (cuuint64_t)num_pages};
  const cuuint64_t strides[3] = {(cuuint64_t)kv_stride_head, (cuuint64_t)kv_stride_tok, (cuuint64_t)kv_stride_page};
  const cuuint32_t box[4] = {(cuuint32_t)head_dim, 1, (cuuint32_t)attn::TILE, 1};
  if (!sm100::encode_bytes(&tmk, k_cache, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !sm100::encode_bytes(&tmv, v_cache, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
    return ADA_ERR_CUDA;

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if ((int64_t)max_pages * page_size <= attn::FUSED_MAX_TOKENS && num_kv_heads <= cl::MAX_CLUSTER) {
    // short cache: split, merge and (optionally) quantisation in one cluster per token
    const int rows = qd ? (int)cdiv(batch, qd->bn) * qd->bn : batch;
    if (rows > 65535) return ADA_ERR_UNSUPPORTED;
    const q::QuantDst none{nullptr, nullptr, nullptr, 1, 16, num_heads * head_dim};
    const q::QuantDst& dq = qd ? *qd : none;
    const dim3 fg((unsigned)num_kv_heads, (unsigned)rows);
#define ADA_FUSED(TQ, TO)                                                                                       \
    do {                                                                                                        \
      if (!attn::fused_smem_ready<TQ, TO>()) return ADA_ERR_CUDA;                                               \
      (void)ada::launch_kc(attn::decode_fused_kernel<TQ, TO>, fg, dim3(attn::SPLIT_WARPS * 32), attn::FUSED_SMEM, \
                           st, num_kv_heads, tmk, tmv, P, reinterpret_cast<TO*>(out), (int)batch, dq, qd ? 1 : 0); \
    } while (0)
    if (q_dtype == ADA_DT_BF16) {
      if (out_dtype == ADA_DT_BF16) ADA_FUSED(__nv_bfloat16, __nv_bfloat16); else ADA_FUSED(__nv_bfloat16, __half);
    } else {
      if (out_dtype == ADA_DT_BF16) ADA_FUSED(__half, __nv_bfloat16); else ADA_FUSED(__half, __half);
    }
#undef ADA_FUSED
    ADA_CHECK_LAUNCH();
    return ADA_OK;
  }
  // persistent-style grid: every warp takes work items (sequence, KV head, split) round-robin
  static std::atomic<int> sms[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ADA_ERR_CUDA;
  int n_sm = sms[dev].load(std::memory_order_relaxed);
  if (!n_sm) {
    if (cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n_sm <= 0)
      return ADA_ERR_CUDA;
    sms[dev].store(n_sm, std::memory_order_relaxed);
  }
  const int64_t items = (int64_t)batch * num_kv_heads * P.max_splits;
  if (items > 0x7fffffff) return ADA_ERR_UNSUPPORTED;
  const int64_t want = (items + attn::SPLIT_WARPS - 1) / attn::SPLIT_WARPS;
  const unsigned grid = (unsigned)(want < 3 * (int64_t)n_sm ? want : 3 * (int64_t)n_sm);
  if (q_dtype == ADA_DT_BF16) {
    if (!attn::split_smem_ready<__nv_bfloat16>()) return ADA_ERR_CUDA;
    (void)ada::launch_k(attn::decode_split_kernel<__nv_bfloat16>, dim3(grid), dim3(attn::SPLIT_WARPS * 32),
                        attn::SPLIT_SMEM_V3, st, tmk, tmv, P, (int)num_kv_heads, (int)batch);
  } else {
    if (!attn::split_smem_ready<__half>()) return ADA_ERR_CUDA;
    (void)ada::launch_k(attn::decode_split_kernel<__half>, dim3(grid), dim3(attn::SPLIT_WARPS * 32),
                        attn::SPLIT_SMEM_V3, st, tmk, tmv, P, (int)num_kv_heads, (int)batch);
  }
  ADA_CHECK_LAUNCH();
  if (qd) {
    const int m_pad = (int)cdiv(batch, qd->bn) * qd->bn;
    const cl::RowSplit sp = cl::row_split(num_heads * head_dim / 16);
    if (!sp.maxu || sp.maxu > 4 || m_pad > 65535) return ADA_ERR_UNSUPPORTED;
    const dim3 rg((unsigned)sp.ctas, (unsigned)m_pad), rb((unsigned)sp.threads);
    // staged merge weights: the heads one CTA's slice touches x the splits, plus their sums
    const int units = num_heads * head_dim / 16;
    const int nh_max = (2 * ((units + sp.ctas - 1) / sp.ctas) * 8 + attn::D - 1) / attn::D + 1;
    const size_t msmem = (size_t)nh_max * (P.max_splits + 1) * sizeof(float);
    if (msmem > 48 * 1024) return ADA_ERR_UNSUPPORTED;
#define ADA_RQ(TO, MU)                                                                                         \
    (void)ada::launch_kc(attn::decode_reduce_quant_kernel<TO, MU>, rg, rb, msmem, st, sp.ctas, P,              \
                         reinterpret_cast<TO*>(out), batch, *qd)
    if (out_dtype == ADA_DT_BF16) {
      if (sp.maxu == 1) ADA_RQ(__nv_bfloat16, 1); else if (sp.maxu == 2) ADA_RQ(__nv_bfloat16, 2); else ADA_RQ(__nv_bfloat16, 4);
    } else {
      if (sp.maxu == 1) ADA_RQ(__half, 1); else if (sp.maxu == 2) ADA_RQ(__half, 2); else ADA_RQ(__half, 4);
    }
#undef ADA_RQ
    ADA_CHECK_LAUNCH();
    return ADA_OK;
  }
  dim3 rgrid(num_heads, batch);
  const size_t rsmem = (size_t)P.max_splits * sizeof(float);
  if (rsmem > 48 * 1024) return ADA_ERR_UNSUPPORTED;
  if (out_dtype == ADA_DT_BF16)
    (void)ada::launch_k(attn::decode_reduce_kernel<__nv_bfloat16>, rgrid, dim3(128), rsmem, st, P,
                        reinterpret_cast<__nv_bfloat16*>(out));
  else
    (void)ada::launch_k(attn::decode_reduce_kernel<__half>, rgrid, dim3(128), rsmem, st, P,
                        reinterpret_cast<__half*>(out));
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}