// FP8 paged split-K decode attention for B200 (sm_100a).
//
// Replaces fp8_kv_decode_group_kernel (reference adallm/ops/attention.py:126-233).
// Same math: per (sequence, kv head) the Hq/Hkv query heads of the GQA group
// attend to tokens [start, ctx) of the paged e4m3 cache, with q rounded to
// fp16, K/V widened to fp16, fp32 scores and softmax statistics, fp16
// probabilities for P.V and fp32 accumulation.  Differences by design:
//   * split-K over the context (flash-decoding): each CTA owns one CHUNK of
//     tokens of one (sequence, kv head) and writes an unnormalised partial
//     (max, sum, O) to the workspace; a reduction kernel merges the splits;
//   * the page walk is exact for any page size that is a multiple of 16
//     (the reference reads past a page for pages < 64);
//   * optional per-tensor k_scale / v_scale (1.0 reproduces the reference).
//
// Tile = 16 tokens of one page.  One warp computes S^T = K_tile . Q^T with
// mma.m16n8k16 (tokens on M, heads on N), an online softmax per head, and
// O^T += V_tile^T . P^T.  Every thread gathers its K and V bytes straight
// from HBM with 16-byte loads: for the K operand the head dimension is
// permuted so that thread (g, c) needs bytes [32c, 32c+32) of tokens g and
// g+8 (the permutation is applied to Q identically); for the V operand the
// output dimension is permuted so thread (g, c) needs bytes [16g, 16g+16) of
// tokens 2c, 2c+1, 2c+8, 2c+9.  A warp therefore reads whole 128-byte rows.
#include "cluster.cuh"
#include "quant.cuh"

namespace ada {
namespace attn {

constexpr int D = 128;
constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int CHUNK = 256;  // tokens per split (CTA)
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
};

// Tokens beyond the block table's reach (ctx > max_pages * page) cannot be addressed and are
// dropped, so every index below stays inside the table and the workspace.
__device__ __forceinline__ int clamp_ctx(const Params& P, int ctx) {
  return min(ctx, P.max_pages * P.page);
}

__device__ __forceinline__ void seq_range(const Params& P, int ctx, int& start, int& start16, int& nsplit) {
  start = P.window > 0 ? max(ctx - P.window, 0) : 0;
  start16 = start & ~15;
  nsplit = ctx > 0 ? min((ctx - start16 + CHUNK - 1) / CHUNK, P.max_splits) : 0;
}

struct TileRegs {
  uint4 k0[2];  // token g,   bytes [32c, 32c+32)
  uint4 k8[2];  // token g+8
  uint4 v[4];   // tokens 2c, 2c+1, 2c+8, 2c+9, bytes [16g, 16g+16)
  int block;
};

__device__ __forceinline__ void load_tile(const Params& P, int b, int kvh, int tile_t0, int ctx, int g, int c,
                                          TileRegs& r) {
  const int page_idx = tile_t0 / P.page;
  const int row0 = tile_t0 - page_idx * P.page;
  r.block = __ldg(P.bt + (int64_t)b * P.bt_stride + page_idx);
  if (r.block >= P.num_pages) r.block = -1;
  const uint4 z = make_uint4(0, 0, 0, 0);
  if (r.block < 0) {
    r.k0[0] = r.k0[1] = r.k8[0] = r.k8[1] = z;
    r.v[0] = r.v[1] = r.v[2] = r.v[3] = z;
    return;
  }
  const int64_t base = (int64_t)r.block * P.s_page + (int64_t)row0 * P.s_tok + (int64_t)kvh * P.s_head;
  const uint8_t* kp = P.k + base + 32 * c;
  r.k0[0] = ldg_stream16(kp + (int64_t)g * P.s_tok);
  r.k0[1] = ldg_stream16(kp + (int64_t)g * P.s_tok + 16);
  r.k8[0] = ldg_stream16(kp + (int64_t)(g + 8) * P.s_tok);
  r.k8[1] = ldg_stream16(kp + (int64_t)(g + 8) * P.s_tok + 16);
  const uint8_t* vp = P.v + base + 16 * g;
  const int toks[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // Rows at or past ctx may hold uninitialised bytes (NaN in e4m3); they get
    // probability 0, so their V must be finite: zero them.
    r.v[i] = (tile_t0 + toks[i] < ctx) ? ldg_stream16(vp + (int64_t)toks[i] * P.s_tok) : z;
  }
}

template <typename TQ>
__global__ void __launch_bounds__(THREADS, 3) decode_split_kernel(Params P) {
  pdl_wait();
  pdl_trigger();

  const int s = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int ctx = clamp_ctx(P, __ldg(P.ctx + b));
  int start, start16, nsplit;
  seq_range(P, ctx, start, start16, nsplit);
  if (s >= nsplit) return;
  const int t0 = start16 + s * CHUNK;
  const int t1 = min(ctx, t0 + CHUNK);
  const int ntiles = (t1 - t0 + 15) >> 4;
  const int lo = max(start, t0);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int group = P.group;

  __shared__ __align__(16) __half p_s[WARPS][8][16];
  __shared__ float sm_m[WARPS][8], sm_l[WARPS][8];
  __shared__ __align__(16) float sm_o[WARPS][8][D];

  // Q operand (B of the score MMA): head g of the group, d in [32c, 32c+32),
  // fp16 as the reference (attention.py:314-324).  qf[2s], qf[2s+1] = k-step s.
  uint32_t qf[16];
  if (g < group) {
    const TQ* qp = reinterpret_cast<const TQ*>(P.q) + (int64_t)b * P.q_sb + (int64_t)(kvh * group + g) * P.q_sh + 32 * c;
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

  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  TileRegs cur, nxt;
  int tile = warp;
  if (tile < ntiles) load_tile(P, b, kvh, t0 + 16 * tile, ctx, g, c, cur);
  for (; tile < ntiles; tile += WARPS) {
    const int tt = t0 + 16 * tile;
    const bool has_next = tile + WARPS < ntiles;
    if (has_next) load_tile(P, b, kvh, tt + 16 * WARPS, ctx, g, c, nxt);

    // ---- scores S^T[token][head] -------------------------------------------
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t* kg = reinterpret_cast<const uint32_t*>(cur.k0);
    const uint32_t* kg8 = reinterpret_cast<const uint32_t*>(cur.k8);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t a[4];
      a[0] = e4m3x2_to_f16x2((uint16_t)(kg[ks] & 0xFFFFu));
      a[1] = e4m3x2_to_f16x2((uint16_t)(kg8[ks] & 0xFFFFu));
      a[2] = e4m3x2_to_f16x2((uint16_t)(kg[ks] >> 16));
      a[3] = e4m3x2_to_f16x2((uint16_t)(kg8[ks] >> 16));
      mma_16816_f16(sc, a, &qf[2 * ks]);
    }
    const bool blk_ok = cur.block >= 0;
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
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    float al0 = 1.f, al1 = 1.f, p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
    if (mn0 != -INFINITY) {
      al0 = fast_exp2(m0 - mn0);
      p0 = fast_exp2(x0 - mn0);
      p2 = fast_exp2(x2 - mn0);
    }
    if (mn1 != -INFINITY) {
      al1 = fast_exp2(m1 - mn1);
      p1 = fast_exp2(x1 - mn1);
      p3 = fast_exp2(x3 - mn1);
    }
    m0 = mn0;
    m1 = mn1;
    // fp32 probabilities feed the row sum, fp16 ones feed P.V (attention.py:219-223)
    const __half hp0 = __float2half_rn(p0), hp1 = __float2half_rn(p1);
    const __half hp2 = __float2half_rn(p2), hp3 = __float2half_rn(p3);
    l0 = l0 * al0 + (p0 + p2);
    l1 = l1 * al1 + (p1 + p3);
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      acc[mt][0] *= al0;
      acc[mt][1] *= al1;
      acc[mt][2] *= al0;
      acc[mt][3] *= al1;
    }
    // ---- transpose P through shared memory: P^T operand wants (token pairs, head g)
    p_s[warp][2 * c][g] = hp0;
    p_s[warp][2 * c + 1][g] = hp1;
    p_s[warp][2 * c][g + 8] = hp2;
    p_s[warp][2 * c + 1][g + 8] = hp3;
    __syncwarp();
    uint32_t bp[2];
    bp[0] = *reinterpret_cast<const uint32_t*>(&p_s[warp][g][2 * c]);
    bp[1] = *reinterpret_cast<const uint32_t*>(&p_s[warp][g][2 * c + 8]);
    __syncwarp();

    // ---- O^T[d][head] += V^T . P^T ----------------------------------------
    const uint32_t* v0 = reinterpret_cast<const uint32_t*>(&cur.v[0]);
    const uint32_t* v1 = reinterpret_cast<const uint32_t*>(&cur.v[1]);
    const uint32_t* v8 = reinterpret_cast<const uint32_t*>(&cur.v[2]);
    const uint32_t* v9 = reinterpret_cast<const uint32_t*>(&cur.v[3]);
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
        mma_16816_f16(acc[2 * j + half], a, bp);
      }
    }
    if (has_next) cur = nxt;
  }

  // ---- merge the warps' partial states ------------------------------------
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  if (g == 0) {
    sm_m[warp][2 * c] = m0;
    sm_m[warp][2 * c + 1] = m1;
    sm_l[warp][2 * c] = l0;
    sm_l[warp][2 * c + 1] = l1;
  }
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const int d = 16 * g + 2 * mt;
    sm_o[warp][2 * c][d] = acc[mt][0];
    sm_o[warp][2 * c + 1][d] = acc[mt][1];
    sm_o[warp][2 * c][d + 1] = acc[mt][2];
    sm_o[warp][2 * c + 1][d + 1] = acc[mt][3];
  }
  __syncthreads();
  const int d = threadIdx.x;  // THREADS == D
  for (int h = 0; h < group; ++h) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, sm_m[w][h]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
        const float sw = fast_exp2(sm_m[w][h] - M);
        L += sm_l[w][h] * sw;
        O += sm_o[w][h][d] * sw;
      }
    }
    const int64_t row = ((int64_t)b * P.num_heads + kvh * group + h) * P.max_splits + s;
    P.o_part[row * D + d] = O * P.v_scale;
    if (d == 0) {
      P.ml_part[row * 2 + 0] = M;
      P.ml_part[row * 2 + 1] = L;
    }
  }
}

template <typename TO>
__global__ void __launch_bounds__(D) decode_reduce_kernel(Params P, TO* __restrict__ out) {
  pdl_wait();
  pdl_trigger();

  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int ctx = clamp_ctx(P, __ldg(P.ctx + b));
  int start, start16, nsplit;
  seq_range(P, ctx, start, start16, nsplit);
  const int64_t row0 = ((int64_t)b * P.num_heads + h) * P.max_splits;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, P.ml_part[(row0 + s) * 2]);
  float L = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < nsplit; ++s) {
      const float w = fast_exp2(P.ml_part[(row0 + s) * 2] - M);
      L += P.ml_part[(row0 + s) * 2 + 1] * w;
      O += P.o_part[(row0 + s) * D + d] * w;
    }
  }
  const float r = L > 0.f ? O / L : 0.f;
  out[((int64_t)b * P.num_heads + h) * D + d] = from_f32<TO>(r);
}


// Split-K merge fused with the NVFP4 activation quantiser (quant.cuh): the token's
// [num_heads * 128] attention row is spread over a cluster of CTAs (grid (ctas, m_pad),
// cluster.cuh), each merging a contiguous slice of 16-element units; the merged row
// (rounded to the output dtype, as the unfused kernel writes it) is quantised as the
// operand of o_proj once the cluster has combined the row amax.  `out` may be null.
template <typename TO, int MAXU>
__global__ void __launch_bounds__(512) decode_reduce_quant_kernel(Params P, TO* __restrict__ out, int batch,
                                                                  q::QuantDst dst) {
  cl::cluster_arrive_relaxed();
  pdl_wait();
  pdl_trigger();
  __shared__ float red[cl::MAX_WARPS];
  __shared__ float slots[cl::MAX_CLUSTER];
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
  seq_range(P, ctx, start, start16, nsplit);
  float v[MAXU][8];
  float amax = 0.f;
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int o = o0 + threadIdx.x + u * blockDim.x;
#pragma unroll
    for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
    if (o >= o1) continue;
    const int h = (o * 8) / D, d0 = (o * 8) % D;
    const int64_t row0 = ((int64_t)b * P.num_heads + h) * P.max_splits;
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, P.ml_part[(row0 + s) * 2]);
    float L = 0.f, O[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) O[i] = 0.f;
    if (M != -INFINITY) {
      for (int s = 0; s < nsplit; ++s) {
        const float w = fast_exp2(P.ml_part[(row0 + s) * 2] - M);
        L += P.ml_part[(row0 + s) * 2 + 1] * w;
        const float4* op = reinterpret_cast<const float4*>(P.o_part + (row0 + s) * D + d0);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float4 f = op[i];
          O[4 * i + 0] += f.x * w;
          O[4 * i + 1] += f.y * w;
          O[4 * i + 2] += f.z * w;
          O[4 * i + 3] += f.w * w;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[u][i] = to_f32(from_f32<TO>(L > 0.f ? O[i] / L : 0.f));
      amax = fmaxf(amax, fabsf(v[u][i]));
    }
    if (out) *reinterpret_cast<uint4*>(out + (int64_t)b * row_len + o * 8) = pack8<TO>(v[u]);
  }
  cl::cluster_wait();
  const q::RowQ rq = q::make_rowq(cl::cluster_allreduce<cl::OpMax>(amax, red, slots), dst.terms);
  if (blockIdx.x == 0 && threadIdx.x == 0) dst.gx[b] = rq.g[0];
#pragma unroll
  for (int u = 0; u < MAXU; ++u) {
    const int o = o0 + threadIdx.x + u * blockDim.x;
    q::quant_oct(dst, b, o < o1 ? o : 0, v[u], rq, o < o1);
  }
}

inline int max_splits_for(int32_t max_pages, int32_t page) {
  const int64_t toks = (int64_t)max_pages * page;
  return (int)cdiv(toks + 15, CHUNK);  // +15: the tile-aligned window start can add one tile
}

}  // namespace attn
}  // namespace ada

using namespace ada;

extern "C" size_t ada_fp8_paged_decode_workspace_size(int32_t batch, int32_t num_heads, int32_t max_pages,
                                                      int32_t page_size, int32_t head_dim) {
  if (batch <= 0 || num_heads <= 0 || max_pages <= 0 || page_size <= 0 || head_dim <= 0) return 0;
  const int64_t S = attn::max_splits_for(max_pages, page_size);
  return (size_t)batch * num_heads * S * (head_dim + 2) * sizeof(float);
}

static int paged_decode_impl(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                             const uint8_t* k_cache, const uint8_t* v_cache, int64_t kv_stride_page,
                             int64_t kv_stride_tok, int64_t kv_stride_head, int64_t num_pages,
                             const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                             const int32_t* context_lens, int32_t batch, int32_t num_heads, int32_t num_kv_heads,
                             int32_t head_dim, int32_t page_size, float scale, float k_scale, float v_scale,
                             int32_t window, void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                             void* stream, const q::QuantDst* qd);

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
                           out_dtype, workspace, workspace_bytes, stream, nullptr);
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
  const int row = num_heads * head_dim;
  if (row % 256) return ADA_ERR_UNSUPPORTED;
  if (!q::dst_ok(terms, block_n, row) || !xq || !gx || (terms == 1 && !sfx)) return ADA_ERR_INVALID_ARG;
  if (((uintptr_t)xq & 15) || ((uintptr_t)gx & 3)) return ADA_ERR_ALIGNMENT;
  const q::QuantDst qd{xq, sfx, gx, terms, block_n, row};
  return paged_decode_impl(q, q_dtype, q_stride_b, q_stride_h, k_cache, v_cache, kv_stride_page, kv_stride_tok,
                           kv_stride_head, num_pages, block_tables, bt_stride, max_pages, context_lens, batch,
                           num_heads, num_kv_heads, head_dim, page_size, scale, k_scale, v_scale, window, out,
                           out_dtype, workspace, workspace_bytes, stream, &qd);
}

static int paged_decode_impl(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                             const uint8_t* k_cache, const uint8_t* v_cache, int64_t kv_stride_page,
                             int64_t kv_stride_tok, int64_t kv_stride_head, int64_t num_pages,
                             const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                             const int32_t* context_lens, int32_t batch, int32_t num_heads, int32_t num_kv_heads,
                             int32_t head_dim, int32_t page_size, float scale, float k_scale, float v_scale,
                             int32_t window, void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                             void* stream, const q::QuantDst* qd) {
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

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid(P.max_splits, num_kv_heads, batch);
  if (q_dtype == ADA_DT_BF16)
    (void)ada::launch_k(attn::decode_split_kernel<__nv_bfloat16>, dim3(grid), dim3(attn::THREADS), 0, st, P);
  else
    (void)ada::launch_k(attn::decode_split_kernel<__half>, dim3(grid), dim3(attn::THREADS), 0, st, P);
  ADA_CHECK_LAUNCH();
  if (qd) {
    const int m_pad = (int)cdiv(batch, qd->bn) * qd->bn;
    const cl::RowSplit sp = cl::row_split(num_heads * head_dim / 16);
    if (!sp.maxu || sp.maxu > 4 || m_pad > 65535) return ADA_ERR_UNSUPPORTED;
    const dim3 rg((unsigned)sp.ctas, (unsigned)m_pad), rb((unsigned)sp.threads);
#define ADA_RQ(TO, MU)                                                                                         \
    (void)ada::launch_kc(attn::decode_reduce_quant_kernel<TO, MU>, rg, rb, 0, st, sp.ctas, P,                  \
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
  if (out_dtype == ADA_DT_BF16)
    (void)ada::launch_k(attn::decode_reduce_kernel<__nv_bfloat16>, dim3(rgrid), dim3(attn::D), 0, st, P, reinterpret_cast<__nv_bfloat16*>(out));
  else
    (void)ada::launch_k(attn::decode_reduce_kernel<__half>, dim3(rgrid), dim3(attn::D), 0, st, P, reinterpret_cast<__half*>(out));
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}