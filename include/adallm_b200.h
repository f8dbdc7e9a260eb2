/*
 * adallm_b200 -- C ABI of the B200 (sm_100a) kernels that replace the decode
 * hot path of the AdaLLM NVFP4 runtime (package `adallm`).
 *
 * Conventions
 *   - Every entry point returns an int status (ADA_OK == 0).  Nothing aborts
 *     or exits; bad arguments are reported before any launch.
 *   - Pointers are device pointers unless stated; sizes and strides are in
 *     elements of the pointed-to type.  `stream` is a cudaStream_t passed as
 *     void* so this header needs no CUDA include.
 *   - dtype codes: ADA_DT_BF16 = 0, ADA_DT_F16 = 1.
 *   - No entry point allocates or frees memory: outputs and workspaces are
 *     owned by the caller (the reference's ops allocate with torch.empty,
 *     adallm/ops/nvfp4_gemm.py:479, adallm/ops/attention.py:367; the Python
 *     layer of this package does the same with the torch caching allocator).
 *   - All launches go to `stream` and are CUDA-graph capturable.
 *
 * The reference interface each entry point replaces is cited beside it as
 * path:line inside the reference project.
 */
#ifndef ADALLM_B200_H_
#define ADALLM_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ADA_API __attribute__((visibility("default")))
#else
#define ADA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ADA_OK = 0,
  ADA_ERR_INVALID_ARG = 1,  /* null pointer, negative or inconsistent size  */
  ADA_ERR_UNSUPPORTED = 2,  /* shape this build does not implement          */
  ADA_ERR_ALIGNMENT = 3,    /* pointer / stride alignment rule violated      */
  ADA_ERR_WORKSPACE = 4,    /* workspace smaller than *_workspace_size()     */
  ADA_ERR_LAUNCH = 5,       /* CUDA reported an error at launch              */
  ADA_ERR_TIMEOUT = 6,      /* a bounded device-side wait gave up            */
  ADA_ERR_CUDA = 7          /* other CUDA runtime / driver failure           */
};

enum { ADA_DT_BF16 = 0, ADA_DT_F16 = 1 };

/* Human-readable text for a status code (static storage). */
ADA_API const char* ada_status_string(int status);
/* ABI version of this library (bumped on any signature change). */
ADA_API int ada_abi_version(void);
/* Programmatic dependent launch (on by default): every kernel may start while the previous
 * kernel on its stream drains, and waits on the device (griddepcontrol.wait) before reading
 * anything that kernel wrote.  ada_set_pdl(0) launches kernels with plain stream ordering.
 * Returns the previous setting.  Process-wide; set it before capturing graphs. */
ADA_API int ada_set_pdl(int enable);
/* CTA-pair GEMM (on by default): dense W4A4 (terms == 1) NVFP4 GEMMs large enough for the
 * persistent kernel, with N a multiple of 256, a 16-byte aligned output (ldy a multiple of 8)
 * and bias, run on pairs of SMs sharing one tcgen05 MMA of 256 tokens x 256 weight rows (the
 * prefill-size path of nvfp4_linear, adallm/ops/nvfp4_gemm.py:460-564).  ada_set_pair_gemm(0)
 * keeps them on the one-CTA 128 x 128 persistent kernel; results are the same either way.
 * Returns the previous setting.  Process-wide. */
ADA_API int ada_set_pair_gemm(int enable);

/* ------------------------------------------------------------------------
 * FP8 paged split-K decode attention
 * Replaces fp8_kv_decode_group_kernel + its launch in Attention.forward
 * (adallm/ops/attention.py:126-233, :359-414).
 *
 * q        [batch, num_heads, head_dim] (q_dtype), strides q_stride_b/q_stride_h, unit stride in D
 * k_cache, v_cache  e4m3fn bytes; element (page, row, kv_head, d) at
 *          page*kv_stride_page + row*kv_stride_tok + kv_head*kv_stride_head + d
 *          (the reference layout [num_pages, page, Hkv, D], adallm/runtime/model_runner.py:137-169);
 *          block ids outside [0, num_pages) are masked like the reference's -1 padding
 * block_tables int32 [batch, >= max_pages] with row stride bt_stride, -1 padded
 * context_lens int32 [batch]  (includes the current token; tokens past max_pages*page_size are ignored)
 * window   0 = full attention; W > 0 attends to tokens [max(ctx - W, 0), ctx)
 * k_scale, v_scale  per-tensor dequant scales of the cache (1.0 = reference)
 * out      [batch, num_heads, head_dim] (out_dtype), contiguous
 * Implemented: head_dim 128, num_heads/num_kv_heads in 1..8, page_size % 16 == 0.
 * A zero-length sequence produces zeros.
 * ---------------------------------------------------------------------- */
ADA_API size_t ada_fp8_paged_decode_workspace_size(int32_t batch, int32_t num_heads, int32_t max_pages,
                                           int32_t page_size, int32_t head_dim);
ADA_API int ada_fp8_paged_decode(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                         const uint8_t* k_cache, const uint8_t* v_cache, int64_t kv_stride_page,
                         int64_t kv_stride_tok, int64_t kv_stride_head, int64_t num_pages,
                         const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                         const int32_t* context_lens, int32_t batch, int32_t num_heads,
                         int32_t num_kv_heads, int32_t head_dim, int32_t page_size, float scale,
                         float k_scale, float v_scale, int32_t window, void* out, int out_dtype,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Same, with the split-K merge fused with the NVFP4 activation quantiser: the merged
 * attention row of every sequence ([num_heads * head_dim], rounded to out_dtype) is written
 * as the operand of o_proj in the ada_nvfp4_act_quant layout (xq / sfx / gx, `terms`,
 * block_n); `out` may be NULL.  num_heads * head_dim must be a multiple of 256. */
ADA_API int ada_fp8_paged_decode_quant(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                                       const uint8_t* k_cache, const uint8_t* v_cache,
                                       int64_t kv_stride_page, int64_t kv_stride_tok,
                                       int64_t kv_stride_head, int64_t num_pages,
                                       const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                                       const int32_t* context_lens, int32_t batch, int32_t num_heads,
                                       int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                                       float scale, float k_scale, float v_scale, int32_t window,
                                       void* out, int out_dtype, int terms, int block_n, uint8_t* xq,
                                       uint8_t* sfx, float* gx, void* workspace, size_t workspace_bytes,
                                       void* stream);
/* As ada_fp8_paged_decode_quant, with launch flags (no counterpart in the reference).
 * ADA_ATTN_META_EARLY: context_lens, block_tables and every cached K/V row except each sequence's
 * newest position (context_lens[b] - 1) were written at least two kernels earlier on `stream`
 * (e.g. the kernel just before is the one appending the new token's K/V): the short-cache kernel
 * then reads the metadata and starts its cache loads before waiting for that kernel, and the
 * long-cache kernel works out its split length (from context_lens) before that wait. */
#define ADA_ATTN_META_EARLY 1
ADA_API int ada_fp8_paged_decode_quant_ex(const void* q, int q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                                          const uint8_t* k_cache, const uint8_t* v_cache,
                                          int64_t kv_stride_page, int64_t kv_stride_tok,
                                          int64_t kv_stride_head, int64_t num_pages,
                                          const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                                          const int32_t* context_lens, int32_t batch, int32_t num_heads,
                                          int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                                          float scale, float k_scale, float v_scale, int32_t window,
                                          void* out, int out_dtype, int terms, int block_n, uint8_t* xq,
                                          uint8_t* sfx, float* gx, void* workspace, size_t workspace_bytes,
                                          int32_t flags, void* stream);

/* ------------------------------------------------------------------------
 * Causal prefill attention reading the FP8 paged cache in place
 * Replaces the prefix-cache prefill branch of Attention.forward (adallm/ops/attention.py:335-358):
 * _gather_kv_from_blocks (:254-286) + flash_attn_varlen_func(causal=True, window_size=(W, 0)).
 *
 * q        [total_q, num_heads, head_dim] (q_dtype), token stride q_stride_t, head stride
 *          q_stride_h, unit stride in D; sequence b owns rows [cu_seqlens_q[b], cu_seqlens_q[b+1])
 * cu_seqlens_q, cu_seqlens_k  int32 [batch + 1] (the reference's forward-context fields):
 *          len_k(b) = cu_seqlens_k[b+1] - cu_seqlens_k[b] keys, cached prefix + the new tokens,
 *          all already stored in the pages (store_kvcache runs first)
 * max_seqlen_q  max over b of len_q(b) (sizes the grid; larger is allowed; smaller leaves the
 *          rows past it unwritten, which the kernel cannot detect without reading cu_seqlens_q
 *          on the host)
 * k_cache, v_cache, block_tables, num_pages, page_size, k_scale, v_scale: as the decode entry
 * window   0 = causal only; W > 0: query i (0-based among the new tokens) sees keys
 *          [i + len_k - len_q - W, i + len_k - len_q] (flash-attn's window_size = (W, 0))
 * out      [total_q, num_heads, head_dim] (out_dtype), strides out_stride_t / out_stride_h
 * err      optional uint32 word: 0x70 is OR-ed in if a tile load wait ran out (~2 s)
 * scale * k_scale must be > 0.
 * Implemented: head_dim 128, num_heads / num_kv_heads <= 256, page_size % 16 == 0.  Rows that
 * see no key are written as zeros.  One CTA per 256 (token, head) rows of a KV head uses
 * 230 KB of shared memory and all 512 TMEM columns of its SM.
 * ---------------------------------------------------------------------- */
ADA_API int ada_fp8_paged_prefill(const void* q, int q_dtype, int64_t q_stride_t, int64_t q_stride_h,
                                  const uint8_t* k_cache, const uint8_t* v_cache, int64_t kv_stride_page,
                                  int64_t kv_stride_tok, int64_t kv_stride_head, int64_t num_pages,
                                  const int32_t* block_tables, int64_t bt_stride, int32_t max_pages,
                                  const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t batch,
                                  int32_t max_seqlen_q, int32_t num_heads, int32_t num_kv_heads,
                                  int32_t head_dim, int32_t page_size, float scale, float k_scale,
                                  float v_scale, int32_t window, void* out, int out_dtype,
                                  int64_t out_stride_t, int64_t out_stride_h, unsigned int* err, void* stream);

/* ------------------------------------------------------------------------
 * FP8 KV-cache store
 * Replaces store_kvcache / store_kvcache_kernel (adallm/ops/attention.py:11-31, :236-251).
 * key/value [num_tokens, num_kv_heads, head_dim] (in_dtype), row strides key_stride/value_stride,
 * heads contiguous (stride head_dim).  Row slot_mapping[i] of the cache viewed as
 * [-1, num_kv_heads*head_dim] receives e4m3(key[i] / k_scale) (round-to-nearest-even,
 * saturating); slot -1 is skipped.  cache_row_stride = elements between slots.
 * ---------------------------------------------------------------------- */
ADA_API int ada_store_kvcache_fp8(const void* key, const void* value, int in_dtype, int64_t num_tokens,
                          int32_t num_kv_heads, int32_t head_dim, int64_t key_stride,
                          int64_t value_stride, const int32_t* slot_mapping, uint8_t* k_cache,
                          uint8_t* v_cache, int64_t cache_row_stride, float k_scale, float v_scale,
                          void* stream);

/* ------------------------------------------------------------------------
 * RMSNorm family
 * Replaces RMSNorm.rms_forward / add_rms_forward (adallm/ops/layernorm.py:16-40) and
 * GemmaRMSNorm.rms_forward / add_rms_forward (adallm/ops/layernorm.py:64-92).
 * x [rows, hidden] (row stride ldx); weight [hidden]; y [rows, hidden] (row stride ldy).
 * residual == NULL: plain norm.  Otherwise sum = x + residual (row stride ld_res) is
 * written back to residual_out (row stride ld_res_out; may alias residual) and normalised.
 * gemma = 0: y = bf16(bf16(x*rsqrt) * w)   gemma = 1: y = bf16(x*rsqrt*(1+w))
 * ---------------------------------------------------------------------- */
ADA_API int ada_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ld_res,
                void* residual_out, int64_t ld_res_out, const void* weight, void* y, int64_t ldy,
                int64_t rows, int32_t hidden, float eps, int gemma, int dtype, void* stream);

/* RMSNorm fused with the NVFP4 activation quantiser: the normalised row (exactly what
 * ada_rmsnorm returns) is written as the GEMM operand in the ada_nvfp4_act_quant layout
 * (xq / sfx / gx for `terms` and block_n; rows up to ceil(rows/block_n)*block_n, padding
 * rows zero).  y may be NULL (no bf16 copy).  hidden must be a multiple of 256.  The row scale
 * comes from a bound on the normalised row's amax taken with its sum of squares (one cluster
 * exchange): amax_bound = rsqrt(mean(x^2) + eps) * max|x * w'| * (1 + 2^-6) (w' = w, or 1 + w
 * for gemma), never below the exact amax and at most ~2.4% above it; given that scale the codes
 * are exactly ada_nvfp4_act_quant's.  The same holds for every RMSNorm+quant producer below. */
ADA_API int ada_rmsnorm_quant(const void* x, int64_t ldx, const void* residual, int64_t ld_res,
                              void* residual_out, int64_t ld_res_out, const void* weight, void* y,
                              int64_t ldy, int64_t rows, int32_t hidden, float eps, int gemma, int dtype,
                              int terms, int block_n, uint8_t* xq, uint8_t* sfx, float* gx, void* stream);

/* ------------------------------------------------------------------------
 * Rotary embedding (NeoX rotate-half) from the reference's fp32 cos/sin cache
 * Replaces RotaryEmbedding.forward (adallm/ops/rotary_embedding.py:45-56).
 * positions int64 [num_tokens]; cos_sin [max_position, head_dim] fp32 = [cos | sin];
 * positions outside [0, max_position) are clamped into it (never read out of bounds).
 * q [num_tokens, num_q_heads, head_dim] row stride q_stride (heads contiguous), k likewise;
 * results go to q_out/k_out (contiguous [num_tokens, heads, head_dim]); may alias the inputs.
 * ---------------------------------------------------------------------- */
ADA_API int ada_rope(const int64_t* positions, const void* q, int64_t q_stride, const void* k,
             int64_t k_stride, void* q_out, void* k_out, int64_t num_tokens, int32_t num_q_heads,
             int32_t num_kv_heads, int32_t head_dim, const float* cos_sin, int64_t max_position,
             int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Fused attention-block prologue for decode: per token of the fused qkv row
 * [q heads | k heads | v heads] (row stride ld): q/k RMSNorm over head_dim with
 * q_norm_w / k_norm_w (adallm/architectures/qwen3.py:481-483; NULL weight = no norm),
 * RoPE from the fp32 cos/sin cache (adallm/ops/rotary_embedding.py:45-56), e4m3 store
 * of k and v at slot_mapping[t] into caches laid out [slots, num_kv_heads, head_dim]
 * (adallm/ops/attention.py:236-251), q written to q_out [T, num_q_heads, head_dim];
 * k_out (optional, may be NULL) receives the normalised, rotated k.  head_dim 128.
 * ---------------------------------------------------------------------- */
ADA_API int ada_qk_norm_rope_store(const void* qkv, int64_t ld, int64_t num_tokens, int32_t num_q_heads,
                                   int32_t num_kv_heads, int32_t head_dim, const void* q_norm_w,
                                   const void* k_norm_w, float eps, const int64_t* positions,
                                   const float* cos_sin, int64_t max_position, const int32_t* slot_mapping,
                                   uint8_t* k_cache, uint8_t* v_cache, float k_scale, float v_scale,
                                   void* q_out, void* k_out, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Gated activation: y[t, i] = act(x[t, i]) * x[t, I + i]
 * Replaces SiluAndMul / GeluAndMul (adallm/ops/activation.py:6-26).  act 0 = SiLU, 1 = GELU(tanh).
 * ---------------------------------------------------------------------- */
ADA_API int ada_gated_act(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t rows,
                  int32_t inter, int act, int dtype, void* stream);

/* Gated activation fused with the NVFP4 activation quantiser (operand of down_proj);
 * y may be NULL.  inter must be a multiple of 256. */
ADA_API int ada_gated_act_quant(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t rows,
                                int32_t inter, int act, int dtype, int terms, int block_n, uint8_t* xq,
                                uint8_t* sfx, float* gx, void* stream);

/* ------------------------------------------------------------------------
 * Token embedding gather: y[t] = table[ids[t]] (bf16/f16 rows of width hidden).
 * Replaces the lookup of VocabParallelEmbedding.forward (adallm/ops/embed_head.py:28-42)
 * at tensor-parallel size 1, and the per-rank masked lookup when vocab_start/vocab_end
 * delimit this rank's shard (rows outside it are written as zeros).
 * ---------------------------------------------------------------------- */
ADA_API int ada_embedding(const int64_t* ids, int64_t num_tokens, const void* table, int64_t vocab_start,
                  int64_t vocab_end, int32_t hidden, void* y, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * NVFP4 linear: y[m, n] = sum_k x[m, k] * W[n, k] (+ bias[n])
 * Replaces nvfp4_linear / nvfp4_gemm_kernel (adallm/ops/nvfp4_gemm.py:58-136, :460-564);
 * W uses the reference's parameter layout (adallm/ops/linear.py:31-43):
 *   w_packed  uint8 [N, K/2] (row stride ldw bytes), e2m1 codes, even k in the low nibble
 *   scales    [N, K/16] e4m3 values (stored as fp16 by the reference loader, or raw bytes)
 *   w_scale_2 fp32 per-tensor scale (device pointer to one float)
 * The scales are first re-laid out once per weight with ada_nvfp4_prepack_scales into
 * ada_nvfp4_sf_bytes(N, K) bytes (the layout the block-scaled tensor-core MMA reads;
 * this is the post-load hook next to adallm/infra/loader.py:129-162).
 * x [M, K] bf16/f16 (row stride ldx) is quantised on the device into `terms` e2m1 terms
 * (see ada_nvfp4_act_quant; 4 terms keep the result within ~1e-3 of the fp32
 * dequantise-then-matmul result, 1 = W4A4) and multiplied with tcgen05 kind::mxf4nvf4
 * MMAs.  y [M, N] bf16/f16, row stride ldy.
 * Implemented: N % 128 == 0, K % 256 == 0, terms in 1..8.
 * workspace: ada_nvfp4_linear_workspace_size(M, N, K, terms) bytes, 256-byte aligned; its
 * first 4 bytes are the error word (ada_nvfp4_workspace_status), which must be zero before
 * the first use.  Calls that share a workspace must be ordered (same stream).
 * ---------------------------------------------------------------------- */
ADA_API size_t ada_nvfp4_sf_bytes(int64_t n, int64_t k);
ADA_API int ada_nvfp4_prepack_scales(const void* scale, int scale_is_fp16, int64_t ld_scale, int64_t n,
                                     int64_t k, uint8_t* sf_out, void* stream);
ADA_API size_t ada_nvfp4_linear_workspace_size(int64_t m, int64_t n, int64_t k, int terms);
ADA_API int ada_nvfp4_linear(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k,
                             const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                             const float* w_scale_2, int64_t n, const void* bias, void* y, int y_dtype,
                             int64_t ldy, int terms, void* workspace, size_t workspace_bytes, void* stream);
/* The reference's W4A16 arithmetic for prefill-size M (adallm/ops/nvfp4_gemm.py:460-564):
 * x [M, K] bf16/f16 is cast to fp16 (bf16 input: into the workspace), the e2m1 weights are
 * widened to fp16 on chip (code value x e4m3 block scale, exact), and
 * tcgen05.mma.cta_group::2.kind::f16 tiles of 256 tokens x 256 weight rows accumulate in fp32;
 * the fp32 global scale and the bias are applied in the epilogue.  sf_w is the prepacked scale
 * layout of ada_nvfp4_prepack_scales.  Implemented: N % 256 == 0, K % 64 == 0; x, y, bias,
 * w_packed and sf_w 16-byte aligned, ldx and ldy multiples of 8, ldw a multiple of 16;
 * (N/256) x ceil(M/256) x (K/64) below 2^31 (else ADA_ERR_UNSUPPORTED).
 * workspace: ada_nvfp4_linear_w4a16_workspace_size(M, K) bytes, 256-byte aligned; its first 4
 * bytes are an error word (bounded waits that gave up OR a code into it).  Calls that share a
 * workspace must be ordered (same stream). */
ADA_API size_t ada_nvfp4_linear_w4a16_workspace_size(int64_t m, int64_t k);
ADA_API int ada_nvfp4_linear_w4a16(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k,
                                   const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                                   const float* w_scale_2, int64_t n, const void* bias, void* y, int y_dtype,
                                   int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);
/* Same as ada_nvfp4_linear with an explicit split-K factor (0 = library choice, else 1..8
 * CTAs per output tile; tests and tuning). */
ADA_API int ada_nvfp4_linear_ex(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k,
                                const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                                const float* w_scale_2, int64_t n, const void* bias, void* y, int y_dtype,
                                int64_t ldy, int terms, int force_ksplit, void* workspace,
                                size_t workspace_bytes, void* stream);
/* The activation quantiser on its own (the first half of ada_nvfp4_linear; no reference
 * counterpart -- the reference never quantises activations to e2m1).  Row m of x becomes:
 *   terms == 1   NVFP4: gx[m] = g = amax(row) / 2688, per 16-block ue4m3 scale
 *                s = e4m3(blockamax / (6g)) in sfx, codes e2m1(x / (s*g));
 *   terms 2..8   `terms` row-scaled e2m1 terms with unit block scales: gx[m] = g_0 =
 *                amax(row) / 6, term t has scale g_t = g_{t-1} / 6 and quantises the
 *                residual left by the terms before it (sfx unused, may be NULL).
 * Token m = mt*block_n + j, term t is operand row t*block_n + j of token tile mt:
 *   xq  [m_pad/block_n][terms*block_n][k/2]   packed e2m1, even k in the low nibble
 *   sfx [m_pad/block_n][k/64][512]            (terms == 1) ue4m3 scales, MMA scale-factor layout
 *   gx  [m_pad]                               (1.0 for the zero padding rows)
 * with m_pad = ceil(m / block_n) * block_n, block_n in {16, 32, 64, 128} and
 * terms * block_n <= 128 (ada_nvfp4_block_n(m, terms) gives the GEMM's choice). */
/* Grouped NVFP4 linear: row m of x uses expert expert_ids[m] (int32, in [0, num_experts)).
 * Replaces nvfp4_linear_gather (adallm/ops/nvfp4_gemm.py:657-714, kernel :363-457).  w_packed is the
 * contiguous stack [num_experts][n][k/2] (row stride ldw, expert stride n * ldw), sf_w its prepacked
 * scales (ada_nvfp4_prepack_scales of the [num_experts * n, k/16] scale matrix), w_scale_2 [num_experts].
 * A routing kernel gives every expert whole 16-row operand tiles, the quantiser gathers the rows into
 * them and one tensor-core GEMM streams only the weights of the experts in use; no host sync.  An id
 * outside the range sets the workspace error word (0x60) and leaves its row unwritten. */
ADA_API size_t ada_nvfp4_linear_grouped_workspace_size(int64_t m, int64_t n, int64_t k, int terms,
                                                       int32_t num_experts);
ADA_API int ada_nvfp4_linear_grouped(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k,
                                     const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                                     const float* w_scale_2, int32_t num_experts, int64_t n,
                                     const int32_t* expert_ids, void* y, int y_dtype, int64_t ldy, int terms,
                                     void* workspace, size_t workspace_bytes, void* stream);
/* MoE routing and combine around ada_nvfp4_linear_grouped (Qwen3MoeSparseMoeBlock.forward,
 * adallm/architectures/qwen3.py:1026-1032): ada_moe_route_topk takes router logits [tokens, experts]
 * (row stride ld; experts <= 1024, topk <= 32) to fp32 softmax, top-k (descending; ties: lower expert
 * first) and, when norm_topk_prob, weights renormalised to sum 1; writes ids int32 [tokens * topk] and
 * weights [tokens * topk] in dtype.  ada_moe_combine: out[t] = sum_j weights[t*topk+j] * y[t*topk+j]
 * (fp32, slot order; hidden % 8 == 0). */
ADA_API int ada_moe_route_topk(const void* logits, int dtype, int64_t ld, int64_t tokens, int32_t experts,
                               int32_t topk, int32_t norm_topk_prob, int32_t* ids, void* weights, void* stream);
/* The router GEMM (router_logits = x . router_w^T, rounded to dtype as the reference's F.linear
 * output, qwen3.py:1026) fused with ada_moe_route_topk: x [tokens, hidden], router_w [experts,
 * hidden] (row strides ldx, ldw; hidden % 8 == 0, experts <= 1024); ids / weights as
 * ada_moe_route_topk.  err: a device word ORed with 0x80 if a bounded wait ran out. */
ADA_API int ada_moe_router_topk(const void* x, int dtype, int64_t ldx, int64_t tokens, const void* router_w,
                                int64_t ldw, int32_t hidden, int32_t experts, int32_t topk, int32_t norm_topk_prob,
                                int32_t* ids, void* weights, unsigned int* err, void* stream);
ADA_API int ada_moe_combine(const void* y, int dtype, int64_t ldy, const void* weights, int64_t tokens,
                            int32_t topk, int32_t hidden, void* out, int64_t ldo, void* stream);
/* Expert parallelism (no reference counterpart: the reference runs MoE at TP = 1 only,
 * qwen3.py:1383).  Each rank holds experts [expert_base, expert_base + num_local) of the model.
 * ada_nvfp4_linear_grouped_ep is ada_nvfp4_linear_grouped over the rank's stacked local experts
 * ([num_experts = num_local][n][k/2]): rows routed to another rank's expert are skipped (their
 * output rows are left untouched), not an error.  ada_moe_combine_ep sums only the slots whose
 * expert (expert_ids [tokens][topk]) is local; summing the ranks' outputs (all-reduce) gives
 * the block's output. */
ADA_API int ada_nvfp4_linear_grouped_ep(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k,
                                        const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                                        const float* w_scale_2, int32_t num_experts, int32_t expert_base,
                                        int64_t n, const int32_t* expert_ids, void* y, int y_dtype, int64_t ldy,
                                        int terms, void* workspace, size_t workspace_bytes, void* stream);
ADA_API int ada_moe_combine_ep(const void* y, int dtype, int64_t ldy, const void* weights,
                               const int32_t* expert_ids, int32_t expert_base, int32_t num_local, int64_t tokens,
                               int32_t topk, int32_t hidden, void* out, int64_t ldo, void* stream);
/* ada_moe_combine_ep with the rank's fp32 sums left unrounded (out fp32, ldo % 4 == 0): an fp32
 * all-reduce of them, rounded once to the model dtype, is the single-GPU combine up to the order
 * of the fp32 additions. */
ADA_API int ada_moe_combine_ep_f32(const void* y, int dtype, int64_t ldy, const void* weights,
                                   const int32_t* expert_ids, int32_t expert_base, int32_t num_local,
                                   int64_t tokens, int32_t topk, int32_t hidden, float* out, int64_t ldo,
                                   void* stream);
/* The expert MLP of a MoE block in one call (Qwen3MoeSparseMoeBlock's expert loop,
 * adallm/architectures/qwen3.py:1263-1290, for the rows routed to this rank's experts): for every
 * routed row r = t * topk + j with expert e = expert_ids[r] in [expert_base, expert_base +
 * num_experts): y[r] = down_e(act(gate_e(x[t])) * up_e(x[t])), act SiLU (0) or GELU-tanh (1).
 * w_gate_up is the stack [num_experts][2 * inter][hidden / 2] (gate rows first, row stride
 * ld_gate_up), w_down [num_experts][hidden][inter / 2]; sf_* their prepacked scales, scale2_*
 * [num_experts].  One routing (16-row expert tiles) serves both projections; x's rows are gathered
 * by the quantiser, act(gate) * up is quantised straight into the down operand.  Rows routed to
 * another rank's expert are left untouched when all_local == 0, an error (workspace error word)
 * when all_local == 1.  workspace: ada_moe_experts_workspace_size bytes, 256-byte aligned, its
 * first 4 bytes the error word (zero before the first use). */
ADA_API size_t ada_moe_experts_workspace_size(int64_t tokens, int32_t topk, int64_t hidden, int64_t inter, int terms,
                                              int32_t num_experts);
ADA_API int ada_moe_experts(const void* x, int x_dtype, int64_t ldx, int64_t tokens, int32_t topk,
                            const int32_t* expert_ids, int32_t num_experts, int32_t expert_base, int32_t all_local,
                            const uint8_t* w_gate_up, int64_t ld_gate_up, const uint8_t* sf_gate_up,
                            const float* scale2_gate_up, const uint8_t* w_down, int64_t ld_down,
                            const uint8_t* sf_down, const float* scale2_down, int64_t inter, int64_t hidden, int act,
                            void* y, int64_t ldy, int terms, void* workspace, size_t workspace_bytes, void* stream);
ADA_API int ada_nvfp4_act_quant(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k, int terms,
                                int block_n, uint8_t* xq, uint8_t* sfx, float* gx, void* stream);
/* The tensor-core GEMM on its own, for activations already quantised by
 * ada_nvfp4_act_quant (or by a fused producer writing the same layout) with
 * block_n == ada_nvfp4_block_n(m, terms) (sfx only read for terms == 1).  workspace:
 * ada_nvfp4_gemm_workspace_size(m, n, k, terms) bytes (the error word), 256-byte aligned,
 * zero before first use.  force_ksplit: 0 = library choice, else the number of CTAs (1..8,
 * one thread-block cluster) that split each output tile's K range. */
ADA_API int ada_nvfp4_block_n(int64_t m, int terms);
ADA_API size_t ada_nvfp4_gemm_workspace_size(int64_t m, int64_t n, int64_t k, int terms);
ADA_API int ada_nvfp4_gemm(const uint8_t* xq, const uint8_t* sfx, const float* gx, int64_t m, int terms,
                           int block_n, const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                           const float* w_scale_2, int64_t n, int64_t k, const void* bias, void* y,
                           int y_dtype, int64_t ldy, int force_ksplit, void* workspace,
                           size_t workspace_bytes, void* stream);
/* Reads the device error word of an NVFP4 workspace (0 = ok; bit 1/2/4 = a bounded
 * pipeline wait timed out).  Synchronises `stream`.  Not capturable. */
ADA_API int ada_nvfp4_workspace_status(const void* workspace, int64_t m, int64_t n, int64_t k, int terms,
                                       unsigned int* status_out, void* stream);

/* Split-K partial mode of the GEMM (no reference counterpart; used by the decode engine):
 * instead of reducing its K splits, the GEMM writes each split's scaled fp32 partial
 * y_s[m, n] to parts + s * part_plane + m * part_ld + n (s < nplanes, m < M), and the
 * kernel that consumes the output sums the planes in order (the *_parts entry points
 * below), which gives bit for bit what ada_nvfp4_gemm with the same split count stores.
 * nplanes: 1..8 (ada_nvfp4_gemm_splits gives the library's choice: as many splits as
 * keep every CTA resident); no bias.  workspace as ada_nvfp4_gemm. */
ADA_API int ada_nvfp4_gemm_splits(int64_t m, int64_t n, int64_t k, int terms);
ADA_API int ada_nvfp4_gemm_partials(const uint8_t* xq, const uint8_t* sfx, const float* gx, int64_t m, int terms,
                                    int block_n, const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                                    const float* w_scale_2, int64_t n, int64_t k, float* parts, int64_t part_ld,
                                    int64_t part_plane, int nplanes, void* workspace, size_t workspace_bytes,
                                    void* stream);

/* ada_nvfp4_gemm_partials with the next projection's weights pulled into L2: once each CTA has
 * issued its own loads it requests its share of [next_w, next_w + next_w_bytes) and
 * [next_sf, + next_sf_bytes) into L2 (fire-and-forget prefetches, no result, no wait), so the
 * GEMM after the latency-bound kernels between the two finds its weights in L2.  Either range may
 * be NULL / 0; addresses and sizes 16-byte aligned.  No reference counterpart. */
ADA_API int ada_nvfp4_gemm_partials_pf(const uint8_t* xq, const uint8_t* sfx, const float* gx, int64_t m, int terms,
                                       int block_n, const uint8_t* w_packed, int64_t ldw, const uint8_t* sf_w,
                                       const float* w_scale_2, int64_t n, int64_t k, float* parts, int64_t part_ld,
                                       int64_t part_plane, int nplanes, const void* next_w, size_t next_w_bytes,
                                       const void* next_sf, size_t next_sf_bytes, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Tensor parallelism over NVLink peer memory (no counterpart in the reference, whose row-parallel
 * linears all-reduce their outputs with NCCL, adallm/ops/linear.py:193-215).  One process per GPU;
 * every rank allocates an inbox with ada_peer_alloc, the ranks exchange the 64-byte handles
 * (e.g. with torch.distributed) and map the peers' inboxes with ada_peer_open.  Plain peer stores
 * and loads; no multicast object.
 *
 * ada_nvfp4_gemm_partials_peer: the partial-plane GEMM of a row-parallel projection (this rank's
 * K shard) writes its fp32 partial of K split s into plane tp_rank * nplanes + s of EVERY rank's
 * inbox (inboxes[d] = rank d's inbox as mapped here, 16-byte aligned; planes of 8-byte words
 * [world * nplanes][m][part_ld]).  Each word is the value's bits | tag << 32 with
 * tag = *epoch * tag_mul + tag_add, written by one 8-byte store, so no fence or counter is needed.
 * ada_rmsnorm_quant_peer: ada_rmsnorm_quant_parts over this rank's inbox (nparts = world * nplanes,
 * summed in plane order, so every rank computes the same rows), polling each word until its tag is
 * this step's (bounded, ~2 s; then *err = 0x50 and the stale words are used).
 * *epoch counts the steps completed on this rank; ada_tp_epoch_advance(epoch) ends a step (after
 * its last consumer); give each projection of each layer its own tag_add in [1, tag_mul].  An inbox
 * may be rewritten by the peers only after this rank's consumer finished reading it: use one inbox
 * per projection kind (o_proj, down_proj), whose next writes depend, through the other kind's
 * words, on this rank having moved on. */
#define ADA_PEER_HANDLE_BYTES 64
ADA_API int ada_peer_alloc(size_t bytes, void** ptr, void* handle);
ADA_API int ada_peer_open(const void* handle, void** ptr);
ADA_API int ada_peer_close(void* ptr);
ADA_API int ada_peer_free(void* ptr);
ADA_API int ada_tp_epoch_advance(uint32_t* epoch, void* stream);
ADA_API int ada_nvfp4_gemm_ctas(int64_t m, int64_t n, int64_t k, int terms, int nplanes);
ADA_API int ada_nvfp4_gemm_partials_peer(const uint8_t* xq, const uint8_t* sfx, const float* gx, int64_t m,
                                         int terms, int block_n, const uint8_t* w_packed, int64_t ldw,
                                         const uint8_t* sf_w, const float* w_scale_2, int64_t n, int64_t k,
                                         int64_t part_ld, int64_t part_plane, int nplanes, int32_t world,
                                         int32_t tp_rank, void* const* inboxes, const uint32_t* epoch,
                                         uint32_t tag_mul, uint32_t tag_add, void* workspace,
                                         size_t workspace_bytes, void* stream);
ADA_API int ada_rmsnorm_quant_peer(const void* inbox, int32_t nparts, int64_t plane, int64_t ldp,
                                   const void* residual, int64_t ld_res, void* residual_out, int64_t ld_res_out,
                                   const void* weight, void* y, int64_t ldy, int64_t rows, int32_t hidden,
                                   float eps, int gemma, int dtype, int terms, int block_n, uint8_t* xq,
                                   uint8_t* sfx, float* gx, const uint32_t* epoch, uint32_t tag_mul,
                                   uint32_t tag_add, uint32_t* err, void* stream);

/* Consumers of partial planes (parts: nparts fp32 planes, plane / ldp = floats between planes /
 * rows, 16-byte aligned): the input element is the plane sum rounded to dtype, then exactly
 * ada_rmsnorm_quant (xq == NULL: plain RMSNorm into y), ada_gated_act_quant and
 * ada_qk_norm_rope_store. */
ADA_API int ada_rmsnorm_quant_parts(const float* parts, int32_t nparts, int64_t plane, int64_t ldp,
                                    const void* residual, int64_t ld_res, void* residual_out, int64_t ld_res_out,
                                    const void* weight, void* y, int64_t ldy, int64_t rows, int32_t hidden, float eps,
                                    int gemma, int dtype, int terms, int block_n, uint8_t* xq, uint8_t* sfx,
                                    float* gx, void* stream);
/* RMSNorm whose input row is the MoE block's weighted combine (the reference's
 * sum_k w_k * expert_k(x) of Qwen3MoeSparseMoeBlock, qwen3.py:1263-1290): element (t, c) =
 * sum_j route_w[t][j] * y_rows[t * topk + j][c] (fp32, slot order, rounded to dtype), i.e.
 * exactly ada_moe_combine's output, then exactly ada_rmsnorm_quant (xq == NULL: plain RMSNorm
 * into y).  Replaces the combine kernel and the next layer's input norm by one launch. */
ADA_API int ada_rmsnorm_quant_combine(const void* y_rows, int64_t ld_rows, const void* route_w, int32_t topk,
                                      const void* residual, int64_t ld_res, void* residual_out, int64_t ld_res_out,
                                      const void* weight, void* y, int64_t ldy, int64_t rows, int32_t hidden,
                                      float eps, int gemma, int dtype, int terms, int block_n, uint8_t* xq,
                                      uint8_t* sfx, float* gx, void* stream);
ADA_API int ada_gated_act_quant_parts(const float* parts, int32_t nparts, int64_t plane, int64_t ldp, void* y,
                                      int64_t ldy, int64_t rows, int32_t inter, int act, int dtype, int terms,
                                      int block_n, uint8_t* xq, uint8_t* sfx, float* gx, void* stream);
ADA_API int ada_qk_norm_rope_store_parts(const float* parts, int32_t nparts, int64_t plane, int64_t ldp,
                                         int64_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                                         int32_t head_dim, const void* q_norm_w, const void* k_norm_w, float eps,
                                         const int64_t* positions, const float* cos_sin, int64_t max_position,
                                         const int32_t* slot_mapping, uint8_t* k_cache, uint8_t* v_cache,
                                         float k_scale, float v_scale, void* q_out, void* k_out, int dtype,
                                         void* stream);

/* Gemma3 forms of the producers (adallm/architectures/gemma3.py:156-181; norms layernorm.py:64-92).
 * ada_gemma_norm2_quant_parts: the projection output (sum of the partial planes, rounded to
 * dtype) goes through GemmaRMSNorm(post_weight) -- the layer's post-attention or post-feedforward
 * norm -- then joins the residual stream (bf16: native add, rounded; the new residual is written
 * to residual_out) and the sum goes through GemmaRMSNorm(weight) -- the next pre-attention /
 * pre-feedforward / final norm -- quantised into (xq, sfx, gx) as ada_rmsnorm_quant does
 * (xq == NULL: plain norm into y).  Bit for bit the reference's
 *   h = post_norm(o); x, residual = pre_norm(h, residual).
 * ada_qk_norm_rope_store[_parts]_ex: ada_qk_norm_rope_store[_parts] with the per-head norm
 * chosen by `gemma` (0: RMSNorm, cast then weight multiply; 1: GemmaRMSNorm, x * rs * (1 + w)
 * then cast, gemma3.py:88-89). */
ADA_API int ada_gemma_norm2_quant_parts(const float* parts, int32_t nparts, int64_t plane, int64_t ldp,
                                        const void* post_weight, const void* residual, int64_t ld_res,
                                        void* residual_out, int64_t ld_res_out, const void* weight, void* y,
                                        int64_t ldy, int64_t rows, int32_t hidden, float eps, int dtype, int terms,
                                        int block_n, uint8_t* xq, uint8_t* sfx, float* gx, void* stream);
ADA_API int ada_qk_norm_rope_store_parts_ex(const float* parts, int32_t nparts, int64_t plane, int64_t ldp,
                                            int64_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                                            int32_t head_dim, const void* q_norm_w, const void* k_norm_w, float eps,
                                            int gemma, const int64_t* positions, const float* cos_sin,
                                            int64_t max_position, const int32_t* slot_mapping, uint8_t* k_cache,
                                            uint8_t* v_cache, float k_scale, float v_scale, void* q_out, void* k_out,
                                            int dtype, void* stream);
ADA_API int ada_qk_norm_rope_store_ex(const void* qkv, int64_t ld, int64_t num_tokens, int32_t num_q_heads,
                                      int32_t num_kv_heads, int32_t head_dim, const void* q_norm_w,
                                      const void* k_norm_w, float eps, int gemma, const int64_t* positions,
                                      const float* cos_sin, int64_t max_position, const int32_t* slot_mapping,
                                      uint8_t* k_cache, uint8_t* v_cache, float k_scale, float v_scale, void* q_out,
                                      void* k_out, int dtype, void* stream);

/* Vocabulary projection with the greedy pick fused in.  Replaces ParallelLMHead.forward's
 * F.linear (adallm/ops/embed_head.py:56-66) followed by the greedy argmax over its bf16 logits.
 * x bf16 [m, k] (row stride ldx), w bf16 [vocab, k] (row stride ldw): logits = x . w^T with fp32
 * accumulation rounded to bf16 (written to `logits` [m][ldl] when it is not NULL); out_idx[r] =
 * idx_base + the first row of the maximum bf16 logit of token r (torch.argmax), out_val[r] = that
 * logit as fp32 (either may be NULL).  idx_base: the first vocabulary row of this shard.
 * Implemented: m <= 64, k % 64 == 0, x / w 16-byte aligned with ldx, ldw % 8 == 0.
 * workspace: ada_lm_head_workspace_size(m, vocab) bytes, 256-byte aligned (first 4 bytes: the
 * error word, a bounded pipeline wait that ran out ORs 1/2/4/8 into it).  Two kernels: the
 * persistent tcgen05 projection (one CTA per SM) and the cross-tile pick. */
ADA_API size_t ada_lm_head_workspace_size(int64_t m, int64_t vocab);
ADA_API int ada_lm_head_argmax(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw,
                               int64_t vocab, int64_t idx_base, void* logits, int64_t ldl, int64_t* out_idx,
                               float* out_val, void* workspace, size_t workspace_bytes, void* stream);

/* Greedy sampling helper: out[r] = argmax_j logits[r, j] (first maximum, like torch.argmax),
 * logits bf16/f16.  workspace: ada_argmax_workspace_size(rows, cols) bytes, 8-byte aligned. */
ADA_API size_t ada_argmax_workspace_size(int64_t rows, int64_t cols);
ADA_API int ada_argmax(const void* logits, int64_t ld, int64_t rows, int64_t cols, int dtype,
                       int64_t* out, void* workspace, size_t workspace_bytes, void* stream);
/* ada_argmax without a caller workspace: no counterpart in the reference (its sampler runs
 * torch.argmax).  For callers that cannot allocate device memory where they sample (a host
 * runtime binding this ABI directly, launching into work it records, where cudaMalloc is not
 * allowed).  Partials go through a 256 KiB scratch array inside the library:
 * rows * chunks(cols) * 12 + 16 must be <= 256 KiB (ada_argmax_workspace_size(rows, cols);
 * e.g. up to 291 rows of a 151936-entry vocabulary), else ADA_ERR_WORKSPACE.  The first call on
 * each device looks up the scratch address (make it before recording launches); a call with
 * rows == 0 does only that set-up, so a runtime that records every launch can make it first.
 * Nothing needs to start at zero.  One scratch per device: calls overlapping in time on a
 * device race. */
ADA_API int ada_argmax_noalloc(const void* logits, int64_t ld, int64_t rows, int64_t cols, int dtype,
                               int64_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ADALLM_B200_H_ */
