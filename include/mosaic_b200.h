/*
 * mosaic_b200 — C ABI of the B200 (sm_100a) block-sparse attention forward of
 * Mosaic (maxxxzdn/mosaic). Every entry point takes plain device pointers,
 * sizes and a cudaStream_t (passed as void*), launches asynchronously on that
 * stream, allocates nothing and synchronises nothing. Tensors are dense and
 * row-major in the reference's layouts ([batch, seq, heads, head_dim]); head_dim
 * is 64. Any number of query heads per kv head (G = num_q_heads / num_kv_heads)
 * is accepted by the attention and backward entry points; the top-k selection (and
 * so mosaic_bsa_fwd outside block_attn_only) takes G = 1 to 8. The kernels
 * work on groups of four query heads: G = 4 and 8 fill them, G = 1 and 2 leave
 * three or two of the four head slots empty (computed on zeros, not written).
 * The attention entry points take a
 * `dtype` (MOSAIC_DTYPE_BF16 or MOSAIC_DTYPE_F16) for all their 16-bit tensors; the
 * projection, interpolation, resampling and backward entry points are bf16.
 *
 * Return value: MOSAIC_OK or a MOSAIC_ERR_* code (argument errors are detected
 * on the host before anything is launched). Faults detected on the device are
 * OR-ed into the optional int32 status word (`status`, device memory) as
 * MOSAIC_STATUS_* bits; the caller reads it when it wants to (no implicit sync).
 */
#ifndef MOSAIC_B200_H_
#define MOSAIC_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOSAIC_API __attribute__((visibility("default")))
#else
#define MOSAIC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes ---------------------------------------------------- */
#define MOSAIC_OK 0
#define MOSAIC_ERR_INVALID_ARGUMENT 1 /* null pointer, negative size, misaligned pointer */
#define MOSAIC_ERR_UNSUPPORTED 2      /* a shape this build does not handle (head_dim != 64, top-k with G > 8, ...) */
#define MOSAIC_ERR_WORKSPACE 3        /* workspace missing or smaller than mosaic_bsa_workspace_bytes() */
#define MOSAIC_ERR_CUDA 4             /* a CUDA runtime / driver call failed (launch, tensor map) */

/* ---- activation types (the `dtype` arguments) --------------------------- */
#define MOSAIC_DTYPE_BF16 0 /* bfloat16 */
#define MOSAIC_DTYPE_F16 1  /* IEEE half: the reference's dtype under torch.autocast(float16)
                               (inference.py:59,379); pooled means and top-k scores are then
                               rounded to fp16 as its attn_topk does (primitives.py:37-49) */

/* ---- device status bits (OR-ed into *status) -------------------------- */
#define MOSAIC_STATUS_TIMEOUT 1   /* a pipeline wait exceeded its time limit; the kernel gave up */
#define MOSAIC_STATUS_BAD_INDEX 2 /* a block index was outside [0, seq_len / block_size); it was clamped to 0 */

/* Arguments of mosaic_bsa_fwd (the flags mirror primitives.mosaic_attn_func). */
typedef struct MosaicBsaArgs {
  const void* q;        /* [B, N, Hq, 64] dtype                                           */
  const void* k;        /* [B, N, Hk, 64] dtype                                           */
  const void* v;        /* [B, N, Hk, 64] dtype                                           */
  const void* gates;    /* [3, B, N, Hq] dtype = weight_ba_cmp_slc; NULL iff block_attn_only */
  const float* rope_cos; /* [N, 32] fp32 or NULL. When set, q and k are NOT yet rotated:   */
  const float* rope_sin; /*   the library applies Mosaic's 2D RoPE before pooling.          */
  void* out;            /* [B, N, Hq, 64] dtype                                           */
  int64_t* block_indices; /* [B, N/bs, Hk, K] int64 selected blocks (written); may be NULL */
  void* workspace;      /* device scratch of >= mosaic_bsa_workspace_bytes() bytes, 256-aligned */
  size_t workspace_bytes;
  int* status;          /* device int32 status word or NULL                               */
  int batch;            /* B  */
  int seq_len;          /* N  */
  int num_q_heads;      /* Hq */
  int num_kv_heads;     /* Hk */
  int head_dim;         /* must be 64 */
  int block_attn_size;  /* local window length (primitives.block_attention)               */
  int sparse_block_size;  /* bs: pooling / selection block length, multiple of 64         */
  int sparse_block_count; /* K: selected blocks per query block (0 = no selected branch)  */
  int block_attn_only;  /* != 0: return the local branch only                              */
  int no_compression;   /* != 0: drop the compressed branch, renormalise w_ba / w_slc       */
  float softmax_scale;  /* <= 0 selects head_dim^-0.5                                      */
  int dtype;            /* MOSAIC_DTYPE_BF16 or MOSAIC_DTYPE_F16                           */
} MosaicBsaArgs;

/* Version of this ABI (bumped on any signature or struct change). */
MOSAIC_API int mosaic_abi_version(void);

/* Human-readable text for a MOSAIC_ERR_* code. */
MOSAIC_API const char* mosaic_error_string(int code);

/* Self-test of the device-side failure detection used by every pipeline kernel:
 * a single warp waits (up to timeout_us microseconds) on a barrier that nothing
 * arrives on; the bounded wait gives up, OR-s MOSAIC_STATUS_TIMEOUT into *status
 * and writes result[0] = 0 (wait succeeded: 1) and result[1] = 1 (abort flag
 * raised). Both pointers are device memory. No counterpart in the reference,
 * which has no failure detection. */
MOSAIC_API int mosaic_selftest_wait_timeout(int* status, int* result, int timeout_us, void* stream);

/* Scratch bytes mosaic_bsa_fwd needs for these sizes (pooled q/k/v, coarse
 * attention output, block indices and, with RoPE, rotated q/k). */
MOSAIC_API size_t mosaic_bsa_workspace_bytes(int batch, int seq_len, int num_q_heads, int num_kv_heads, int head_dim,
                                  int sparse_block_size, int sparse_block_count, int with_rope);

/* Full Mosaic block-sparse attention forward: local block attention, compressed
 * attention over mean-pooled blocks, top-k block selection, selected-block
 * attention, gated combine.
 * Replaces primitives.mosaic_attn_func (primitives.py:54-89) including the
 * flash_attn_func calls at primitives.py:31 and :77 and ops.mosaic_sparse_attn
 * (ops.py:557-566) it makes. */
MOSAIC_API int mosaic_bsa_fwd(const MosaicBsaArgs* args, void* stream);

/* mosaic_bsa_fwd for callers that cannot allocate device memory (a foreign-language
 * host with no device allocator, or a service with a fixed memory budget that must
 * not call cudaMalloc/cudaFree per request). It has no counterpart in the reference.
 * args->workspace / workspace_bytes are ignored: the scratch is an 8 MiB array
 * compiled into the library (held on every device that loads it until exit), so
 * calls needing more than 8 MiB of scratch (mosaic_bsa_workspace_bytes) return
 * MOSAIC_ERR_WORKSPACE, and fused RoPE (rope_cos/rope_sin) returns
 * MOSAIC_ERR_UNSUPPORTED; a rejected call launches nothing and writes nothing to
 * out or block_indices. The first call on a device looks up the array's address
 * and keeps it for the life of the process: make that call before any stream
 * capture, and do not use this entry point on a device after cudaDeviceReset (the
 * kept address then belongs to the destroyed context). All calls on a device share
 * the array: calls that overlap on the GPU race and must be serialised by the
 * caller. */
MOSAIC_API int mosaic_bsa_fwd_noalloc(const MosaicBsaArgs* args, void* stream);

/* The fused attention stage of mosaic_bsa_fwd on its own: local-window attention
 * + selected-block attention over the given block_indices + the gated combine
 * with the coarse-attention rows o_cmp ([B, N/bs, Hq, 64] bf16, NULL when
 * no_compression or when sparse_block_count == 0 uses only (w_ba, w_cmp)).
 * combine: 0 = w0*o_ba + w1*o_cmp + w2*o_slc (primitives.py:89),
 *          1 = no_compression renormalisation (primitives.py:71-74),
 *          2 = sparse_block_count == 0 renormalisation (primitives.py:81-84). */
MOSAIC_API int mosaic_bsa_attend_fwd(const void* q, const void* k, const void* v, const int64_t* block_indices,
                                     const void* gates, const void* o_cmp, void* out, int* status, int batch,
                                     int seq_len, int num_q_heads, int num_kv_heads, int head_dim,
                                     int block_attn_size, int sparse_block_size, int sparse_block_count,
                                     int combine, float softmax_scale, int dtype, void* stream);

/* Selected-block attention: out[b,n,j] = softmax over the K*bs keys of blocks
 * block_indices[b, n/bs, j/G, :] of kv head j/G. Optional lse (log2 units, fp32
 * [B,N,Hq]). Replaces ops.mosaic_attn_fwd / mosaic_attn_fwd_kernel
 * (ops.py:137-176, ops.py:25-134) behind ops.mosaic_sparse_attn (ops.py:557). */
MOSAIC_API int mosaic_sparse_attn_fwd(const void* q, const void* k, const void* v, const int64_t* block_indices, void* out,
                           float* lse, int* status, int batch, int seq_len, int num_q_heads, int num_kv_heads,
                           int head_dim, int block_size, int block_count, float softmax_scale, int dtype,
                           void* stream);

/* Local block attention: full (non-causal) GQA attention inside each window of
 * block_size consecutive tokens. Replaces primitives.block_attention
 * (primitives.py:28-32) = flash_attn_func on [(B*N/bs), bs, H, 64]. */
MOSAIC_API int mosaic_block_attn_fwd(const void* q, const void* k, const void* v, void* out, int* status, int batch,
                          int seq_len, int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                          float softmax_scale, int dtype, void* stream);

/* Mean-pool q, k, v over contiguous blocks of block_size tokens (fp32 sums,
 * results rounded to dtype); with rope_cos/rope_sin set, rotate q and k first and also write
 * the rotated tensors to q_rot / k_rot. q_cmp and v_cmp may be NULL to skip them.
 * Replaces the einops reduce calls at primitives.py:65-66,76 and, with RoPE,
 * RoPE.forward (primitives.py:132-135) for q and k. */
MOSAIC_API int mosaic_block_pool(const void* q, const void* k, const void* v, const float* rope_cos, const float* rope_sin,
                      void* q_rot, void* k_rot, void* q_cmp, void* k_cmp, void* v_cmp, int batch, int seq_len,
                      int num_q_heads, int num_kv_heads, int head_dim, int block_size, int dtype,
                      void* stream);

/* Coarse (compressed) attention over nb pooled tokens: full GQA attention with
 * scale softmax_scale. Replaces flash_attn_func(q_cmp, k_cmp, v_cmp) at
 * primitives.py:77 (without the repeat_interleave of :78, which the fused
 * epilogue of mosaic_bsa_fwd does by indexing). */
MOSAIC_API int mosaic_cmp_attn_fwd(const void* q_cmp, const void* k_cmp, const void* v_cmp, void* o_cmp, int* status,
                        int batch, int num_blocks, int num_q_heads, int num_kv_heads, int head_dim,
                        float softmax_scale, int dtype, void* stream);

/* Top-k block selection: scores_j = q_cmp[:, :, j] . k_cmp[:, :, j/G]^T (fp32 sums
 * rounded to dtype), mean over the strided head group {h, h+Hk, ...} (rounded to
 * dtype), then the indices of
 * the block_count largest per (b, query block, kv head), sorted by score
 * descending, ties to the lower index. Replaces primitives.attn_topk
 * (primitives.py:35-51). */
MOSAIC_API int mosaic_attn_topk(const void* q_cmp, const void* k_cmp, int64_t* block_indices, int batch, int num_blocks,
                     int num_q_heads, int num_kv_heads, int head_dim, int block_count, int dtype,
                     void* stream);

/* Scratch bytes mosaic_sparse_attn_bwd needs for these sizes (row dot products
 * D = rowsum(out * grad_out) and the inverted block index). */
MOSAIC_API size_t mosaic_sparse_attn_bwd_workspace_bytes(int batch, int seq_len, int num_q_heads, int num_kv_heads,
                                                         int head_dim, int block_size, int block_count);

/* Backward of mosaic_sparse_attn_fwd: given the forward's out and lse (log2 units,
 * as mosaic_sparse_attn_fwd writes it) and grad_out, writes grad_q [B,N,Hq,64],
 * grad_k and grad_v [B,N,Hk,64] (bf16, every element written). grad_q sums over
 * every selection of the query block (duplicates count twice, as in the forward);
 * grad_k / grad_v sum over the distinct query blocks that selected each kv block.
 * Replaces ops.mosaic_attn_bwd (ops.py:436-507) with its kernels
 * mosaic_attn_bwd_q_kernel (ops.py:184-274), mosaic_block_mask (ops.py:277-297)
 * and mosaic_attn_bwd_kv_kernel (ops.py:305-433), behind
 * ops.MosaicAttnFunction.backward (ops.py:542-554). */
MOSAIC_API int mosaic_sparse_attn_bwd(const void* q, const void* k, const void* v, const void* out,
                                      const void* grad_out, const float* lse, const int64_t* block_indices,
                                      void* grad_q, void* grad_k, void* grad_v, void* workspace,
                                      size_t workspace_bytes, int* status, int batch, int seq_len, int num_q_heads,
                                      int num_kv_heads, int head_dim, int block_size, int block_count,
                                      float softmax_scale, void* stream);

/* Input projections of primitives.MosaicAttention.forward (primitives.py:182-194):
 * [q | k | v | gate logits] = x W^T with W = cat(to_q.weight, to_k.weight, to_v.weight,
 * to_strategy_combine_mlp.weight) ([(Hq + 2 Hk) 64 + 3 Hq, dim] bf16; without the gate
 * rows when gates is NULL), x [S, B, dim] bf16 (sequence-first). Writes, in the layouts
 * mosaic_bsa_fwd takes: q [B, S, Hq, 64] and k, v [B, S, Hk, 64] bf16, with Mosaic's 2D
 * RoPE (RoPE.forward, primitives.py:132-135) applied to q and k when rope_cos/rope_sin
 * ([S, 32] fp32) are given; gates [3, B, S, Hq] bf16 = softmax over the three strategies
 * of the bf16 gate logits (generate_strategy_weights, primitives.py:172-178).
 * head_dim 64, dim a multiple of 64, Hq <= 21 with gates. */
MOSAIC_API int mosaic_attn_qkv_proj(const void* x, const void* w_qkvg, const float* rope_cos, const float* rope_sin,
                                    void* q, void* k, void* v, void* gates, int* status, int seq_len, int batch,
                                    int dim, int num_q_heads, int num_kv_heads, int head_dim, void* stream);

/* Output projection of primitives.MosaicAttention.forward (primitives.py:207-208):
 * out [S, B, dim] = rearrange(attn, 'b s h d -> s b (h d)') to_o.weight^T, attn
 * [B, S, Hq, 64] bf16 (mosaic_bsa_fwd's output), w_o [dim, Hq*64] bf16. */
MOSAIC_API int mosaic_attn_out_proj(const void* attn, const void* w_o, void* out, int* status, int seq_len,
                                    int batch, int dim, int num_q_heads, int head_dim, void* stream);

/* mosaic_attn_out_proj followed by the residual add of MosaicBlock.forward
 * (primitives.py:228, `x = x + self.attention(...)`): out [S, B, dim] = T(residual +
 * T(to_o(attn))) with T = dtype, the type of residual and out (bf16, or fp16: the
 * block's residual stream under fp16 autocast, whose Linear outputs are fp16); attn and
 * w_o bf16; out may be residual (in place). dim a multiple of 32. */
MOSAIC_API int mosaic_attn_out_proj_residual(const void* attn, const void* w_o, const void* residual, void* out,
                                             int* status, int seq_len, int batch, int dim, int num_q_heads,
                                             int head_dim, int dtype, void* stream);

/* torch.nn.RMSNorm of 16-bit rows (the norm1 / norm2 of MosaicBlock, primitives.py:225-226,
 * with elementwise_affine weight or NULL): y = bf16(x * rsqrt(mean(x^2) + eps) * weight),
 * fp32 arithmetic, the sum of squares in a fixed order. x [rows, dim] of type dtype (bf16,
 * or fp16 for a residual stream under fp16 autocast), y [rows, dim] bf16 (y may be x when
 * x is bf16), weight [dim] fp32 or NULL. dim a multiple of 8. */
MOSAIC_API int mosaic_rms_norm(const void* x, const float* weight, void* y, int rows, int dim, float eps, int dtype,
                               void* stream);

/* out [rows, out_features] = row_scale[r] * (a [rows, in_features] w^T) in bf16 (fp32
 * accumulation), row_scale optional (NULL = 1): a Linear layer without bias on the
 * tensor core. Serves CrossAttentionInterpolate's to_kv (primitives.py:275, with the
 * row factor of its RMSNorm, primitives.py:273, as row_scale) and to_o (:283).
 * in_features a multiple of 64, out_features a multiple of 32. */
MOSAIC_API int mosaic_linear(const void* a, const void* w, void* out, const float* row_scale, int* status, int rows,
                             int in_features, int out_features, void* stream);

/* out = T(residual + T(row_scale[r] * (a w^T))) with T = dtype, the type of residual and
 * out (bf16, or fp16 for a residual stream under fp16 autocast): a Linear layer followed
 * by a residual add, as `x = x + self.ffn(...)` in MosaicBlock.forward (primitives.py:229)
 * with cSwiGLU's w2 (primitives.py:106) as the Linear. a and w bf16. out may be residual
 * itself (in place). Shapes and limits as mosaic_linear. */
MOSAIC_API int mosaic_linear_residual(const void* a, const void* w, const void* residual, void* out,
                                      const float* row_scale, int* status, int rows, int in_features,
                                      int out_features, int dtype, void* stream);

/* First half of the conditional SwiGLU FFN of a Mosaic block (cSwiGLU.forward,
 * primitives.py:102-106, with MosaicBlock's norm2, primitives.py:227, as row_scale):
 * for x [rows, dim] bf16 with rows (s, b) of a sequence-first [S, batch, dim] tensor,
 *   x1 = bf16(row_scale[r] * x w1^T), x3 = bf16(row_scale[r] * x w3^T)   (w13.chunk(2))
 *   h [rows, hidden] = bf16(bf16(silu(bf16(x1 + noise[r % batch]))) * x3)
 * with noise [batch, hidden] bf16 (noise_bias(z), NULL = none). w13 [2 hidden, dim]
 * bf16 holds the rows of cSwiGLU.w13.weight interleaved in blocks of 128: rows
 * [256 i, 256 i + 128) = w1 rows [128 i, 128 i + 128) and rows [256 i + 128, 256 i + 256)
 * = the w3 rows of the same hidden units (w3 row j = w13 row hidden + j). dim a
 * multiple of 64, hidden a multiple of 128, rows a multiple of batch. */
MOSAIC_API int mosaic_ffn_swiglu(const void* x, const void* w13, const float* row_scale, const void* noise, void* h,
                                 int* status, int rows, int dim, int hidden, int batch, void* stream);

/* rinv[r] = 1 / sqrt(mean_d x[r, d]^2 + eps) for x [rows, dim] bf16: the row factor of
 * torch.nn.RMSNorm without an affine weight (the kv_norm of CrossAttentionInterpolate,
 * primitives.py:247,273; rmsnorm_elementwise_affine=False in every preset). */
MOSAIC_API int mosaic_row_rms(const void* x, float* rinv, int rows, int dim, float eps, void* stream);

/* The gather-attention of CrossAttentionInterpolate.forward (primitives.py:268-281):
 * for target point s, batch b, head h: q_j = w_q[h rows] . rel_pos[s, j] (w_q = to_q.weight
 * [dim, 3] fp32, rel_pos [points_to, k, 3] fp32), scores scale * q_j . k[neighbors[s, j], b, h],
 * softmax over the k neighbours (fp32), out[s, b, h] = sum_j a_j v[neighbors[s, j], b, h].
 * kv [points_from, B, 2 dim] bf16 is to_kv's output ('s b (n h d)'), neighbors int32
 * [points_to, k], out [points_to, B, dim] bf16 (before to_o). head_dim 64, dim a multiple
 * of 256. Out-of-range neighbour indices set MOSAIC_STATUS_BAD_INDEX and read point 0. */
MOSAIC_API int mosaic_interp_attend(const void* kv, const int* neighbors, const float* rel_pos, const float* w_q,
                                    void* out, int* status, int points_to, int points_from, int batch, int dim,
                                    int num_heads, int num_neighbors, float scale, void* stream);

/* mosaic_interp_attend over tiles of spatially adjacent targets whose neighbour lists
 * were merged beforehand (the neighbour table is static). Tile t covers the at most 32
 * targets order[tile_targets[t] .. tile_targets[t+1]) (order may be null: the identity)
 * and the source points tile_points[tile_point_off[t] .. tile_point_off[t+1]): the union
 * of their neighbours, padded with repeats to a multiple of 16, at most max_union <= 256
 * (a multiple of 16). local_idx [points_to, k] (uint8) is each neighbour's position in its
 * tile's list; a target's neighbours are distinct points; num_neighbors <= 32, dim a
 * multiple of 128. kw_workspace holds points_from * batch * num_heads * 4 floats: the
 * per-point, per-head vectors (to_q.weight_h^T k_h, 0), computed here first unless
 * kw_ready is nonzero (the caller wrote them; w_q may then be NULL). Each tile copies its points' v rows once into shared memory and runs the
 * attention as P (softmax weights, bf16) x V on the tensor cores, so the outputs equal
 * mosaic_interp_attend's up to the bf16 rounding of the weights (as the reference
 * module's bf16 softmax) and fp32 summation order. Inconsistent tables set
 * MOSAIC_STATUS_BAD_INDEX. */
MOSAIC_API int mosaic_interp_attend_tiled(const void* kv, float* kw_workspace, const int* tile_targets,
                                          const int* tile_point_off, const int* tile_points,
                                          const uint8_t* local_idx, const int* order, const float* rel_pos,
                                          const float* w_q, void* out, int* status, int num_tiles, int max_union,
                                          int points_from, int batch, int dim, int num_heads, int num_neighbors,
                                          int kw_ready, float scale, void* stream);

/* HEALPixDownsample.forward (primitives.py:325-329) for x [(n f), batch, in_dim] bf16
 * (f = factor nested children per coarse pixel n): out [n, batch, out_dim] bf16 =
 * RMSNorm(rearrange(x, '(n f) b c -> n b (f c)') w_x^T + pos_bias[n]) with w_x
 * [out_dim, factor * in_dim] bf16 (proj_x.weight), pos_bias [n, out_dim] bf16 (the
 * static proj_pos(rel_pos)), norm_weight [out_dim] fp32 or NULL (no affine), eps the
 * RMSNorm epsilon. The projection output and the bias sum are rounded to bf16 as the
 * reference's bf16 layers do; the norm is fp32 over the stored bf16 row (a
 * deterministic sum). in_dim a multiple of 64, out_dim a multiple of 128. */
MOSAIC_API int mosaic_healpix_downsample(const void* x, const void* w_x, const void* pos_bias,
                                         const float* norm_weight, void* out, int* status, int n_coarse, int factor,
                                         int batch, int in_dim, int out_dim, float eps, void* stream);

/* HEALPixUpsample.forward (primitives.py:352-357) for x [n, batch, in_dim] bf16: out
 * [(n f), batch, out_dim] bf16 = RMSNorm(rearrange(x w_x^T + pos_bias[n],
 * 'n b (f d) -> (n f) b d') + shortcut) with w_x [factor * out_dim, in_dim] bf16,
 * pos_bias [n, factor * out_dim] bf16, shortcut [(n f), batch, out_dim] bf16 or NULL
 * (out may be the shortcut's buffer), norm_weight and eps as for the downsample. */
MOSAIC_API int mosaic_healpix_upsample(const void* x, const void* shortcut, const void* w_x, const void* pos_bias,
                                       const float* norm_weight, void* out, int* status, int n_coarse, int factor,
                                       int batch, int in_dim, int out_dim, float eps, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOSAIC_B200_H_ */
