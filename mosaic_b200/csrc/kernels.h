// Internal (C++) launch interface shared by the .cu files of libmosaic_b200.
// The public C ABI lives in include/mosaic_b200.h; nothing here crosses it.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace mosaic {

constexpr int kHeadDim = 64;

// How the attention engine combines its branches in the epilogue, per output row
// with gates (w0, w1, w2) = weight_ba_cmp_slc[:, b, n, head]:
enum Combine : int {
  kCombineGated = 0,  // w0*o_ba + w1*o_cmp + w2*o_slc              primitives.py:89
  kCombineNoCmp = 1,  // (w0*o_ba + w2*o_slc) / (w0 + w2 + 1e-8)     primitives.py:71-74
  kCombineNoSlc = 2,  // (w0*o_ba + w1*o_cmp) / (w0 + w1 + 1e-8)     primitives.py:81-84
  kCombineLocal = 3,  // o_ba                                         primitives.py:28-32, 62-63
  kCombineSel = 4,    // o_slc                                        ops.py:25-134
};

// One launch of the fused attention engine: for every (batch b, kv head h,
// 64-query tile) it runs the local-window branch and/or the selected-block branch
// for the G = 4 query heads of kv group h and writes the combined rows. Every
// 16-bit tensor below has the launch's activation type (bf16, or fp16 when f16).
struct EngineLaunch {
  const void* q;  // [B, Nq, Hq, 64]
  const void* k;  // [B, Nk, Hk, 64]
  const void* v;  // [B, Nk, Hk, 64]
  const int64_t* block_idx;  // [B, Nq/bs, Hk, K] or null when K == 0
  const void* gates;         // [3, B, Nq, Hq] or null
  const void* o_cmp;         // [B, Nq/bs, Hq, 64] or null
  void* out;                 // [B, Nq, Hq, 64]
  float* lse;                // [B, Nq, Hq] fp32 (selected branch, log2 units) or null
  int* status;               // device status word or null
  int B, Nq, Nk, Hq, Hk;
  int win;  // local window length; 0 = no local branch
  int bs;   // selected block length (multiple of 64)
  int K;    // selected blocks per query block; 0 = no selected branch
  int combine;
  float softmax_scale;
  bool f16;  // activations are fp16 (else bf16)
  bool after_topk;  // launched with programmatic serialization after the top-k kernel
};

// Mean-pool (optionally after 2D RoPE) of q, k, v over contiguous blocks of `bs` rows.
struct PoolLaunch {
  const void* q;  // [B, N, Hq, 64]
  const void* k;  // [B, N, Hk, 64]
  const void* v;  // [B, N, Hk, 64]
  const float* rope_cos;  // [N, 32] fp32 or null (no rotation)
  const float* rope_sin;  // [N, 32] fp32 or null
  void* q_rot;            // [B, N, Hq, 64] rotated copy (only when rope_cos != null)
  void* k_rot;            // [B, N, Hk, 64] rotated copy (only when rope_cos != null)
  void* q_cmp;            // [B, N/bs, Hq, 64] (may be null: skip q)
  void* k_cmp;            // [B, N/bs, Hk, 64]
  void* v_cmp;            // [B, N/bs, Hk, 64] (may be null: skip v)
  int B, N, Hq, Hk, bs;
  bool f16;  // every 16-bit tensor above is fp16 instead of bf16 (means rounded to fp16)
};

// Block scores + top-k selection (GQA group shared, strided head mean).
struct TopkLaunch {
  const void* q_cmp;  // [B, nb, Hq, 64]
  const void* k_cmp;  // [B, nb, Hk, 64]
  int64_t* idx;       // [B, nb, Hk, K]
  int B, nb, Hq, Hk, K;
  int* status;  // device status word or null (timeouts of the tensor-core variant)
  bool f16;     // q_cmp / k_cmp are fp16 and scores are rounded to fp16 (else bf16)
  // Launch with programmatic stream serialization, so that the kernel may start
  // while the previous kernel of the stream (which must not produce this
  // kernel's inputs) is still running.
  bool overlap_previous;
};

// Backward of the selected-block attention (bsa_bwd.cu).
struct SparseBwdLaunch {
  const void* q;         // [B, N, Hq, 64] bf16
  const void* k;         // [B, N, Hk, 64] bf16
  const void* v;         // [B, N, Hk, 64] bf16
  const void* out;       // [B, N, Hq, 64] bf16 forward output
  const void* grad_out;  // [B, N, Hq, 64] bf16
  const float* lse;      // [B, N, Hq] fp32, log2 units (forward)
  const int64_t* block_idx;  // [B, N/bs, Hk, K]
  void* grad_q;          // [B, N, Hq, 64] bf16
  void* grad_k;          // [B, N, Hk, 64] bf16
  void* grad_v;          // [B, N, Hk, 64] bf16
  void* workspace;       // sparse_bwd_workspace(...).total bytes, 256-aligned
  int* status;
  int B, N, Hq, Hk, bs, K;
  float softmax_scale;
};

// Byte offsets of the backward's scratch arrays inside its workspace.
struct SparseBwdWorkspace {
  size_t delta, count, cursor, offs, list, sorted, ucount, total;
};

SparseBwdWorkspace sparse_bwd_workspace(int B, int N, int Hq, int Hk, int bs, int K);
int sparse_bwd_max_selected();
int launch_sparse_bwd(const SparseBwdLaunch& a, cudaStream_t stream);

// Projections around the attention op (proj.cu).
struct QkvProjLaunch {
  const void* x;          // [S, B, dim] bf16
  const void* w;          // [(Hq + 2 Hk) 64 (+ 3 Hq), dim] bf16 = cat(to_q, to_k, to_v[, gate]) weights
  const float* rope_cos;  // [S, 32] fp32 or null
  const float* rope_sin;
  void* q;                // [B, S, Hq, 64] bf16
  void* k;                // [B, S, Hk, 64] bf16
  void* v;                // [B, S, Hk, 64] bf16
  void* gates;            // [3, B, S, Hq] bf16 or null (then w has no gate rows)
  int* status;
  int S, B, dim, Hq, Hk;
};
struct OutProjLaunch {
  const void* attn;      // [B, S, Hq*64] bf16
  const void* w;         // [dim, Hq*64] bf16 (to_o.weight)
  void* out;             // [S, B, dim] bf16
  const void* residual;  // [S, B, dim] added to the rounded output (may alias out) or null
  int out_f16;           // with a residual: residual and output fp16 (else bf16)
  int* status;
  int S, B, dim, Hq;
};
struct LinearLaunch {
  const void* a;         // [M, K] bf16
  const void* w;         // [N, K] bf16
  void* out;             // [M, N] bf16
  const float* rscale;   // [M] fp32 row factors or null
  const void* residual;  // [M, N] added to the rounded output (may alias out) or null
  int out_f16;           // with a residual: residual and output fp16 (else bf16)
  int* status;
  int M, K, N;
};
// First half of the conditional SwiGLU FFN (proj.cu, mode kSwiGLU):
// h = bf16(bf16(silu(bf16(x1 + noise[b]))) * x3) with x1, x3 = bf16(rscale * (x w1^T)),
// bf16(rscale * (x w3^T)).
struct SwigluLaunch {
  const void* x;         // [M, dim] bf16: rows (s, b) of x [S, B, dim]
  const void* w13;       // [2 hidden, dim] bf16, rows interleaved in blocks of 128: w1 rows
                         // [128 i, 128 i + 128) then the w3 rows of the same hidden units
  const float* rscale;   // [M] fp32 row factors (the RMSNorm in front) or null
  const void* noise;     // [B, hidden] bf16 (the block's noise_bias(z)) or null
  void* h;               // [M, hidden] bf16
  int* status;
  int M, dim, hidden, B;
};
// Cross-attention interpolation (interp.cu).
struct InterpLaunch {
  const void* kv;        // [S_from, B, 2 dim] bf16 (to_kv output, 's b (n h d)')
  const int* neighbors;  // [S_to, k] int32 indices into the S_from points
  const float* rel_pos;  // [S_to, k, 3] fp32 unit vectors
  const float* w_q;      // [dim, 3] fp32 (to_q.weight)
  void* out;             // [S_to, B, dim] bf16
  int* status;
  int S_to, S_from, B, dim, k;
  float scale;
};
struct InterpTiledLaunch {
  const void* kv;            // [S_from, B, 2 dim] bf16
  float* kw;                 // [S_from, B, H, 4] fp32 scratch, written here
  const int* tile_targets;   // [n_tiles + 1] offsets into `order`; <= 32 targets per tile
  const int* tile_point_off; // [n_tiles + 1] offsets into tile_points; multiples of 16
  const int* tile_points;    // source points of each tile's neighbour union (padded to 16)
  const uint8_t* local_idx;  // [S_to, k] position of neighbour j inside its tile's union
  const int* order;          // [S_to] targets in tile order, or null = identity
  const float* rel_pos;      // [S_to, k, 3]
  const float* w_q;          // [dim, 3]
  void* out;                 // [S_to, B, dim] bf16
  int* status;
  int S_from, B, dim, k, n_tiles, max_union;
  float scale;
  bool kw_ready;             // kw already holds the vectors (the caller computed them)
};
// HEALPix down/upsampling (proj.cu): GEMM + position bias (+ shortcut) + RMSNorm.
struct UpDownLaunch {
  const void* x;         // down: [(n f), B, c_in]; up: [n, B, c_in] bf16
  const void* shortcut;  // up: [(n f), B, c_out] bf16 or null
  const void* w;         // down: [c_out, F c_in]; up: [F c_out, c_in] bf16 (proj_x.weight)
  const void* pos;       // down: [n, c_out]; up: [n, F c_out] bf16 (proj_pos(rel_pos))
  const float* norm_w;   // [c_out] fp32 or null
  void* out;             // down: [n, B, c_out]; up: [(n f), B, c_out] bf16
  int* status;
  int n, F, B, c_in, c_out;
  float eps;
};
int launch_healpix_down(const UpDownLaunch& a, cudaStream_t stream);
int launch_healpix_up(const UpDownLaunch& a, cudaStream_t stream);
int launch_qkv_proj(const QkvProjLaunch& a, cudaStream_t stream);
int launch_interp_tiled(const InterpTiledLaunch& a, cudaStream_t stream);
size_t tiled_interp_smem_bytes(int max_union, int H, int k);
int launch_linear(const LinearLaunch& a, cudaStream_t stream);
int launch_swiglu(const SwigluLaunch& a, cudaStream_t stream);
int launch_interp_attend(const InterpLaunch& a, cudaStream_t stream);
int launch_row_rms(const void* x, float* rinv, long long rows, int dim, float eps, cudaStream_t stream);
int launch_out_proj(const OutProjLaunch& a, cudaStream_t stream);
// y = bf16(x * rsqrt(mean(x^2) + eps) (* w)) per row of x [rows, D], x bf16 (y may be x)
// or fp16 (x_f16).
int launch_rms_norm(const void* x, void* y, const float* w, long long rows, int D, float eps, bool x_f16,
                    cudaStream_t stream);

int launch_engine(const EngineLaunch& a, cudaStream_t stream);
int launch_pool(const PoolLaunch& a, cudaStream_t stream);
int launch_topk(const TopkLaunch& a, cudaStream_t stream);
// The tensor-core top-k (topk_tc.cu) for G <= 4 and K <= 32; launch_topk picks it.
bool topk_tc_supported(const TopkLaunch& a);
int launch_topk_tc(const TopkLaunch& a, cudaStream_t stream);

// Encodes a 2D tensor map of 16-bit elements (bf16, or fp16 when f16) over
// `rows` x `cols` elements (row pitch = cols), 64x64 boxes, 128-byte swizzle.
// Returns 0 on success.
int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, bool f16);
inline int make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols) {
  return make_tmap_2d(map, base, rows, cols, false);
}
// 3D bf16 tensor map (d0 innermost, contiguous), strides of dims 1 and 2 in bytes,
// 64 x 1 x 64 boxes, 128-byte swizzle: a box lands in shared memory like a 64 x 64 2D box.
int make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                      uint64_t stride1_bytes, uint64_t stride2_bytes);

}  // namespace mosaic
