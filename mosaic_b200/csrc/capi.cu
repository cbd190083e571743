// extern "C" entry points of libmosaic_b200.so (declared in include/mosaic_b200.h).
//
// Each entry point validates its arguments on the host before touching CUDA, so
// a bad call returns an error code and launches nothing. Validation mirrors what
// the reference path requires implicitly (einops rearranges that need N % bs == 0,
// topk's K <= nb) plus the limits of these kernels (head_dim 64, G = 4).
#include <cstring>

#include <cudaTypedefs.h>

#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {

int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, bool f16) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return 1;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, 64};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                            const_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 1;
}

int make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                      uint64_t stride1_bytes, uint64_t stride2_bytes) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return 1;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {64, 1, 64};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 1;
}

namespace {

// Self-test of the bounded-wait machinery every pipeline kernel uses: one warp
// waits, with a short limit, on an mbarrier that nothing ever arrives on. The
// wait must give up, raise the CTA abort flag and record MOSAIC_STATUS_TIMEOUT;
// the kernel then returns normally (no trap, no hang).
__global__ void selftest_wait_kernel(int* status, uint64_t timeout_ns, int* result) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = bounded_wait(&bar, 0, &abort_flag, status, timeout_ns);
    result[0] = ok ? 1 : 0;
    result[1] = abort_flag;
  }
}

constexpr int kMaxTopK = 128;    // topk.cu kMaxK
constexpr int kMaxSelect = 1024;  // bsa_engine.cu kMaxSel

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool valid_dtype(int dtype) { return dtype == MOSAIC_DTYPE_BF16 || dtype == MOSAIC_DTYPE_F16; }
inline size_t round256(size_t x) { return (x + 255) & ~size_t(255); }
inline float default_scale(float s) { return s > 0.f ? s : 0.125f; }  // 64 ** -0.5

// Shape checks shared by every attention entry point.
int check_heads(int B, int N, int Hq, int Hk, int D) {
  if (B < 0 || N < 0 || Hq <= 0 || Hk <= 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (D != kHeadDim) return MOSAIC_ERR_UNSUPPORTED;
  if (Hq % Hk != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  return MOSAIC_OK;
}

// The top-k kernels are instantiated for 1 to 8 query heads per kv head (every
// preset has 4); the attention kernels take any ratio.
bool topk_group_supported(int Hq, int Hk) {
  const int G = Hq / Hk;
  return G >= 1 && G <= 8;
}

struct Workspace {
  size_t q_cmp, k_cmp, v_cmp, o_cmp, idx, q_rot, k_rot, total;
};

Workspace workspace_layout(int B, int N, int Hq, int Hk, int bs, int K, bool rope) {
  Workspace w;
  const size_t nb = bs > 0 ? static_cast<size_t>(N) / bs : 0;
  size_t off = 0;
  w.q_cmp = off; off += round256(static_cast<size_t>(B) * nb * Hq * 128);
  w.k_cmp = off; off += round256(static_cast<size_t>(B) * nb * Hk * 128);
  w.v_cmp = off; off += round256(static_cast<size_t>(B) * nb * Hk * 128);
  w.o_cmp = off; off += round256(static_cast<size_t>(B) * nb * Hq * 128);
  w.idx = off; off += round256(static_cast<size_t>(B) * nb * Hk * (K > 0 ? K : 0) * 8);
  w.q_rot = off; off += rope ? round256(static_cast<size_t>(B) * N * Hq * 128) : 0;
  w.k_rot = off; off += rope ? round256(static_cast<size_t>(B) * N * Hk * 128) : 0;
  w.total = off;
  return w;
}

}  // namespace
}  // namespace mosaic

using namespace mosaic;

extern "C" {

int mosaic_abi_version(void) { return 2; }

int mosaic_selftest_wait_timeout(int* status, int* result, int timeout_us, void* stream) {
  if (status == nullptr || result == nullptr || timeout_us <= 0 || timeout_us > 10000000)
    return MOSAIC_ERR_INVALID_ARGUMENT;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      status, static_cast<uint64_t>(timeout_us) * 1000ull, result);
  return cudaGetLastError() == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

const char* mosaic_error_string(int code) {
  switch (code) {
    case MOSAIC_OK: return "ok";
    case MOSAIC_ERR_INVALID_ARGUMENT: return "invalid argument (null/misaligned pointer, negative or inconsistent size)";
    case MOSAIC_ERR_UNSUPPORTED: return "unsupported shape (needs head_dim 64, block sizes multiple of 64; top-k: 1 to 8 query heads per kv head)";
    case MOSAIC_ERR_WORKSPACE: return "workspace missing or smaller than mosaic_bsa_workspace_bytes()";
    case MOSAIC_ERR_CUDA: return "CUDA call failed (kernel launch or tensor-map encoding)";
    default: return "unknown mosaic_b200 error code";
  }
}

size_t mosaic_bsa_workspace_bytes(int batch, int seq_len, int num_q_heads, int num_kv_heads, int head_dim,
                                  int sparse_block_size, int sparse_block_count, int with_rope) {
  (void)head_dim;
  if (batch < 0 || seq_len < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || sparse_block_size <= 0) return 0;
  return workspace_layout(batch, seq_len, num_q_heads, num_kv_heads, sparse_block_size, sparse_block_count,
                          with_rope != 0)
      .total;
}

int mosaic_sparse_attn_fwd(const void* q, const void* k, const void* v, const int64_t* block_indices, void* out,
                           float* lse, int* status, int batch, int seq_len, int num_q_heads, int num_kv_heads,
                           int head_dim, int block_size, int block_count, float softmax_scale, int dtype,
                           void* stream) {
  int rc = check_heads(batch, seq_len, num_q_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (!valid_dtype(dtype)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seq_len == 0) return MOSAIC_OK;
  if (!q || !k || !v || !out || !block_indices) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (block_size <= 0 || block_count <= 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (block_size % 64 != 0) return MOSAIC_ERR_UNSUPPORTED;
  if (seq_len % block_size != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (block_count > kMaxSelect) return MOSAIC_ERR_UNSUPPORTED;
  if (batch == 0 || seq_len == 0) return MOSAIC_OK;
  EngineLaunch a;
  std::memset(&a, 0, sizeof(a));
  a.q = q; a.k = k; a.v = v;
  a.block_idx = block_indices;
  a.out = out; a.lse = lse; a.status = status;
  a.B = batch; a.Nq = seq_len; a.Nk = seq_len; a.Hq = num_q_heads; a.Hk = num_kv_heads;
  a.win = 0; a.bs = block_size; a.K = block_count;
  a.combine = kCombineSel;
  a.softmax_scale = default_scale(softmax_scale);
  a.f16 = dtype == MOSAIC_DTYPE_F16;
  return launch_engine(a, static_cast<cudaStream_t>(stream));
}

int mosaic_bsa_attend_fwd(const void* q, const void* k, const void* v, const int64_t* block_indices,
                          const void* gates, const void* o_cmp, void* out, int* status, int batch, int seq_len,
                          int num_q_heads, int num_kv_heads, int head_dim, int block_attn_size,
                          int sparse_block_size, int sparse_block_count, int combine, float softmax_scale,
                          int dtype, void* stream) {
  int rc = check_heads(batch, seq_len, num_q_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (!valid_dtype(dtype)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seq_len == 0) return MOSAIC_OK;
  if (combine < kCombineGated || combine > kCombineNoSlc) return MOSAIC_ERR_INVALID_ARGUMENT;
  const bool want_slc = combine != kCombineNoSlc;
  const bool want_cmp = combine != kCombineNoCmp;
  if (!q || !k || !v || !out || !gates) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (want_slc && !block_indices) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (want_cmp && !o_cmp) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || (o_cmp && !aligned16(o_cmp)))
    return MOSAIC_ERR_INVALID_ARGUMENT;
  if (block_attn_size <= 0 || seq_len % block_attn_size != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (block_attn_size % 64 != 0 && block_attn_size != seq_len) return MOSAIC_ERR_UNSUPPORTED;
  if (sparse_block_size <= 0 || seq_len % sparse_block_size != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (sparse_block_size % 64 != 0) return MOSAIC_ERR_UNSUPPORTED;
  if (want_slc && (sparse_block_count <= 0 || sparse_block_count > seq_len / sparse_block_size))
    return MOSAIC_ERR_INVALID_ARGUMENT;
  if (sparse_block_count > kMaxSelect) return MOSAIC_ERR_UNSUPPORTED;
  EngineLaunch a;
  std::memset(&a, 0, sizeof(a));
  a.q = q; a.k = k; a.v = v;
  a.block_idx = want_slc ? block_indices : nullptr;
  a.gates = gates;
  a.o_cmp = want_cmp ? o_cmp : nullptr;
  a.out = out; a.status = status;
  a.B = batch; a.Nq = seq_len; a.Nk = seq_len; a.Hq = num_q_heads; a.Hk = num_kv_heads;
  a.win = block_attn_size; a.bs = sparse_block_size; a.K = want_slc ? sparse_block_count : 0;
  a.combine = combine;
  a.softmax_scale = default_scale(softmax_scale);
  a.f16 = dtype == MOSAIC_DTYPE_F16;
  return launch_engine(a, static_cast<cudaStream_t>(stream));
}

int mosaic_block_attn_fwd(const void* q, const void* k, const void* v, void* out, int* status, int batch,
                          int seq_len, int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                          float softmax_scale, int dtype, void* stream) {
  int rc = check_heads(batch, seq_len, num_q_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (!valid_dtype(dtype)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seq_len == 0) return MOSAIC_OK;
  if (!q || !k || !v || !out) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (block_size <= 0 || seq_len % block_size != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (block_size % 64 != 0 && block_size != seq_len) return MOSAIC_ERR_UNSUPPORTED;
  if (batch == 0 || seq_len == 0) return MOSAIC_OK;
  EngineLaunch a;
  std::memset(&a, 0, sizeof(a));
  a.q = q; a.k = k; a.v = v; a.out = out; a.status = status;
  a.B = batch; a.Nq = seq_len; a.Nk = seq_len; a.Hq = num_q_heads; a.Hk = num_kv_heads;
  a.win = block_size; a.bs = 64; a.K = 0;
  a.combine = kCombineLocal;
  a.softmax_scale = default_scale(softmax_scale);
  a.f16 = dtype == MOSAIC_DTYPE_F16;
  return launch_engine(a, static_cast<cudaStream_t>(stream));
}

int mosaic_cmp_attn_fwd(const void* q_cmp, const void* k_cmp, const void* v_cmp, void* o_cmp, int* status,
                        int batch, int num_blocks, int num_q_heads, int num_kv_heads, int head_dim,
                        float softmax_scale, int dtype, void* stream) {
  int rc = check_heads(batch, num_blocks, num_q_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (!valid_dtype(dtype)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (batch == 0 || num_blocks == 0) return MOSAIC_OK;
  if (!q_cmp || !k_cmp || !v_cmp || !o_cmp) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(q_cmp) || !aligned16(k_cmp) || !aligned16(v_cmp) || !aligned16(o_cmp))
    return MOSAIC_ERR_INVALID_ARGUMENT;
  if (batch == 0 || num_blocks == 0) return MOSAIC_OK;
  EngineLaunch a;
  std::memset(&a, 0, sizeof(a));
  a.q = q_cmp; a.k = k_cmp; a.v = v_cmp; a.out = o_cmp; a.status = status;
  a.B = batch; a.Nq = num_blocks; a.Nk = num_blocks; a.Hq = num_q_heads; a.Hk = num_kv_heads;
  a.win = num_blocks; a.bs = 64; a.K = 0;
  a.combine = kCombineLocal;
  a.softmax_scale = default_scale(softmax_scale);
  a.f16 = dtype == MOSAIC_DTYPE_F16;
  return launch_engine(a, static_cast<cudaStream_t>(stream));
}

int mosaic_block_pool(const void* q, const void* k, const void* v, const float* rope_cos, const float* rope_sin,
                      void* q_rot, void* k_rot, void* q_cmp, void* k_cmp, void* v_cmp, int batch, int seq_len,
                      int num_q_heads, int num_kv_heads, int head_dim, int block_size, int dtype,
                      void* stream) {
  if (batch < 0 || seq_len < 0 || num_q_heads <= 0 || num_kv_heads <= 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(dtype)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (head_dim != kHeadDim) return MOSAIC_ERR_UNSUPPORTED;
  if (block_size <= 0 || seq_len % block_size != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!k || !k_cmp || (q_cmp && !q) || (v_cmp && !v)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (rope_cos && (!q || !q_cmp || !q_rot || !k_rot)) return MOSAIC_ERR_INVALID_ARGUMENT;
  const void* ptrs[] = {q, k, v, q_rot, k_rot, q_cmp, k_cmp, v_cmp, rope_cos, rope_sin};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seq_len == 0) return MOSAIC_OK;
  PoolLaunch a;
  a.q = q; a.k = k; a.v = v;
  a.rope_cos = rope_cos; a.rope_sin = rope_sin;
  a.q_rot = q_rot; a.k_rot = k_rot;
  a.q_cmp = q_cmp; a.k_cmp = k_cmp; a.v_cmp = v_cmp;
  a.B = batch; a.N = seq_len; a.Hq = num_q_heads; a.Hk = num_kv_heads; a.bs = block_size;
  a.f16 = dtype == MOSAIC_DTYPE_F16;
  return launch_pool(a, static_cast<cudaStream_t>(stream));
}

int mosaic_attn_topk(const void* q_cmp, const void* k_cmp, int64_t* block_indices, int batch, int num_blocks,
                     int num_q_heads, int num_kv_heads, int head_dim, int block_count, int dtype,
                     void* stream) {
  if (batch < 0 || num_blocks < 0 || num_q_heads <= 0 || num_kv_heads <= 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(dtype)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (head_dim != kHeadDim) return MOSAIC_ERR_UNSUPPORTED;
  if (num_q_heads % num_kv_heads != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!topk_group_supported(num_q_heads, num_kv_heads)) return MOSAIC_ERR_UNSUPPORTED;
  if (!q_cmp || !k_cmp || !block_indices) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(q_cmp) || !aligned16(k_cmp)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (block_count < 0 || block_count > num_blocks) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (block_count > kMaxTopK || num_blocks > 65535) return MOSAIC_ERR_UNSUPPORTED;
  if (batch == 0 || num_blocks == 0 || block_count == 0) return MOSAIC_OK;
  TopkLaunch a;
  a.q_cmp = q_cmp; a.k_cmp = k_cmp; a.idx = block_indices;
  a.B = batch; a.nb = num_blocks; a.Hq = num_q_heads; a.Hk = num_kv_heads; a.K = block_count;
  a.status = nullptr;
  a.f16 = dtype == MOSAIC_DTYPE_F16;
  a.overlap_previous = false;
  return launch_topk(a, static_cast<cudaStream_t>(stream));
}

int mosaic_bsa_fwd(const MosaicBsaArgs* args, void* stream) {
  if (args == nullptr) return MOSAIC_ERR_INVALID_ARGUMENT;
  const MosaicBsaArgs& A = *args;
  const int B = A.batch, N = A.seq_len, Hq = A.num_q_heads, Hk = A.num_kv_heads;
  const int bas = A.block_attn_size, bs = A.sparse_block_size, K = A.sparse_block_count;
  const bool local_only = A.block_attn_only != 0, no_cmp = A.no_compression != 0;
  const bool rope = A.rope_cos != nullptr;
  int rc = check_heads(B, N, Hq, Hk, A.head_dim);
  if (rc) return rc;
  if (!valid_dtype(A.dtype)) return MOSAIC_ERR_INVALID_ARGUMENT;
  const bool f16 = A.dtype == MOSAIC_DTYPE_F16;
  if (B == 0 || N == 0) return MOSAIC_OK;
  if (!A.q || !A.k || !A.v || !A.out) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!local_only && !A.gates) return MOSAIC_ERR_INVALID_ARGUMENT;
  if ((A.rope_cos == nullptr) != (A.rope_sin == nullptr)) return MOSAIC_ERR_INVALID_ARGUMENT;
  const void* ptrs[] = {A.q, A.k, A.v, A.out, A.rope_cos, A.rope_sin, A.workspace};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (bas <= 0 || N % bas != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (bas % 64 != 0 && bas != N) return MOSAIC_ERR_UNSUPPORTED;
  if (!local_only || rope) {
    if (bs <= 0 || N % bs != 0 || K < 0) return MOSAIC_ERR_INVALID_ARGUMENT;
    if (bs % 64 != 0) return MOSAIC_ERR_UNSUPPORTED;
  }
  const int nb = bs > 0 ? N / bs : 0;
  if (!local_only) {
    if (K > nb) return MOSAIC_ERR_INVALID_ARGUMENT;
    if (no_cmp && K == 0) return MOSAIC_ERR_INVALID_ARGUMENT;
    if (K > kMaxTopK || nb > 65535) return MOSAIC_ERR_UNSUPPORTED;
    if (!topk_group_supported(Hq, Hk)) return MOSAIC_ERR_UNSUPPORTED;
  }
  const Workspace ws = workspace_layout(B, N, Hq, Hk, bs > 0 ? bs : 64, local_only ? 0 : K, rope);
  const bool need_ws = !local_only || rope;
  if (need_ws && (A.workspace == nullptr || A.workspace_bytes < ws.total)) return MOSAIC_ERR_WORKSPACE;
  if (B == 0 || N == 0) return MOSAIC_OK;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* w = static_cast<uint8_t*>(A.workspace);
  const void* q = A.q;
  const void* k = A.k;
  void* q_cmp = w ? w + ws.q_cmp : nullptr;
  void* k_cmp = w ? w + ws.k_cmp : nullptr;
  void* v_cmp = w ? w + ws.v_cmp : nullptr;
  void* o_cmp = w ? w + ws.o_cmp : nullptr;
  int64_t* idx = A.block_indices ? A.block_indices : (w ? reinterpret_cast<int64_t*>(w + ws.idx) : nullptr);
  const float scale = default_scale(A.softmax_scale);
  const bool want_cmp = !local_only && !no_cmp;     // compressed branch
  const bool want_slc = !local_only && K > 0;       // selected branch

  // (a) RoPE + block mean-pool
  if (need_ws) {
    PoolLaunch pl;
    pl.q = A.q; pl.k = A.k; pl.v = A.v;
    pl.rope_cos = A.rope_cos; pl.rope_sin = A.rope_sin;
    pl.q_rot = rope ? w + ws.q_rot : nullptr;
    pl.k_rot = rope ? w + ws.k_rot : nullptr;
    pl.q_cmp = q_cmp; pl.k_cmp = k_cmp;
    pl.v_cmp = want_cmp ? v_cmp : nullptr;
    pl.B = B; pl.N = N; pl.Hq = Hq; pl.Hk = Hk; pl.bs = bs > 0 ? bs : 64;
    pl.f16 = f16;
    if ((rc = launch_pool(pl, st))) return rc;
    if (rope) {
      q = pl.q_rot;
      k = pl.k_rot;
    }
  }
  // (a) coarse attention over the pooled blocks
  if (want_cmp) {
    EngineLaunch e;
    std::memset(&e, 0, sizeof(e));
    e.q = q_cmp; e.k = k_cmp; e.v = v_cmp; e.out = o_cmp; e.status = A.status;
    e.B = B; e.Nq = nb; e.Nk = nb; e.Hq = Hq; e.Hk = Hk;
    e.win = nb; e.bs = 64; e.K = 0; e.combine = kCombineLocal; e.softmax_scale = scale; e.f16 = f16;
    if ((rc = launch_engine(e, st))) return rc;
  }
  // (b) block scores + top-k
  if (want_slc) {
    TopkLaunch t;
    t.q_cmp = q_cmp; t.k_cmp = k_cmp; t.idx = idx;
    t.B = B; t.nb = nb; t.Hq = Hq; t.Hk = Hk; t.K = K;
    t.status = A.status;
    t.f16 = f16;
    t.overlap_previous = want_cmp;  // runs beside the coarse attention (both only read the pooled tensors)
    if ((rc = launch_topk(t, st))) return rc;
  }
  // (c) fused local + selected attention with the gated combine
  EngineLaunch e;
  std::memset(&e, 0, sizeof(e));
  e.q = q; e.k = k; e.v = A.v;
  e.block_idx = want_slc ? idx : nullptr;
  e.gates = A.gates;
  e.o_cmp = want_cmp ? o_cmp : nullptr;
  e.out = A.out;
  e.status = A.status;
  e.B = B; e.Nq = N; e.Nk = N; e.Hq = Hq; e.Hk = Hk;
  e.win = bas;
  e.bs = bs > 0 ? bs : 64;
  e.K = want_slc ? K : 0;
  e.combine = local_only ? kCombineLocal : (no_cmp ? kCombineNoCmp : (want_slc ? kCombineGated : kCombineNoSlc));
  e.softmax_scale = scale;
  e.f16 = f16;
  e.after_topk = want_slc;
  return launch_engine(e, st);
}


size_t mosaic_sparse_attn_bwd_workspace_bytes(int batch, int seq_len, int num_q_heads, int num_kv_heads,
                                              int head_dim, int block_size, int block_count) {
  (void)head_dim;
  if (batch < 0 || seq_len < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || block_size <= 0 || block_count < 0)
    return 0;
  return sparse_bwd_workspace(batch, seq_len, num_q_heads, num_kv_heads, block_size, block_count).total;
}

int mosaic_sparse_attn_bwd(const void* q, const void* k, const void* v, const void* out, const void* grad_out,
                           const float* lse, const int64_t* block_indices, void* grad_q, void* grad_k, void* grad_v,
                           void* workspace, size_t workspace_bytes, int* status, int batch, int seq_len,
                           int num_q_heads, int num_kv_heads, int head_dim, int block_size, int block_count,
                           float softmax_scale, void* stream) {
  int rc = check_heads(batch, seq_len, num_q_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (block_size <= 0 || block_count <= 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (block_size % 64 != 0) return MOSAIC_ERR_UNSUPPORTED;
  if (seq_len % block_size != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (block_count > sparse_bwd_max_selected()) return MOSAIC_ERR_UNSUPPORTED;
  if (batch == 0 || seq_len == 0) return MOSAIC_OK;
  if (!q || !k || !v || !out || !grad_out || !lse || !block_indices || !grad_q || !grad_k || !grad_v)
    return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(grad_out) ||
      !aligned16(grad_q) || !aligned16(grad_k) || !aligned16(grad_v))
    return MOSAIC_ERR_INVALID_ARGUMENT;
  const size_t need =
      sparse_bwd_workspace(batch, seq_len, num_q_heads, num_kv_heads, block_size, block_count).total;
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return MOSAIC_ERR_WORKSPACE;
  SparseBwdLaunch a;
  std::memset(&a, 0, sizeof(a));
  a.q = q; a.k = k; a.v = v; a.out = out; a.grad_out = grad_out; a.lse = lse;
  a.block_idx = block_indices;
  a.grad_q = grad_q; a.grad_k = grad_k; a.grad_v = grad_v;
  a.workspace = workspace;
  a.status = status;
  a.B = batch; a.N = seq_len; a.Hq = num_q_heads; a.Hk = num_kv_heads; a.bs = block_size; a.K = block_count;
  a.softmax_scale = default_scale(softmax_scale);
  return launch_sparse_bwd(a, static_cast<cudaStream_t>(stream));
}

int mosaic_attn_qkv_proj(const void* x, const void* w_qkvg, const float* rope_cos, const float* rope_sin, void* q,
                         void* k, void* v, void* gates, int* status, int seq_len, int batch, int dim,
                         int num_q_heads, int num_kv_heads, int head_dim, void* stream) {
  if (seq_len < 0 || batch < 0 || dim <= 0 || num_q_heads <= 0 || num_kv_heads <= 0)
    return MOSAIC_ERR_INVALID_ARGUMENT;
  if (head_dim != kHeadDim) return MOSAIC_ERR_UNSUPPORTED;
  if (dim % 64 != 0) return MOSAIC_ERR_UNSUPPORTED;
  if (gates != nullptr && num_q_heads > 21) return MOSAIC_ERR_UNSUPPORTED;  // 3 Hq gate columns fit one 64-column group
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (seq_len == 0 || batch == 0) return MOSAIC_OK;
  if (!x || !w_qkvg || !q || !k || !v) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(w_qkvg) || !aligned16(q) || !aligned16(k) || !aligned16(v))
    return MOSAIC_ERR_INVALID_ARGUMENT;
  QkvProjLaunch a;
  std::memset(&a, 0, sizeof(a));
  a.x = x; a.w = w_qkvg; a.rope_cos = rope_cos; a.rope_sin = rope_sin;
  a.q = q; a.k = k; a.v = v; a.gates = gates; a.status = status;
  a.S = seq_len; a.B = batch; a.dim = dim; a.Hq = num_q_heads; a.Hk = num_kv_heads;
  return launch_qkv_proj(a, static_cast<cudaStream_t>(stream));
}

int mosaic_attn_out_proj(const void* attn, const void* w_o, void* out, int* status, int seq_len, int batch, int dim,
                         int num_q_heads, int head_dim, void* stream) {
  if (seq_len < 0 || batch < 0 || dim <= 0 || num_q_heads <= 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (head_dim != kHeadDim) return MOSAIC_ERR_UNSUPPORTED;
  if (dim % 8 != 0) return MOSAIC_ERR_UNSUPPORTED;  // 16-byte rows for the weight's tensor map and the stores
  if (seq_len == 0 || batch == 0) return MOSAIC_OK;
  if (!attn || !w_o || !out) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(attn) || !aligned16(w_o) || !aligned16(out)) return MOSAIC_ERR_INVALID_ARGUMENT;
  OutProjLaunch a;
  std::memset(&a, 0, sizeof(a));
  a.attn = attn; a.w = w_o; a.out = out; a.status = status;
  a.S = seq_len; a.B = batch; a.dim = dim; a.Hq = num_q_heads;
  return launch_out_proj(a, static_cast<cudaStream_t>(stream));
}

int mosaic_attn_out_proj_residual(const void* attn, const void* w_o, const void* residual, void* out, int* status,
                                  int seq_len, int batch, int dim, int num_q_heads, int head_dim, int dtype,
                                  void* stream) {
  if (seq_len < 0 || batch < 0 || dim <= 0 || num_q_heads <= 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(dtype)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (head_dim != kHeadDim) return MOSAIC_ERR_UNSUPPORTED;
  if (dim % 32 != 0) return MOSAIC_ERR_UNSUPPORTED;  // whole 32-column chunks of residual and output rows
  if (seq_len == 0 || batch == 0) return MOSAIC_OK;
  if (!attn || !w_o || !residual || !out) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(attn) || !aligned16(w_o) || !aligned16(residual) || !aligned16(out))
    return MOSAIC_ERR_INVALID_ARGUMENT;
  OutProjLaunch a;
  std::memset(&a, 0, sizeof(a));
  a.attn = attn; a.w = w_o; a.out = out; a.residual = residual; a.out_f16 = dtype == MOSAIC_DTYPE_F16;
  a.status = status;
  a.S = seq_len; a.B = batch; a.dim = dim; a.Hq = num_q_heads;
  return launch_out_proj(a, static_cast<cudaStream_t>(stream));
}

int mosaic_rms_norm(const void* x, const float* weight, void* y, int rows, int dim, float eps, int dtype,
                    void* stream) {
  if (rows < 0 || dim <= 0 || !(eps >= 0.f) || !valid_dtype(dtype)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (dtype == MOSAIC_DTYPE_F16 && x == y) return MOSAIC_ERR_INVALID_ARGUMENT;  // y is bf16: no in-place
  if (dim % 8 != 0) return MOSAIC_ERR_UNSUPPORTED;
  if (rows == 0) return MOSAIC_OK;
  if (!x || !y || !aligned16(x) || !aligned16(y) || (weight && !aligned16(weight))) return MOSAIC_ERR_INVALID_ARGUMENT;
  return launch_rms_norm(x, y, weight, rows, dim, eps, dtype == MOSAIC_DTYPE_F16, static_cast<cudaStream_t>(stream));
}

int mosaic_linear(const void* a, const void* w, void* out, const float* row_scale, int* status, int rows,
                  int in_features, int out_features, void* stream) {
  if (rows < 0 || in_features <= 0 || out_features <= 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  // the epilogue writes whole 32-column chunks of a row
  if (in_features % 64 != 0 || out_features % 32 != 0) return MOSAIC_ERR_UNSUPPORTED;
  if (rows == 0) return MOSAIC_OK;
  if (!a || !w || !out) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(a) || !aligned16(w) || !aligned16(out)) return MOSAIC_ERR_INVALID_ARGUMENT;
  LinearLaunch l;
  std::memset(&l, 0, sizeof(l));
  l.a = a; l.w = w; l.out = out; l.rscale = row_scale; l.status = status;
  l.M = rows; l.K = in_features; l.N = out_features;
  return launch_linear(l, static_cast<cudaStream_t>(stream));
}

int mosaic_linear_residual(const void* a, const void* w, const void* residual, void* out, const float* row_scale,
                           int* status, int rows, int in_features, int out_features, int dtype, void* stream) {
  if (rows < 0 || in_features <= 0 || out_features <= 0 || !valid_dtype(dtype)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (in_features % 64 != 0 || out_features % 32 != 0) return MOSAIC_ERR_UNSUPPORTED;
  if (rows == 0) return MOSAIC_OK;
  if (!a || !w || !residual || !out) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(a) || !aligned16(w) || !aligned16(residual) || !aligned16(out)) return MOSAIC_ERR_INVALID_ARGUMENT;
  LinearLaunch l;
  std::memset(&l, 0, sizeof(l));
  l.a = a; l.w = w; l.out = out; l.rscale = row_scale; l.residual = residual; l.out_f16 = dtype == MOSAIC_DTYPE_F16;
  l.status = status;
  l.M = rows; l.K = in_features; l.N = out_features;
  return launch_linear(l, static_cast<cudaStream_t>(stream));
}

int mosaic_ffn_swiglu(const void* x, const void* w13, const float* row_scale, const void* noise, void* h, int* status,
                      int rows, int dim, int hidden, int batch, void* stream) {
  if (rows < 0 || dim <= 0 || hidden <= 0 || batch <= 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (rows % batch != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (dim % 64 != 0 || hidden % 128 != 0) return MOSAIC_ERR_UNSUPPORTED;
  if (rows == 0) return MOSAIC_OK;
  if (!x || !w13 || !h) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(w13) || !aligned16(h) || (noise && !aligned16(noise)))
    return MOSAIC_ERR_INVALID_ARGUMENT;
  SwigluLaunch l;
  std::memset(&l, 0, sizeof(l));
  l.x = x; l.w13 = w13; l.rscale = row_scale; l.noise = noise; l.h = h; l.status = status;
  l.M = rows; l.dim = dim; l.hidden = hidden; l.B = batch;
  return launch_swiglu(l, static_cast<cudaStream_t>(stream));
}

int mosaic_row_rms(const void* x, float* rinv, int rows, int dim, float eps, void* stream) {
  if (rows < 0 || dim <= 0 || !(eps >= 0.f)) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (dim % 8 != 0) return MOSAIC_ERR_UNSUPPORTED;
  if (rows == 0) return MOSAIC_OK;
  if (!x || !rinv || !aligned16(x)) return MOSAIC_ERR_INVALID_ARGUMENT;
  return launch_row_rms(x, rinv, rows, dim, eps, static_cast<cudaStream_t>(stream));
}

int mosaic_interp_attend(const void* kv, const int* neighbors, const float* rel_pos, const float* w_q, void* out,
                         int* status, int points_to, int points_from, int batch, int dim, int num_heads,
                         int num_neighbors, float scale, void* stream) {
  if (points_to < 0 || points_from <= 0 || batch < 0 || dim <= 0 || num_heads <= 0 || num_neighbors <= 0)
    return MOSAIC_ERR_INVALID_ARGUMENT;
  if (dim % num_heads != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (dim / num_heads != kHeadDim || dim % 256 != 0) return MOSAIC_ERR_UNSUPPORTED;
  if (points_to == 0 || batch == 0) return MOSAIC_OK;
  if (!kv || !neighbors || !rel_pos || !w_q || !out) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(kv) || !aligned16(out)) return MOSAIC_ERR_INVALID_ARGUMENT;
  InterpLaunch l;
  std::memset(&l, 0, sizeof(l));
  l.kv = kv; l.neighbors = neighbors; l.rel_pos = rel_pos; l.w_q = w_q; l.out = out; l.status = status;
  l.S_to = points_to; l.S_from = points_from; l.B = batch; l.dim = dim; l.k = num_neighbors;
  l.scale = scale > 0.f ? scale : 0.125f;
  return launch_interp_attend(l, static_cast<cudaStream_t>(stream));
}

int mosaic_interp_attend_tiled(const void* kv, float* kw_workspace, const int* tile_targets,
                               const int* tile_point_off, const int* tile_points, const uint8_t* local_idx,
                               const int* order, const float* rel_pos, const float* w_q, void* out, int* status,
                               int num_tiles, int max_union, int points_from, int batch, int dim, int num_heads,
                               int num_neighbors, int kw_ready, float scale, void* stream) {
  if (num_tiles < 0 || max_union < 0 || points_from <= 0 || batch < 0 || dim <= 0 || num_heads <= 0 ||
      num_neighbors <= 0)
    return MOSAIC_ERR_INVALID_ARGUMENT;
  if (dim % num_heads != 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (dim / num_heads != kHeadDim || dim % 128 != 0) return MOSAIC_ERR_UNSUPPORTED;
  // local indices are bytes, unions padded to 16-row mma steps; two lanes per target
  if (max_union > 256 || max_union % 16 != 0 || num_neighbors > 32) return MOSAIC_ERR_UNSUPPORTED;
  if (tiled_interp_smem_bytes(max_union, num_heads, num_neighbors) > 227 * 1024) return MOSAIC_ERR_UNSUPPORTED;
  if (num_tiles == 0 || batch == 0) return MOSAIC_OK;
  if (!kv || !kw_workspace || !tile_targets || !tile_point_off || !tile_points || !local_idx || !rel_pos ||
      (!w_q && !kw_ready) ||
      !out)
    return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(kv) || !aligned16(out)) return MOSAIC_ERR_INVALID_ARGUMENT;
  InterpTiledLaunch l;
  std::memset(&l, 0, sizeof(l));
  l.kv = kv; l.kw = kw_workspace; l.tile_targets = tile_targets; l.tile_point_off = tile_point_off;
  l.tile_points = tile_points; l.local_idx = local_idx; l.order = order; l.rel_pos = rel_pos; l.w_q = w_q;
  l.out = out; l.status = status;
  l.S_from = points_from; l.B = batch; l.dim = dim; l.k = num_neighbors; l.n_tiles = num_tiles;
  l.max_union = max_union;
  l.scale = scale > 0.f ? scale : 0.125f;
  l.kw_ready = kw_ready != 0;
  return launch_interp_tiled(l, static_cast<cudaStream_t>(stream));
}

static int check_updown(const void* x, const void* w_x, const void* pos_bias, const float* norm_weight, void* out,
                        int n_coarse, int factor, int batch, int in_dim, int out_dim, float eps) {
  if (n_coarse < 0 || factor < 1 || batch < 0 || in_dim <= 0 || out_dim <= 0 || !(eps >= 0.f))
    return MOSAIC_ERR_INVALID_ARGUMENT;
  if (in_dim % 64 != 0 || out_dim % 128 != 0) return MOSAIC_ERR_UNSUPPORTED;
  if (n_coarse == 0 || batch == 0) return MOSAIC_OK;
  if (!x || !w_x || !pos_bias || !out) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(w_x) || !aligned16(pos_bias) || !aligned16(out) ||
      (norm_weight != nullptr && !aligned16(norm_weight)))
    return MOSAIC_ERR_INVALID_ARGUMENT;
  return -1;  // go on
}

int mosaic_healpix_downsample(const void* x, const void* w_x, const void* pos_bias, const float* norm_weight,
                              void* out, int* status, int n_coarse, int factor, int batch, int in_dim, int out_dim,
                              float eps, void* stream) {
  const int rc = check_updown(x, w_x, pos_bias, norm_weight, out, n_coarse, factor, batch, in_dim, out_dim, eps);
  if (rc >= 0) return rc;
  UpDownLaunch l;
  std::memset(&l, 0, sizeof(l));
  l.x = x; l.w = w_x; l.pos = pos_bias; l.norm_w = norm_weight; l.out = out;
  l.status = status; l.n = n_coarse; l.F = factor; l.B = batch; l.c_in = in_dim; l.c_out = out_dim; l.eps = eps;
  return launch_healpix_down(l, static_cast<cudaStream_t>(stream));
}

int mosaic_healpix_upsample(const void* x, const void* shortcut, const void* w_x, const void* pos_bias,
                            const float* norm_weight, void* out, int* status, int n_coarse, int factor, int batch,
                            int in_dim, int out_dim, float eps, void* stream) {
  const int rc = check_updown(x, w_x, pos_bias, norm_weight, out, n_coarse, factor, batch, in_dim, out_dim, eps);
  if (rc >= 0) return rc;
  if (shortcut != nullptr && !aligned16(shortcut)) return MOSAIC_ERR_INVALID_ARGUMENT;
  UpDownLaunch l;
  std::memset(&l, 0, sizeof(l));
  l.x = x; l.shortcut = shortcut; l.w = w_x; l.pos = pos_bias; l.norm_w = norm_weight; l.out = out;
  l.status = status; l.n = n_coarse; l.F = factor; l.B = batch; l.c_in = in_dim;
  l.c_out = out_dim; l.eps = eps;
  return launch_healpix_up(l, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
