// Block scores + top-k block selection for Mosaic's selected branch.
//
// Reference attn_topk (primitives.py:35-51):
//   k = k_cmp.repeat_interleave(G, dim=2)              -> q head j uses kv head j // G
//   S_j = q_cmp[:, :, j] @ k[:, :, j]^T                (bf16 matmul: fp32 sum, bf16 result)
//   T_h = mean_g S_{g*Hk + h}                          ('b (g h) t k -> b h t k': a STRIDED
//                                                       head group; fp32 sum, bf16 result)
//   idx[b, i, h, :] = topk(T_h[i, :], K, largest)      (int64)
// The strided group is what the reference computes even though the sparse kernel
// then uses idx[..., h, :] for the contiguous heads h*G .. h*G+G-1 (ops.py:49);
// this kernel reproduces it on purpose.
//
// One CTA handles 16 query blocks of one (b, h) and streams the nb key blocks in
// chunks of 256: 8 warps compute the 16 x 256 T chunk with mma.sync (the score
// GEMM is 0.9 GFLOP at Nside 64, far below the tensor pipe; the kernel is bound
// by reading q_cmp/k_cmp), then each warp merges 2 rows' candidates into the
// running top-K list. A candidate is the 32-bit key (order-preserving bf16 bits
// << 16) | (65535 - block): its maximum is the largest score, ties going to the
// lower block index, so the output is sorted descending like torch.topk.
#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {
namespace {

constexpr int kRows = 16;
constexpr int kChunk = 256;
constexpr int kThreads = 256;
constexpr int kMaxG = 8;
constexpr int kMaxK = 128;

struct TopkParams {
  const __nv_bfloat16* q_cmp;
  const __nv_bfloat16* k_cmp;
  int64_t* idx;
  int B, nb, Hq, Hk, K, G;
};

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint32_t order_key(float t, int block) {
  uint32_t u = __bfloat16_as_ushort(__float2bfloat16_rn(t));
  if (u == 0x8000u) u = 0;  // -0 ties with +0, as in torch.topk
  const uint32_t ord = (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
  return (ord << 16) | (0xFFFFu - static_cast<uint32_t>(block));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kThreads) topk_kernel(const TopkParams p) {
  __shared__ __align__(16) __nv_bfloat16 qs[kMaxG][kRows][64];
  __shared__ uint32_t tile[kRows][kChunk];
  __shared__ uint32_t top[kRows][kMaxK];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i0 = blockIdx.x * kRows, h = blockIdx.y, b = blockIdx.z;

  // q_cmp rows of the strided group {h, h+Hk, ...} for this CTA's 16 query blocks.
  for (int e = threadIdx.x; e < p.G * kRows * 8; e += kThreads) {
    const int g = e / (kRows * 8), r = (e / 8) % kRows, c = e % 8;
    const int i = i0 + r;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (i < p.nb) {
      const int j = g * p.Hk + h;
      val = *reinterpret_cast<const uint4*>(p.q_cmp + ((static_cast<size_t>(b) * p.nb + i) * p.Hq + j) * 64 + c * 8);
    }
    *reinterpret_cast<uint4*>(&qs[g][r][c * 8]) = val;
  }
  int count = 0;  // entries in the running top list (same in every warp)
  __syncthreads();

  const int gr = lane >> 2, gc = (lane & 3) * 2;  // mma fragment coordinates
  for (int c0 = 0; c0 < p.nb; c0 += kChunk) {
    // ---- T chunk: warp w covers keys c0 + 32w .. c0 + 32w + 31 (4 n-tiles of 8)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int key = c0 + warp * 32 + nt * 8 + gr;  // B-fragment column of this thread
      float tacc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int g = 0; g < p.G; ++g) {
        const int j = g * p.Hk + h;
        const int kv = j / p.G;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t* krow =
            key < p.nb ? reinterpret_cast<const uint32_t*>(p.k_cmp + ((static_cast<size_t>(b) * p.nb + key) * p.Hk + kv) * 64)
                       : nullptr;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          uint32_t a[4];
          a[0] = *reinterpret_cast<const uint32_t*>(&qs[g][gr][ks * 16 + gc]);
          a[1] = *reinterpret_cast<const uint32_t*>(&qs[g][gr + 8][ks * 16 + gc]);
          a[2] = *reinterpret_cast<const uint32_t*>(&qs[g][gr][ks * 16 + gc + 8]);
          a[3] = *reinterpret_cast<const uint32_t*>(&qs[g][gr + 8][ks * 16 + gc + 8]);
          const uint32_t b0 = krow ? __ldg(krow + (ks * 16 + gc) / 2) : 0u;
          const uint32_t b1 = krow ? __ldg(krow + (ks * 16 + gc + 8) / 2) : 0u;
          mma_bf16_16816(d, a, b0, b1);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) tacc[e] += round_bf16(d[e]);
      }
      // d[e]: row gr (+8 for e >= 2), key column nt*8 + gc + (e & 1)
      const float fg = static_cast<float>(p.G);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = gr + (e >= 2 ? 8 : 0);
        const int col = warp * 32 + nt * 8 + gc + (e & 1);
        const int kb = c0 + col;
        tile[r][col] = kb < p.nb ? order_key(__fdiv_rn(tacc[e], fg), kb) : 0u;
      }
    }
    __syncthreads();

    // ---- merge: warp w owns rows 2w and 2w+1
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int r = 2 * warp + rr;
      uint32_t cand[kChunk / 32 + kMaxK / 32];
#pragma unroll
      for (int s = 0; s < kChunk / 32; ++s) cand[s] = tile[r][lane + 32 * s];
#pragma unroll
      for (int s = 0; s < kMaxK / 32; ++s) {
        const int e = lane + 32 * s;
        cand[kChunk / 32 + s] = e < count ? top[r][e] : 0u;
      }
      // Skip the merge when no new candidate beats the current K-th entry.
      bool any_new = true;
      if (count >= p.K) {
        const uint32_t kth = top[r][p.K - 1];
        bool mine = false;
#pragma unroll
        for (int s = 0; s < kChunk / 32; ++s) mine |= cand[s] > kth;
        any_new = __any_sync(0xffffffffu, mine);
      }
      __syncwarp();
      if (any_new) {
        for (int e = 0; e < p.K; ++e) {
          uint32_t best = 0;
#pragma unroll
          for (int s = 0; s < kChunk / 32 + kMaxK / 32; ++s) best = max(best, cand[s]);
          best = __reduce_max_sync(0xffffffffu, best);
#pragma unroll
          for (int s = 0; s < kChunk / 32 + kMaxK / 32; ++s)
            if (cand[s] == best) cand[s] = 0u;
          if (lane == 0) top[r][e] = best;
        }
      }
      __syncwarp();
    }
    count = min(p.K, count + kChunk);
    __syncthreads();
  }

  // ---- write indices
  for (int e = threadIdx.x; e < kRows * p.K; e += kThreads) {
    const int r = e / p.K, s = e % p.K;
    const int i = i0 + r;
    if (i < p.nb)
      p.idx[((static_cast<size_t>(b) * p.nb + i) * p.Hk + h) * p.K + s] =
          static_cast<int64_t>(0xFFFFu - (top[r][s] & 0xFFFFu));
  }
}

}  // namespace

int launch_topk(const TopkLaunch& a, cudaStream_t stream) {
  TopkParams p;
  p.q_cmp = static_cast<const __nv_bfloat16*>(a.q_cmp);
  p.k_cmp = static_cast<const __nv_bfloat16*>(a.k_cmp);
  p.idx = a.idx;
  p.B = a.B;
  p.nb = a.nb;
  p.Hq = a.Hq;
  p.Hk = a.Hk;
  p.K = a.K;
  p.G = a.Hq / a.Hk;
  if (p.G > kMaxG || p.K > kMaxK || p.K > p.nb || p.nb > 65535) return MOSAIC_ERR_UNSUPPORTED;
  dim3 grid((a.nb + kRows - 1) / kRows, a.Hk, a.B);
  topk_kernel<<<grid, kThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int topk_max_k() { return kMaxK; }

}  // namespace mosaic
