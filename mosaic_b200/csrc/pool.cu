// Block mean-pooling of q, k, v over HEALPix-nested contiguous blocks, with
// Mosaic's 2D RoPE optionally applied to q and k on the way in.
//
// Reference: q_cmp/k_cmp/v_cmp = reduce(x, 'b (nb bs) h d -> b nb h d', 'mean')
// (primitives.py:65-66,76): fp32 accumulation, one rounding to bf16. RoPE
// (primitives.py:126-135): for pair p of a head, out[2p] = x[2p]*cos - x[2p+1]*sin,
// out[2p+1] = x[2p+1]*cos + x[2p]*sin in fp32 (each product and the sum rounded
// separately, as torch evaluates `x*cos + rotate_half(x)*sin`), then cast to bf16;
// pooling then averages the rotated bf16 values, exactly as the reference pools
// the rotated tensor.
//
// Layout: a block of bs rows of q is one contiguous bs x (Hq*128 B) slab (rows of
// q are [Hq, 64] contiguous), so one CTA streams the q, k and v slabs of one block
// with 16-byte vector loads: thread (chunk c, row group g) sums rows g, g+RG, ...
// of the 16-byte column chunk c, then the RG partial sums meet in shared memory.
// HBM-bound: every input byte is read exactly once.
#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {
namespace {

struct PoolParams {
  const uint4* q;
  const uint4* k;
  const uint4* v;
  const float* cos;
  const float* sin;
  uint4* q_rot;
  uint4* k_rot;
  __nv_bfloat16* q_cmp;
  __nv_bfloat16* k_cmp;
  __nv_bfloat16* v_cmp;
  int B, N, Hq, Hk, bs, nb;
  int cq, ck, cv;  // 16-byte chunks per row of q, k, v (0 when that tensor is skipped)
  int rg;          // row groups summed in parallel per chunk
};

__device__ __forceinline__ float fmul_rn(float a, float b) { return __fmul_rn(a, b); }

// Rotates the 8 bf16 values (4 RoPE pairs starting at pair index p0) of one chunk.
__device__ __forceinline__ uint4 rope_chunk(uint4 x, const float* cos_row, const float* sin_row, int p0) {
  const __nv_bfloat162* xv = reinterpret_cast<const __nv_bfloat162*>(&x);
  const float4 c = *reinterpret_cast<const float4*>(cos_row + p0);
  const float4 s = *reinterpret_cast<const float4*>(sin_row + p0);
  const float cc[4] = {c.x, c.y, c.z, c.w};
  const float ss[4] = {s.x, s.y, s.z, s.w};
  uint4 r;
  uint32_t* rv = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(xv[j]);
    const float o0 = __fadd_rn(fmul_rn(f.x, cc[j]), fmul_rn(-f.y, ss[j]));
    const float o1 = __fadd_rn(fmul_rn(f.y, cc[j]), fmul_rn(f.x, ss[j]));
    rv[j] = pack_bf16x2(o0, o1);
  }
  return r;
}

template <bool kRope>
__global__ void __launch_bounds__(512, 1) pool_kernel(const PoolParams p) {
  extern __shared__ float part[];  // [rg][C][8]
  const int C = p.cq + p.ck + p.cv;
  const int blk = blockIdx.x, b = blockIdx.y;
  const int c = threadIdx.x % C;
  const int g = threadIdx.x / C;
  if (g < p.rg) {
    const uint4* src;
    uint4* rot = nullptr;
    int cpr, cc;  // chunks per row of this tensor, chunk within the row
    if (c < p.cq) {
      src = p.q; cpr = p.cq; cc = c; rot = p.q_rot;
    } else if (c < p.cq + p.ck) {
      src = p.k; cpr = p.ck; cc = c - p.cq; rot = p.k_rot;
    } else {
      src = p.v; cpr = p.cv; cc = c - p.cq - p.ck;
    }
    const bool rotate = kRope && c < p.cq + p.ck;
    const int p0 = (cc & 7) * 4;  // first RoPE pair of this chunk within its head
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    const int row0 = blk * p.bs;
    const size_t base = (static_cast<size_t>(b) * p.N + row0) * cpr + cc;
    // 8 rows per step, all loads issued before any is used, so that each thread
    // keeps 128 bytes in flight (the kernel is bound by HBM latency x bandwidth).
    for (int r0 = g; r0 < p.bs; r0 += 8 * p.rg) {
      uint4 x[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int r = r0 + u * p.rg;
        x[u] = r < p.bs ? __ldg(src + base + static_cast<size_t>(r) * cpr) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int r = r0 + u * p.rg;
        if (r >= p.bs) continue;
        uint4 xv = x[u];
        if (rotate) {
          xv = rope_chunk(xv, p.cos + static_cast<size_t>(row0 + r) * 32, p.sin + static_cast<size_t>(row0 + r) * 32, p0);
          rot[base + static_cast<size_t>(r) * cpr] = xv;
        }
        const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(xh[j]);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) part[(g * C + c) * 8 + i] = acc[i];
  }
  __syncthreads();
  if (threadIdx.x < C) {
    float s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s[i] = part[c * 8 + i];
#pragma unroll
      for (int gg = 1; gg < p.rg; ++gg) s[i] += part[(gg * C + c) * 8 + i];
    }
    __nv_bfloat16* dst;
    int cpr, cc;
    if (c < p.cq) {
      dst = p.q_cmp; cpr = p.cq; cc = c;
    } else if (c < p.cq + p.ck) {
      dst = p.k_cmp; cpr = p.ck; cc = c - p.cq;
    } else {
      dst = p.v_cmp; cpr = p.cv; cc = c - p.cq - p.ck;
    }
    const float n = static_cast<float>(p.bs);
    uint4 u;
    u.x = pack_bf16x2(__fdiv_rn(s[0], n), __fdiv_rn(s[1], n));
    u.y = pack_bf16x2(__fdiv_rn(s[2], n), __fdiv_rn(s[3], n));
    u.z = pack_bf16x2(__fdiv_rn(s[4], n), __fdiv_rn(s[5], n));
    u.w = pack_bf16x2(__fdiv_rn(s[6], n), __fdiv_rn(s[7], n));
    reinterpret_cast<uint4*>(dst)[(static_cast<size_t>(b) * p.nb + blk) * cpr + cc] = u;
  }
}

}  // namespace

int launch_pool(const PoolLaunch& a, cudaStream_t stream) {
  PoolParams p;
  p.q = static_cast<const uint4*>(a.q);
  p.k = static_cast<const uint4*>(a.k);
  p.v = static_cast<const uint4*>(a.v);
  p.cos = a.rope_cos;
  p.sin = a.rope_sin;
  p.q_rot = static_cast<uint4*>(a.q_rot);
  p.k_rot = static_cast<uint4*>(a.k_rot);
  p.q_cmp = static_cast<__nv_bfloat16*>(a.q_cmp);
  p.k_cmp = static_cast<__nv_bfloat16*>(a.k_cmp);
  p.v_cmp = static_cast<__nv_bfloat16*>(a.v_cmp);
  p.B = a.B;
  p.N = a.N;
  p.Hq = a.Hq;
  p.Hk = a.Hk;
  p.bs = a.bs;
  p.nb = a.N / a.bs;
  const bool rope = a.rope_cos != nullptr;
  // With RoPE the rotated q must be produced even when its pooled mean is not needed.
  p.cq = (a.q_cmp != nullptr || rope) ? a.Hq * 8 : 0;
  p.ck = a.Hk * 8;
  p.cv = a.v_cmp != nullptr ? a.Hk * 8 : 0;
  if (p.cq > 0 && a.q_cmp == nullptr) return MOSAIC_ERR_INVALID_ARGUMENT;
  const int C = p.cq + p.ck + p.cv;
  if (C > 512) return MOSAIC_ERR_UNSUPPORTED;
  p.rg = 512 / C < 4 ? 512 / C : 4;
  const int threads = ((C * p.rg + 31) / 32) * 32;
  const size_t smem = static_cast<size_t>(p.rg) * C * 8 * sizeof(float);
  dim3 grid(p.nb, a.B);
  if (rope) {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(pool_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return MOSAIC_ERR_CUDA;
    pool_kernel<true><<<grid, threads, smem, stream>>>(p);
  } else {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(pool_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return MOSAIC_ERR_CUDA;
    pool_kernel<false><<<grid, threads, smem, stream>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

}  // namespace mosaic
