// Cross-attention interpolation between the lat-lon and HEALPix grids
// (primitives.CrossAttentionInterpolate.forward, primitives.py:264-284): for every
// target point s, batch member b and head h,
//   q_j  = to_q.weight[h] rel_pos[s, j]             (3 -> head_dim, per neighbour j)
//   a_j  = softmax_j(scale * q_j . k[n(s, j), b, h]) over the k neighbours (fp32)
//   o    = sum_j a_j v[n(s, j), b, h]
// with kv = to_kv(RMSNorm(x_from)) laid out [S_from, B, 2, H, 64] ('s b (n h d)').
//
// One warp per (s, b): each lane owns 8 consecutive feature columns (16-byte gathers;
// 8 lanes per head), so a warp covers 4 heads per pass and loops over dim / 256 passes.
// q is recomputed from the 3-component relative position in registers (3 FMAs per
// value) instead of being read: the reference's q tensor is S_to x k x dim. Scores are
// reduced over the head's 8 lanes with shuffles and folded into an online softmax.
// Targets run in index order, so neighbouring targets (which share most neighbours)
// gather from L2 together. HBM / L2-bound gather; no tensor core.
//
// rms_kernel: rinv[r] = 1 / sqrt(mean_d x[r, d]^2 + eps), the row factor of RMSNorm
// without an affine weight (torch.nn.RMSNorm, elementwise_affine=False), applied by
// the to_kv GEMM's epilogue.
#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {
namespace {

__global__ void interp_attend_kernel(const __nv_bfloat16* __restrict__ kv, const int* __restrict__ nbr,
                                     const float* __restrict__ rel, const float* __restrict__ wq,
                                     __nv_bfloat16* __restrict__ out, int* status, int S_to, int S_from, int B,
                                     int dim, int kn, float scale) {
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<long long>(S_to) * B) return;  // warp-uniform
  const int s = static_cast<int>(w / B), b = static_cast<int>(w % B);
  const int* nb = nbr + static_cast<size_t>(s) * kn;
  const float* rp = rel + static_cast<size_t>(s) * kn * 3;
  for (int d0 = lane * 8; d0 < dim; d0 += 256) {
    float wx[8], wy[8], wz[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      wx[i] = __ldg(wq + (d0 + i) * 3);
      wy[i] = __ldg(wq + (d0 + i) * 3 + 1);
      wz[i] = __ldg(wq + (d0 + i) * 3 + 2);
    }
    float m = -INFINITY, l = 0.f, acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j = 0; j < kn; ++j) {
      int n = __ldg(nb + j);
      if (n < 0 || n >= S_from) {  // out-of-range neighbour: reported, read as point 0
        if (status != nullptr && lane == 0) atomicOr(status, MOSAIC_STATUS_BAD_INDEX);
        n = 0;
      }
      const float r0 = __ldg(rp + 3 * j), r1 = __ldg(rp + 3 * j + 1), r2 = __ldg(rp + 3 * j + 2);
      const __nv_bfloat16* row = kv + (static_cast<size_t>(n) * B + b) * 2 * dim;
      const uint4 kk = __ldg(reinterpret_cast<const uint4*>(row + d0));
      const uint4 vv = __ldg(reinterpret_cast<const uint4*>(row + dim + d0));
      const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kk);
      float part = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 kf = __bfloat1622float2(k2[i]);
        const float q0 = fmaf(wz[2 * i], r2, fmaf(wy[2 * i], r1, wx[2 * i] * r0));
        const float q1 = fmaf(wz[2 * i + 1], r2, fmaf(wy[2 * i + 1], r1, wx[2 * i + 1] * r0));
        part = fmaf(q0, kf.x, fmaf(q1, kf.y, part));
      }
      // the head's 8 lanes (lanes 8h' .. 8h'+7 of the warp)
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      part += __shfl_xor_sync(0xffffffffu, part, 4);
      const float sc = part * scale;
      const float m_new = fmaxf(m, sc);
      const float alpha = __expf(m - m_new);  // 0 on the first neighbour (m = -inf)
      const float pj = __expf(sc - m_new);
      l = fmaf(l, alpha, pj);
      const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&vv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 vf = __bfloat1622float2(v2[i]);
        acc[2 * i] = fmaf(acc[2 * i], alpha, pj * vf.x);
        acc[2 * i + 1] = fmaf(acc[2 * i + 1], alpha, pj * vf.y);
      }
      m = m_new;
    }
    const float inv = 1.0f / l;
    uint4 o;
    o.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
    o.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
    o.z = pack_bf16x2(acc[4] * inv, acc[5] * inv);
    o.w = pack_bf16x2(acc[6] * inv, acc[7] * inv);
    *reinterpret_cast<uint4*>(out + (static_cast<size_t>(s) * B + b) * dim + d0) = o;
  }
}

// One warp per row: 16-byte loads, fp32 sum of squares, shuffle reduction.
__global__ void rms_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ rinv, long long rows, int dim,
                           float eps) {
  const long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const __nv_bfloat16* row = x + r * dim;
  float ss = 0.f;
  for (int d0 = lane * 8; d0 < dim; d0 += 256) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + d0));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) rinv[r] = rsqrtf(ss / dim + eps);
}

}  // namespace

int launch_interp_attend(const InterpLaunch& a, cudaStream_t stream) {
  const long long warps = static_cast<long long>(a.S_to) * a.B;
  if (warps == 0) return MOSAIC_OK;
  const unsigned grid = static_cast<unsigned>((warps * 32 + 255) / 256);
  interp_attend_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(a.kv), a.neighbors, a.rel_pos,
                                                 a.w_q, static_cast<__nv_bfloat16*>(a.out), a.status, a.S_to,
                                                 a.S_from, a.B, a.dim, a.k, a.scale);
  return cudaGetLastError() == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int launch_row_rms(const void* x, float* rinv, long long rows, int dim, float eps, cudaStream_t stream) {
  if (rows == 0) return MOSAIC_OK;
  const unsigned grid = static_cast<unsigned>((rows * 32 + 255) / 256);
  rms_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), rinv, rows, dim, eps);
  return cudaGetLastError() == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

}  // namespace mosaic
