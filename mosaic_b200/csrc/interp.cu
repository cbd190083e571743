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
// interp_tiled_kernel: the same attention over tiles of spatially adjacent targets whose
// neighbour lists were merged on the host into one union of source points per tile (the
// neighbour table is static). Two changes of arithmetic order, exact in real numbers:
// the score uses kw = (to_q.weight per head)^T k, a 3-vector per (point, head) computed
// once per source point by interp_kw_kernel, so a score costs 3 FMAs instead of 64 q
// values rebuilt from rel_pos; and the softmax is the two-pass form (all k scores, then
// max and sum) in place of the online one. One CTA per (tile, b) copies the union's v
// columns of a 256-column pass (and its kw, once) into shared memory; each warp takes a
// target: lanes are neighbours for the scores and softmax, then columns for sum_j p_j v_j,
// reading v from shared memory. Adjacent targets share most neighbours, so L2 -> SM
// traffic drops by the union reuse factor (about 9x from lat-lon to HEALPix).
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

// kw[p, b, h, 0:3] = sum over the head's 64 columns c of k[p, b, c] * to_q.weight[c, :]
// (fp32, from the bf16 k; kw[.., 3] = 0): by linearity q_j . k = rel_pos[s, j] .
// kw[n(s, j), b, h], so one 3-vector per (source point, head) replaces the 64-wide q of
// every (target, neighbour) pair. Lanes own 8 columns (8 lanes per head); a warp holds
// the 24 weights of its columns in registers for a 256-column pass over its 4 rows.
constexpr int kKwRowsPerWarp = 4;

__global__ void __launch_bounds__(256) interp_kw_kernel(const __nv_bfloat16* __restrict__ kv,
                                                        const float* __restrict__ wq, float4* __restrict__ kw,
                                                        long long rows, int dim) {
  const int lane = threadIdx.x & 31, H = dim >> 6;
  const long long row0 = (static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * kKwRowsPerWarp;
  if (row0 >= rows) return;
  for (int c0 = 0; c0 < dim; c0 += 256) {
    const int c = c0 + lane * 8;
    // dim % 256 == 128: lanes beyond dim in the last pass contribute zeros
    const bool in = c < dim;
    uint4 raw[kKwRowsPerWarp];  // the warp's rows first, so that their loads are in flight together
#pragma unroll
    for (int r = 0; r < kKwRowsPerWarp; ++r)
      raw[r] = in && row0 + r < rows ? __ldg(reinterpret_cast<const uint4*>(kv + (row0 + r) * 2 * dim + c))
                                     : make_uint4(0, 0, 0, 0);
    float w[24];
    const float4* w4 = reinterpret_cast<const float4*>(wq + (in ? c : 0) * 3);  // 24 floats, 96 B
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const float4 t = __ldg(w4 + i);
      w[4 * i] = t.x; w[4 * i + 1] = t.y; w[4 * i + 2] = t.z; w[4 * i + 3] = t.w;
    }
#pragma unroll
    for (int r = 0; r < kKwRowsPerWarp; ++r) {
      const uint32_t kwd[4] = {raw[r].x, raw[r].y, raw[r].z, raw[r].w};
      float a0 = 0.f, a1 = 0.f, a2 = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float kx = __uint_as_float(kwd[i] << 16), ky = __uint_as_float(kwd[i] & 0xffff0000u);
        a0 = fmaf(kx, w[6 * i], a0);
        a1 = fmaf(kx, w[6 * i + 1], a1);
        a2 = fmaf(kx, w[6 * i + 2], a2);
        a0 = fmaf(ky, w[6 * i + 3], a0);
        a1 = fmaf(ky, w[6 * i + 4], a1);
        a2 = fmaf(ky, w[6 * i + 5], a2);
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        a0 += __shfl_xor_sync(0xffffffffu, a0, o);
        a1 += __shfl_xor_sync(0xffffffffu, a1, o);
        a2 += __shfl_xor_sync(0xffffffffu, a2, o);
      }
      if ((lane & 7) == 0 && in && row0 + r < rows) kw[(row0 + r) * H + (c >> 6)] = make_float4(a0, a1, a2, 0.f);
    }
  }
}

// ---- interp_tiled_kernel ------------------------------------------------------------
// Per tile (<= 32 targets, a union of U <= 256 source points padded to a multiple of 16)
// and batch member b, for every head h the tile's attention is the product
//     out_h [targets x 64] = P_h [targets x U] . V_h [U x 64]
// where row t of P_h holds target t's softmax weights at the union positions of its
// neighbours and zeros elsewhere (a tile's neighbour lists have no repeats, so the
// positions are fixed per tile). The product runs on the tensor cores with mma.sync
// m16n8k16 bf16 / fp32 accumulate; only the scores and the softmax are per neighbour, on
// the FMA pipe. Warp w owns rows 16 (w / 2) .. + 15 of the tile and the head of parity
// w % 2 in every 2-head chunk, so each lane loads its 16 neighbour slots (relative
// position, union position) once per tile and keeps them in registers for all heads,
// and the P_s positions it writes stay the same from head to head. Shared memory:
//   V_s[2]  U x (2 heads x 64 bf16), rows padded to 272 B  (cp.async 16-byte copies,
//                                                          double-buffered over chunks)
//   kw_s    H x U x float4, head-major                    (cp.async, once; at fixed head,
//                                                          random points spread over all banks)
//   P_s     per warp 16 x U bf16, rows padded (+16 B)     (scattered softmax weights)
//   pts_s   U int32
// The copies are the per-thread asynchronous kind: a tile moves a few hundred 256-byte
// rows, for which per-operation bulk (TMA) copies cost far more than the bytes.
constexpr int kTileWarps = 4;
constexpr int kTileThreads = kTileWarps * 32;
constexpr int kTileMaxTargets = 32;
constexpr int kVRow = 272;  // 256 B of v (2 heads) + 16 B: ldmatrix rows hit distinct banks

struct TiledSmem {
  size_t v0, v1, kw, p, pts, total;
  int p_stride;
};
__host__ __device__ inline TiledSmem tiled_layout(int U, int H) {
  TiledSmem L;
  size_t o = 0;
  L.v0 = o; o += static_cast<size_t>(U) * kVRow;
  L.v1 = o; o += static_cast<size_t>(U) * kVRow;
  L.kw = o; o += static_cast<size_t>(U) * H * 16;
  L.p_stride = 2 * U + 16;
  L.p = o; o += static_cast<size_t>(kTileWarps) * 16 * L.p_stride;
  L.pts = o; o += static_cast<size_t>(U) * 4;
  L.total = o;
  return L;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(__cvta_generic_to_global(src))
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// v columns [chunk * 128, chunk * 128 + 128) of the tile's union rows into one V_s buffer
__device__ __forceinline__ void stage_v_chunk(uint8_t* dst, const int* pts_s, const __nv_bfloat16* kv, int U,
                                              size_t row_elems, size_t b_off, int chunk) {
  for (int e = threadIdx.x; e < U * 16; e += kTileThreads) {
    const int u = e >> 4, piece = e & 15;
    cp_async16(dst + u * kVRow + piece * 16,
               kv + static_cast<size_t>(pts_s[u]) * row_elems + b_off + chunk * 128 + piece * 8);
  }
}

// Quad transpose of an m16n8 accumulator row (elements `e`, `e` + 1 of the 8 n tiles) so
// that each lane stores 16 contiguous bytes per n tile it ends up owning.
__device__ __forceinline__ void store_quad_rows(const float (&acc)[8][4], int e, __nv_bfloat16* orow, int h,
                                                int lane) {
  const int q = lane & 3;
  uint32_t w[8];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) w[nt] = pack_bf16x2(acc[nt][e], acc[nt][e + 1]);
  // step 1 (partner q ^ 1): even q keeps even n tiles, odd q odd ones; 2 words each
  uint32_t x[8];  // x[2k], x[2k+1]: columns 4 (q / 2) .. + 3 of n tile 2k + (q & 1)
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t send = (q & 1) ? w[2 * k] : w[2 * k + 1];
    const uint32_t got = __shfl_xor_sync(0xffffffffu, send, 1);
    const uint32_t mine = (q & 1) ? w[2 * k + 1] : w[2 * k];
    x[2 * k] = (q & 1) ? got : mine;
    x[2 * k + 1] = (q & 1) ? mine : got;
  }
  // step 2 (partner q ^ 2): q < 2 keeps n tiles 2k with k even, q >= 2 those with k odd
  uint32_t y[8];  // y[4m .. 4m+3]: columns 0..7 of n tile (q & 1) + 2 (q >> 1) + 4 m
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    const int ke = 2 * m, ko = 2 * m + 1;  // the pair of k this step merges
    const uint32_t s0 = (q & 2) ? x[2 * ke] : x[2 * ko];
    const uint32_t s1 = (q & 2) ? x[2 * ke + 1] : x[2 * ko + 1];
    const uint32_t g0 = __shfl_xor_sync(0xffffffffu, s0, 2);
    const uint32_t g1 = __shfl_xor_sync(0xffffffffu, s1, 2);
    const uint32_t m0 = (q & 2) ? x[2 * ko] : x[2 * ke];
    const uint32_t m1 = (q & 2) ? x[2 * ko + 1] : x[2 * ke + 1];
    // the lane with q < 2 holds columns 0-3 and receives 4-7; q >= 2 the reverse
    y[4 * m] = (q & 2) ? g0 : m0;
    y[4 * m + 1] = (q & 2) ? g1 : m1;
    y[4 * m + 2] = (q & 2) ? m0 : g0;
    y[4 * m + 3] = (q & 2) ? m1 : g1;
  }
  if (orow != nullptr) {
    const int nt0 = (q & 1) + 2 * (q >> 1);
    __nv_bfloat16* base = orow - q * 2 + h * 64;  // orow points at column 2q of the row
    *reinterpret_cast<uint4*>(base + nt0 * 8) = make_uint4(y[0], y[1], y[2], y[3]);
    *reinterpret_cast<uint4*>(base + (nt0 + 4) * 8) = make_uint4(y[4], y[5], y[6], y[7]);
  }
}

__global__ void __launch_bounds__(kTileThreads) interp_tiled_kernel(
    const __nv_bfloat16* __restrict__ kv, const float4* __restrict__ kw, const int* __restrict__ tile_targets,
    const int* __restrict__ tile_point_off, const int* __restrict__ tile_points, const uint8_t* __restrict__ local,
    const int* __restrict__ order, const float* __restrict__ rel, __nv_bfloat16* __restrict__ out, int* status,
    int S_from, int B, int dim, int kn, int max_union, float scale_log2) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tile = blockIdx.x, b = blockIdx.y;
  const int t0 = __ldg(tile_targets + tile);
  const int T = __ldg(tile_targets + tile + 1) - t0;
  const int p0 = __ldg(tile_point_off + tile), U = __ldg(tile_point_off + tile + 1) - p0;
  if (T < 0 || T > kTileMaxTargets || U <= 0 || (U & 15) != 0 || U > max_union) {  // inconsistent tile tables
    if (threadIdx.x == 0 && status != nullptr) atomicOr(status, MOSAIC_STATUS_BAD_INDEX);
    return;
  }
  const int H = dim >> 6, n_chunks = H >> 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Warp w takes the head of parity w % 2 in every chunk, for row block w / 2; a tile of
  // at most 16 targets has one row block, and then warps 2 and 3 take the next chunk
  // instead (two chunks per step, both buffers in use).
  const bool pair = T <= 16 && n_chunks > 1;
  const int rb = pair ? 0 : warp >> 1, hl = warp & 1, cw_off = pair ? warp >> 1 : 0;
  const TiledSmem L = tiled_layout(U, H);
  uint8_t* const v_s0 = smem + L.v0;  // chunk c lives in v_s0 + (c & 1) * v_step
  const size_t v_step = L.v1 - L.v0;
  const float4* kw_s = reinterpret_cast<const float4*>(smem + L.kw);
  uint8_t* p_w = smem + L.p + static_cast<size_t>(warp) * 16 * L.p_stride;
  int* pts_s = reinterpret_cast<int*>(smem + L.pts);
  const size_t row_elems = static_cast<size_t>(B) * 2 * dim;
  const size_t b_off = static_cast<size_t>(b) * 2 * dim + dim;  // v of member b inside a point's row

  for (int u = threadIdx.x; u < U; u += kTileThreads) {
    int n = __ldg(tile_points + p0 + u);
    if (n < 0 || n >= S_from) {
      if (status != nullptr) atomicOr(status, MOSAIC_STATUS_BAD_INDEX);
      n = 0;
    }
    pts_s[u] = n;
  }
  __syncthreads();
  for (int u = threadIdx.x >> 4; u < U; u += kTileThreads >> 4) {  // 16 threads per point
    const float4* src = kw + (static_cast<size_t>(pts_s[u]) * B + b) * H;
    for (int hh = threadIdx.x & 15; hh < H; hh += 16)
      cp_async16(smem + L.kw + (static_cast<size_t>(hh) * U + u) * 16, src + hh);
  }
  stage_v_chunk(v_s0, pts_s, kv, U, row_elems, b_off, 0);
  cp_async_commit();
  if (n_chunks > 1) stage_v_chunk(v_s0 + v_step, pts_s, kv, U, row_elems, b_off, 1);
  cp_async_commit();
  for (int e = lane * 16; e < 16 * L.p_stride; e += 32 * 16)  // this warp's P_s starts at zero
    *reinterpret_cast<uint4*>(p_w + e) = make_uint4(0, 0, 0, 0);

  // score lanes: row sr = lane / 2 of the warp's block, neighbour slots j = 2 i + (lane & 1)
  const int sr = lane >> 1, shalf = lane & 1;
  const int tl = rb * 16 + sr;
  const bool row_ok = tl < T;
  float r0[16], r1[16], r2[16];
  int ku[16];  // union position of slot i, or -1
  {
    const int t = row_ok ? (order != nullptr ? __ldg(order + t0 + tl) : t0 + tl) : 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int j = 2 * i + shalf;
      ku[i] = -1;
      r0[i] = r1[i] = r2[i] = 0.f;
      if (row_ok && j < kn) {
        int u = __ldg(local + static_cast<size_t>(t) * kn + j);
        if (u >= U) {
          if (status != nullptr) atomicOr(status, MOSAIC_STATUS_BAD_INDEX);
          u = 0;
        }
        ku[i] = u;
        const float* rp = rel + (static_cast<size_t>(t) * kn + j) * 3;
        r0[i] = __ldg(rp);
        r1[i] = __ldg(rp + 1);
        r2[i] = __ldg(rp + 2);
      }
    }
  }
  // epilogue rows lane / 4 and lane / 4 + 8 of the warp's block
  const int er0 = rb * 16 + (lane >> 2), er1 = er0 + 8;
  __nv_bfloat16* orow0 = nullptr;
  __nv_bfloat16* orow1 = nullptr;
  if (er0 < T)
    orow0 = out + (static_cast<size_t>(order != nullptr ? __ldg(order + t0 + er0) : t0 + er0) * B + b) * dim +
            (lane & 3) * 2;
  if (er1 < T)
    orow1 = out + (static_cast<size_t>(order != nullptr ? __ldg(order + t0 + er1) : t0 + er1) * B + b) * dim +
            (lane & 3) * 2;
  const bool warp_busy = rb * 16 < T;
  // 16-point blocks of the union that the warp's rows touch: the other k steps are zero
  uint32_t kmask = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if (ku[i] >= 0) kmask |= 1u << (ku[i] >> 4);
  kmask = __reduce_or_sync(0xffffffffu, kmask);
  // mma lanes: ldmatrix row addresses
  const uint32_t a_addr = smem_u32(p_w) + (((lane >> 3) & 1) * 8 + (lane & 7)) * L.p_stride + (lane >> 4) * 16;
  const uint32_t b_off_s = (((lane >> 3) & 1) * 8 + (lane & 7)) * kVRow + (lane >> 4) * 16 + hl * 128;
  for (int c = 0; c < n_chunks; c += pair ? 2 : 1) {
    if (pair)
      cp_async_wait0();  // both chunks of this step (and kw) have landed for this thread
    else
      cp_async_wait1();  // this thread's copies of chunk c (and of kw) have landed
    __syncthreads();     // ... and everyone's
    const int cw = c + cw_off;  // this warp's chunk
    if (warp_busy && cw < n_chunks) {
      const int h = 2 * cw + hl;
      // ---- scores and softmax of the block's 16 targets for head h, into P_s
      float sc[16];
      float m = -INFINITY;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 w = kw_s[h * U + max(ku[i], 0)];
        sc[i] = ku[i] >= 0 ? fmaf(r2[i], w.z, fmaf(r1[i], w.y, r0[i] * w.x)) * scale_log2 : -INFINITY;
        m = fmaxf(m, sc[i]);
      }
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      float l = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        sc[i] = ku[i] >= 0 ? ex2_approx(sc[i] - m) : 0.f;
        l += sc[i];
      }
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      const float inv = row_ok ? __fdividef(1.0f, l) : 0.f;
      uint8_t* p_row = p_w + sr * L.p_stride;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (ku[i] >= 0) *reinterpret_cast<__nv_bfloat16*>(p_row + ku[i] * 2) = __float2bfloat16_rn(sc[i] * inv);
      __syncwarp();
      // ---- out_h[16 x 64] = P_h[16 x U] . V_h[U x 64]
      float acc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
      const uint32_t bb = smem_u32(v_s0 + (cw & 1) * v_step) + b_off_s;
      for (uint32_t km = kmask; km != 0; km &= km - 1) {
        const int ks = __ffs(km) - 1;
        uint32_t a0, a1, a2, a3;
        ldsm_x4(a_addr + ks * 32, a0, a1, a2, a3);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(bb + ks * 16 * kVRow + np * 32, b0, b1, b2, b3);
          mma_bf16_16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
          mma_bf16_16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
        }
      }
      // ---- epilogue: lane q of a quad holds columns 8 nt + 2q, +1 of rows er0 / er1; two
      // butterfly exchanges leave it 8 whole columns of n tiles nt = q' and q' + 4
      // (q' = 0, 2, 1, 3 for q = 0, 1, 2, 3), stored as 16-byte pieces.
      store_quad_rows(acc, 0, orow0, h, lane);
      store_quad_rows(acc, 2, orow1, h, lane);
      __syncwarp();  // the next head rewrites the same P_s positions
    }
    __syncthreads();  // the step's buffers are free: refill them with the chunks two ahead
    if (c + 2 < n_chunks) stage_v_chunk(v_s0 + (c & 1) * v_step, pts_s, kv, U, row_elems, b_off, c + 2);
    cp_async_commit();  // one group per chunk (possibly empty) keeps wait_group 1 exact
    if (pair) {
      if (c + 3 < n_chunks) stage_v_chunk(v_s0 + v_step, pts_s, kv, U, row_elems, b_off, c + 3);
      cp_async_commit();
    }
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

size_t tiled_interp_smem_bytes(int max_union, int H, int /*k*/) { return tiled_layout(max_union, H).total; }

int launch_interp_tiled(const InterpTiledLaunch& a, cudaStream_t stream) {
  if (a.n_tiles == 0 || a.B == 0) return MOSAIC_OK;
  const long long rows = static_cast<long long>(a.S_from) * a.B;
  const long long kw_rows_per_block = 8LL * kKwRowsPerWarp;
  if (!a.kw_ready)
    interp_kw_kernel<<<static_cast<unsigned>((rows + kw_rows_per_block - 1) / kw_rows_per_block), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(a.kv), a.w_q, reinterpret_cast<float4*>(a.kw), rows, a.dim);
  const size_t smem = tiled_layout(a.max_union, a.dim / 64).total;
  static size_t set_bytes[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOSAIC_ERR_CUDA;
  if (set_bytes[dev] < smem) {
    if (cudaFuncSetAttribute(interp_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess ||
        cudaFuncSetAttribute(interp_tiled_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100) !=
            cudaSuccess)
      return MOSAIC_ERR_CUDA;
    set_bytes[dev] = smem;
  }
  interp_tiled_kernel<<<dim3(a.n_tiles, a.B), kTileThreads, smem, stream>>>(
      static_cast<const __nv_bfloat16*>(a.kv), reinterpret_cast<const float4*>(a.kw), a.tile_targets,
      a.tile_point_off, a.tile_points, a.local_idx, a.order, a.rel_pos, static_cast<__nv_bfloat16*>(a.out), a.status,
      a.S_from, a.B, a.dim, a.k, a.max_union, a.scale * 1.4426950408889634f);
  return cudaGetLastError() == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int launch_row_rms(const void* x, float* rinv, long long rows, int dim, float eps, cudaStream_t stream) {
  if (rows == 0) return MOSAIC_OK;
  const unsigned grid = static_cast<unsigned>((rows * 32 + 255) / 256);
  rms_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), rinv, rows, dim, eps);
  return cudaGetLastError() == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

}  // namespace mosaic
