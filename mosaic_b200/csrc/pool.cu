// Block mean-pooling of q, k, v over HEALPix-nested contiguous blocks, with
// Mosaic's 2D RoPE optionally applied to q and k on the way in.
//
// Reference: q_cmp/k_cmp/v_cmp = reduce(x, 'b (nb bs) h d -> b nb h d', 'mean')
// (primitives.py:65-66,76): fp32 accumulation, one rounding to the activation type
// (bf16, or fp16 under the reference's fp16 autocast). RoPE (primitives.py:126-135):
// for pair p of a head, out[2p] = x[2p]*cos - x[2p+1]*sin, out[2p+1] = x[2p+1]*cos +
// x[2p]*sin in fp32 (each product and the sum rounded separately, as torch evaluates
// `x*cos + rotate_half(x)*sin`), then cast to the activation type; pooling then
// averages the rotated values, exactly as the reference pools the rotated tensor.
//
// Layout: a block of bs rows is a contiguous bs x (H*128 B) slab per tensor, and one
// head of one row is 128 contiguous bytes. A work unit is one (batch, block, head of
// q, k or v) and belongs to one warp: lane l owns the 16-byte chunk l % 8 of the head
// and the rows l / 8, l / 8 + 4, ... of the block, loads a 64-row batch as sixteen
// 16-byte loads (every warp instruction touches four full 128-byte lines), and the
// four row groups meet through two shuffles. The warps are persistent: while a warp
// adds one batch, the sixteen loads of its next batch (the next unit's, at the end
// of a block) are already in flight, so every lane keeps 256 bytes outstanding all
// the time. No shared memory and no block barrier.
// Rows past the end of a block (block sizes that are not multiples of 64) are
// skipped. HBM-bound: every input byte is read exactly once.
#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {
namespace {

constexpr int kWarpsPerCta = 4;
// Rows of a block per load batch: 64 (16 loads per lane), or 32 with RoPE, whose
// rotation and rotated-copy stores need the registers (at 64 the RoPE kernel held
// 8 warps per SM and ran at a quarter of the plain kernel's bandwidth).
template <bool kRope>
constexpr int rows_per_batch() { return kRope ? 32 : 64; }

struct PoolParams {
  const uint4* q;
  const uint4* k;
  const uint4* v;
  const float* cos;
  const float* sin;
  uint4* q_rot;
  uint4* k_rot;
  uint4* q_cmp;
  uint4* k_cmp;
  uint4* v_cmp;
  int B, N, Hq, Hk, bs, nb;
  int nq, nv;  // q / v head slots per block (0 when that tensor is skipped)
  int slots;   // nq + Hk + nv
  long long units;
};

// Rotates the 8 values (4 RoPE pairs starting at pair index p0) of one chunk.
template <bool kF16>
__device__ __forceinline__ uint4 rope_chunk(uint4 x, const float* cos_row, const float* sin_row, int p0) {
  using A = Act<kF16>;
  const uint32_t* xv = reinterpret_cast<const uint32_t*>(&x);
  const float4 c = *reinterpret_cast<const float4*>(cos_row + p0);
  const float4 s = *reinterpret_cast<const float4*>(sin_row + p0);
  const float cc[4] = {c.x, c.y, c.z, c.w};
  const float ss[4] = {s.x, s.y, s.z, s.w};
  uint4 r;
  uint32_t* rv = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = A::unpack(xv[j]);
    const float o0 = __fadd_rn(__fmul_rn(f.x, cc[j]), __fmul_rn(-f.y, ss[j]));
    const float o1 = __fadd_rn(__fmul_rn(f.y, cc[j]), __fmul_rn(f.x, ss[j]));
    rv[j] = A::pack(o0, o1);
  }
  return r;
}

template <bool kF16>
__device__ __forceinline__ void add_chunk(float (&acc)[8], uint4 x) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&x);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = Act<kF16>::unpack(w[j]);
    acc[2 * j] += f.x;
    acc[2 * j + 1] += f.y;
  }
}

// One work unit of the warp: which tensor, head and block, and where its rows are.
struct UnitRef {
  const uint4* src;
  uint4* rot;
  uint4* dst;
  size_t base, pitch, out;  // 16-byte chunk indices (of this lane's chunk c) and the row pitch
  int row0;
  bool rotate;
};

template <bool kRope>
__device__ __forceinline__ UnitRef unit_ref(const PoolParams& p, long long u, int c) {
  UnitRef r;
  const int slot = static_cast<int>(u % p.slots);
  const long long bb = u / p.slots;  // b * nb + blk
  const int blk = static_cast<int>(bb % p.nb), b = static_cast<int>(bb / p.nb);
  int H, h;
  r.rot = nullptr;
  if (slot < p.nq) {
    r.src = p.q; r.rot = p.q_rot; r.dst = p.q_cmp; H = p.Hq; h = slot;
  } else if (slot < p.nq + p.Hk) {
    r.src = p.k; r.rot = p.k_rot; r.dst = p.k_cmp; H = p.Hk; h = slot - p.nq;
  } else {
    r.src = p.v; r.dst = p.v_cmp; H = p.Hk; h = slot - p.nq - p.Hk;
  }
  r.rotate = kRope && slot < p.nq + p.Hk;
  r.row0 = blk * p.bs;
  r.pitch = static_cast<size_t>(H) * 8;
  r.base = (static_cast<size_t>(b) * p.N + r.row0) * r.pitch + static_cast<size_t>(h) * 8 + c;
  r.out = (static_cast<size_t>(b) * p.nb + blk) * r.pitch + static_cast<size_t>(h) * 8 + c;
  return r;
}

// Issues the loads of rows r0 + rg + 4 i (i < NR / 4) of a unit.
template <int NR>
__device__ __forceinline__ void load_batch(uint4 (&x)[NR / 4], const UnitRef& r, int r0, int rg, int bs) {
#pragma unroll
  for (int i = 0; i < NR / 4; ++i) {
    const int row = r0 + rg + 4 * i;
    x[i] = row < bs ? __ldg(r.src + r.base + static_cast<size_t>(row) * r.pitch) : make_uint4(0, 0, 0, 0);
  }
}

// Persistent warps: warp w of the grid takes units w, w + warps, ... and keeps the
// next 64-row batch's sixteen 16-byte loads in flight while it adds the current one.
template <bool kF16, bool kRope>
__global__ void __launch_bounds__(kWarpsPerCta * 32) pool_kernel(const PoolParams p) {
  using A = Act<kF16>;
  const long long warps = static_cast<long long>(gridDim.x) * kWarpsPerCta;
  long long u = static_cast<long long>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5);
  if (u >= p.units) return;
  const int lane = threadIdx.x & 31;
  const int c = lane & 7, rg = lane >> 3;
  UnitRef cur = unit_ref<kRope>(p, u, c);
  int r0 = 0;
  constexpr int NR = rows_per_batch<kRope>();
  uint4 x[NR / 4], nx[NR / 4];
  load_batch<NR>(x, cur, 0, rg, p.bs);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  while (true) {
    // the batch after this one: the rest of this block, else the warp's next unit
    long long nu = u;
    int nr0 = r0 + NR;
    if (nr0 >= p.bs) {
      nu = u + warps;
      nr0 = 0;
    }
    const bool more = nu < p.units;
    UnitRef nxt = more ? unit_ref<kRope>(p, nu, c) : cur;
    if (more) load_batch<NR>(nx, nxt, nr0, rg, p.bs);
#pragma unroll
    for (int i = 0; i < NR / 4; ++i) {
      uint4 xv = x[i];
      const int r = r0 + rg + 4 * i;
      if (r >= p.bs) continue;
      if (cur.rotate) {
        const size_t n = static_cast<size_t>(cur.row0 + r);
        xv = rope_chunk<kF16>(xv, p.cos + n * 32, p.sin + n * 32, c * 4);
        cur.rot[cur.base + static_cast<size_t>(r) * cur.pitch] = xv;
      }
      add_chunk<kF16>(acc, xv);
    }
    if (nu != u || !more) {
      // the unit is complete: the four row groups (lanes c, c+8, c+16, c+24) meet
      // in a fixed order and lanes 0-7 write the 128-byte mean row
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 8);
        acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 16);
      }
      if (rg == 0 && cur.dst != nullptr) {
        const float n = static_cast<float>(p.bs);
        uint4 o;
        o.x = A::pack(__fdiv_rn(acc[0], n), __fdiv_rn(acc[1], n));
        o.y = A::pack(__fdiv_rn(acc[2], n), __fdiv_rn(acc[3], n));
        o.z = A::pack(__fdiv_rn(acc[4], n), __fdiv_rn(acc[5], n));
        o.w = A::pack(__fdiv_rn(acc[6], n), __fdiv_rn(acc[7], n));
        cur.dst[cur.out] = o;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    }
    if (!more) break;
    u = nu;
    r0 = nr0;
    cur = nxt;
#pragma unroll
    for (int i = 0; i < NR / 4; ++i) x[i] = nx[i];
  }
}

template <bool kF16>
int launch_typed(const PoolParams& p, bool rope, cudaStream_t stream) {
  // Persistent grid: as many 4-warp CTAs as fit on the GPU at once (by registers),
  // never more than there are units.
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return MOSAIC_ERR_CUDA;
  const void* fn = rope ? reinterpret_cast<const void*>(pool_kernel<kF16, true>)
                        : reinterpret_cast<const void*>(pool_kernel<kF16, false>);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kWarpsPerCta * 32, 0) != cudaSuccess || per_sm < 1)
    return MOSAIC_ERR_CUDA;
  const long long need = (p.units + kWarpsPerCta - 1) / kWarpsPerCta;
  const long long ctas = need < static_cast<long long>(sms) * per_sm ? need : static_cast<long long>(sms) * per_sm;
  if (rope)
    pool_kernel<kF16, true><<<static_cast<unsigned>(ctas), kWarpsPerCta * 32, 0, stream>>>(p);
  else
    pool_kernel<kF16, false><<<static_cast<unsigned>(ctas), kWarpsPerCta * 32, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
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
  p.q_cmp = static_cast<uint4*>(a.q_cmp);
  p.k_cmp = static_cast<uint4*>(a.k_cmp);
  p.v_cmp = static_cast<uint4*>(a.v_cmp);
  p.B = a.B;
  p.N = a.N;
  p.Hq = a.Hq;
  p.Hk = a.Hk;
  p.bs = a.bs;
  if (a.bs <= 0) return MOSAIC_ERR_INVALID_ARGUMENT;
  p.nb = a.N / a.bs;
  const bool rope = a.rope_cos != nullptr;
  // With RoPE the rotated q must be produced even when its pooled mean is not needed.
  if (rope && a.q_cmp == nullptr) return MOSAIC_ERR_INVALID_ARGUMENT;
  p.nq = (a.q_cmp != nullptr || rope) ? a.Hq : 0;
  p.nv = a.v_cmp != nullptr ? a.Hk : 0;
  p.slots = p.nq + a.Hk + p.nv;
  p.units = static_cast<long long>(a.B) * p.nb * p.slots;
  if (p.units == 0) return MOSAIC_OK;
  return a.f16 ? launch_typed<true>(p, rope, stream) : launch_typed<false>(p, rope, stream);
}

}  // namespace mosaic
