// The linear projections around the attention op (primitives.MosaicAttention,
// primitives.py:139-209) as one persistent tcgen05 GEMM with two epilogues.
//
//   mode kQkv:   [q | k | v | gate logits] = x W^T for W = cat(to_q, to_k, to_v,
//                to_strategy_combine_mlp) weights, x [S, B, dim] (sequence-first, as
//                MosaicAttention.forward receives it). The epilogue rounds each output
//                to bf16 (the Linear's output dtype), applies Mosaic's 2D RoPE to q
//                and k (RoPE.forward, primitives.py:132-135, same fp32 operation order
//                as pool.cu), softmaxes the gate logits over the three strategies in
//                fp32 (generate_strategy_weights, primitives.py:172-178) and writes
//                q [B, S, Hq, 64], k, v [B, S, Hk, 64] and gates [3, B, S, Hq] bf16:
//                the layouts mosaic_attn_func takes (the rearranges of
//                primitives.py:187-189,175 become epilogue addressing).
//   mode kPlain: out = a W^T for the output projection to_o, with a the attention
//                output [B, S, Hq*64] and out [S, B, dim] (the rearrange of
//                primitives.py:207 is epilogue addressing).
//   mode kLinear: out[m] = rscale[m] * (a[m] W^T), rows kept in place, rscale optional:
//                the Linear layers of CrossAttentionInterpolate (to_kv with the row
//                factor of its RMSNorm folded in, to_o).
//   mode kDown:  HEALPixDownsample (primitives.py:325-329) for one ensemble member b:
//                A rows are coarse pixels n, A columns (f, c) the F children's channels,
//                read straight from x [(n f), B, c] through a 3D tensor map (the
//                rearrange '(n f) b c -> n b (f c)' is addressing); the epilogue rounds
//                proj_x's output to bf16, adds the bf16 proj_pos(rel_pos) row of n,
//                rounds and stores row (n, b).
//   mode kUp:    HEALPixUpsample (primitives.py:352-357): A = x [n, B, c_in] rows (n, b),
//                output column j = (f, d); the epilogue adds the bias row, then the
//                shortcut, rounding after each add as the reference's bf16 ops do, and
//                stores row ((n f), b) (the rearrange 'n b (f d) -> (n f) b d').
//                RMSNorm then runs as rms_apply_kernel over the stored rows (the norm
//                spans several column tiles): one warp per row sums the squares of the
//                stored bf16 values in a fixed order, so the result is deterministic
//                and equals RMSNorm of the bf16 tensor the reference normalises.
//   mode kSwiGLU: the first half of the conditional SwiGLU FFN (cSwiGLU.forward,
//                primitives.py:102-106) with the RMSNorm in front of it
//                (MosaicBlock.norm2, primitives.py:227) folded in as a row factor: the
//                host interleaves w13's rows in blocks of 128 (w1 rows j..j+127, then
//                the w3 rows of the same hidden units), so one 256-column tile holds
//                x1 and x3 of 128 hidden units and the epilogue forms
//                bf16(silu(bf16(x1 + noise[b])) * x3) with every tensor op's bf16
//                rounding; the chunk(2) views and the elementwise passes over them
//                never exist. kLinear with a residual then gives x + w2(h).
//
// Tiles of 128 rows x 256 columns, K in 64-wide stages (TMA, 128-byte swizzle, 4-stage
// ring), fp32 accumulators double-buffered in TMEM so the epilogue of one tile runs
// under the MMAs of the next. Warp 0 loads, warp 1 issues the MMAs (one elected lane of
// a converged warp), warps 4-11 run the epilogue as two warpgroups, each owning 128 of
// the tile's 256 columns, one output row per thread. Every wait is bounded; no TMA
// multicast.
#include <cstring>

#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {
namespace {

constexpr int kPBM = 128, kPBN = 256, kPBK = 64, kPStages = 4;
constexpr int kPThreads = 384;              // warp 0 TMA, warp 1 MMA, warps 2-3 idle, warps 4-11 epilogue
constexpr int kPBox = 64 * 128;             // one 64-row x 64-column bf16 box
constexpr int kPABytes = kPBM * kPBK * 2;   // 16 KB
constexpr int kPBBytes = kPBN * kPBK * 2;   // 32 KB
constexpr int kPStageBytes = kPABytes + kPBBytes;

enum ProjMode : int { kQkv = 0, kPlain = 1, kLinear = 2, kDown = 3, kUp = 4, kSwiGLU = 5 };

struct ProjParams {
  CUtensorMap tm_a, tm_w;
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  __nv_bfloat16* g;        // gates [3, B, S, Hq] or null
  const float* rope_cos;   // [S, 32] or null
  const float* rope_sin;
  __nv_bfloat16* out;      // kPlain, kLinear
  const float* rscale;     // kLinear: per-row factor or null
  const __nv_bfloat16* pos;       // kDown / kUp: [n, N] bias rows
  const __nv_bfloat16* shortcut;  // kUp: [(n f), B, out_dim]; kLinear: residual [M, N]; or null
  const __nv_bfloat16* noise;     // kSwiGLU: [B, hidden] or null
  int hidden;                     // kSwiGLU: output columns (N / 2)
  int out_f16;                    // kPlain / kLinear with a residual: residual and output are fp16
  int F, out_dim, member, c_blocks;
  int a3d;                        // A is the 3D map (c, f, n) of kDown
  int* status;
  int mode;
  int M, K, N;             // GEMM: M rows of A, K, N output columns
  int S, B, Hq, Hk;
  int m_tiles, n_tiles, tiles, k_blocks;
};

struct ProjSmem {
  uint64_t full[kPStages], empty[kPStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

// Per epilogue warp, a 32-row x 64-byte staging area for the bf16 chunk it stores
// (80-byte row pitch: the row-per-lane writes and the 4-lanes-per-row reads are
// bank-conflict-free or nearly so).
constexpr int kStagePitch = 80;
constexpr size_t kStageBytes = 8 * 32 * kStagePitch;
constexpr size_t kProjSmemBytes = 1024 + kPStages * kPStageBytes + ((sizeof(ProjSmem) + 15) / 16) * 16 + kStageBytes;

__device__ __forceinline__ bool wait_noabort_p(uint64_t* bar, uint32_t parity, int* status) {
  int dummy = 0;
  return bounded_wait(bar, parity, &dummy, status);
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Both values rounded to bf16 (nearest even) by one packed conversion: the scalar
// conversion of bf16_round runs on the MUFU / XU pipe, which the SwiGLU epilogue's
// exponentials and reciprocals need; the packed one does not compete for it.
__device__ __forceinline__ void bf16_round2(float& a, float& b) {
  const uint32_t u = pack_bf16x2(a, b);
  a = __uint_as_float(u << 16);
  b = __uint_as_float(u & 0xffff0000u);
}

// 32 consecutive output columns of one row (fp32 accumulators) -> packed bf16 words,
// each scaled by `rs` first (kLinear's row factor; 1 otherwise).
__device__ __forceinline__ void pack_chunk(uint32_t (&packed)[16], const uint32_t (&acc)[32], float rs = 1.0f) {
#pragma unroll
  for (int i = 0; i < 16; ++i)
    packed[i] = pack_bf16x2(__uint_as_float(acc[2 * i]) * rs, __uint_as_float(acc[2 * i + 1]) * rs);
}

// Stores a warp's 32 rows x 32 bf16 columns (row = lane, `packed` its 16 words, `dst`
// its destination or null) through the warp's staging area, so that each store
// instruction writes 64 contiguous bytes of each of 8 rows instead of 16 bytes of each
// of 32 rows. Every lane of the warp must call it.
__device__ __forceinline__ void warp_store_rows(uint8_t* stage, const uint32_t (&packed)[16], __nv_bfloat16* dst,
                                                int lane) {
  uint4* mine = reinterpret_cast<uint4*>(stage + lane * kStagePitch);
#pragma unroll
  for (int i = 0; i < 4; ++i) mine[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
  __syncwarp();
  const int q = lane & 3;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = 8 * k + (lane >> 2);
    const unsigned long long d =
        __shfl_sync(0xffffffffu, static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(dst)), r);
    const uint4 v = *reinterpret_cast<const uint4*>(stage + r * kStagePitch + q * 16);
    if (d != 0ull) reinterpret_cast<uint4*>(static_cast<uintptr_t>(d))[q] = v;
  }
  __syncwarp();  // the stage is rewritten by the next chunk
}

// The bias (and shortcut) words of 32 output columns, loaded before the accumulators
// are read from TMEM so that the two latencies overlap.
__device__ __forceinline__ void load_chunk_res(uint32_t (&pw)[16], uint32_t (&sw)[16], const __nv_bfloat16* pos,
                                               const __nv_bfloat16* sc) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 t = __ldg(reinterpret_cast<const uint4*>(pos) + i);
    pw[4 * i] = t.x; pw[4 * i + 1] = t.y; pw[4 * i + 2] = t.z; pw[4 * i + 3] = t.w;
    const uint4 u = sc != nullptr ? __ldg(reinterpret_cast<const uint4*>(sc) + i) : make_uint4(0, 0, 0, 0);
    sw[4 * i] = u.x; sw[4 * i + 1] = u.y; sw[4 * i + 2] = u.z; sw[4 * i + 3] = u.w;
  }
}

// 32 output columns of one row for kDown / kUp: y = bf16(bf16(acc) + pos) (+ shortcut,
// rounded again) packed as bf16.
__device__ __forceinline__ void pack_chunk_res(uint32_t (&packed)[16], const uint32_t (&acc)[32],
                                               const uint32_t (&pw)[16], const uint32_t (&sw)[16], bool has_sc) {
  const bool sc = has_sc;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float x0 = __uint_as_float(acc[2 * i]), x1 = __uint_as_float(acc[2 * i + 1]);
    bf16_round2(x0, x1);
    x0 += __uint_as_float(pw[i] << 16);
    x1 += __uint_as_float(pw[i] & 0xffff0000u);
    if (sc) {
      bf16_round2(x0, x1);
      x0 += __uint_as_float(sw[i] << 16);
      x1 += __uint_as_float(sw[i] & 0xffff0000u);
    }
    packed[i] = pack_bf16x2(x0, x1);
  }
}

// 16 words (32 bf16 values) of a row segment, zero when src is null. Plain (coherent)
// loads: a kLinear residual may be the output tensor itself.
__device__ __forceinline__ void load_words16(uint32_t (&w)[16], const __nv_bfloat16* src) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 t = src != nullptr ? reinterpret_cast<const uint4*>(src)[i] : make_uint4(0, 0, 0, 0);
    w[4 * i] = t.x; w[4 * i + 1] = t.y; w[4 * i + 2] = t.z; w[4 * i + 3] = t.w;
  }
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// torch's SiLU in fp32 (x / (1 + exp(-x)), the op math of a bf16 tensor), before its
// rounding to bf16. The exponential and the division are the MUFU forms (a few fp32
// ulps, far below the 2^-9 of the rounding that follows); with the accurate library
// forms the epilogue took as long as the tile's MMAs (U-Net step 409 ms against 388 ms).
__device__ __forceinline__ float silu_f32(float t) { return __fdividef(t, 1.0f + __expf(-t)); }

// 32 hidden units of one row for kSwiGLU from the x1 and x3 accumulators:
// bf16(bf16(silu(bf16(bf16(rs a1) + noise))) * bf16(rs a3)).
__device__ __forceinline__ void pack_chunk_swiglu(uint32_t (&packed)[16], const uint32_t (&a1)[32],
                                                  const uint32_t (&a3)[32], const uint32_t (&nw)[16], float rs) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float x1a = __uint_as_float(a1[2 * i]) * rs, x1b = __uint_as_float(a1[2 * i + 1]) * rs;
    float x3a = __uint_as_float(a3[2 * i]) * rs, x3b = __uint_as_float(a3[2 * i + 1]) * rs;
    bf16_round2(x1a, x1b);
    bf16_round2(x3a, x3b);
    float ta = x1a + bf16_lo(nw[i]), tb = x1b + bf16_hi(nw[i]);
    bf16_round2(ta, tb);
    float sa = silu_f32(ta), sb = silu_f32(tb);
    bf16_round2(sa, sb);
    packed[i] = pack_bf16x2(sa * x3a, sb * x3b);
  }
}

// 32 output columns of one row for kLinear / kPlain with a residual, in the residual's
// 16-bit type T (bf16, or fp16 for a residual stream under fp16 autocast, where the
// Linear's output is fp16): T(T(rs acc) + res).
template <bool kF16>
__device__ __forceinline__ void pack_chunk_residual(uint32_t (&packed)[16], const uint32_t (&acc)[32],
                                                    const uint32_t (&rw)[16], float rs) {
  using T = Act<kF16>;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 y = T::unpack(T::pack(__uint_as_float(acc[2 * i]) * rs, __uint_as_float(acc[2 * i + 1]) * rs));
    const float2 r = T::unpack(rw[i]);
    packed[i] = T::pack(y.x + r.x, y.y + r.y);
  }
}

// RMSNorm of 16-bit rows into bf16 rows: y = bf16(x * rsqrt(mean(x^2) + eps) (* w)), one
// warp per row, x bf16 (kF16In false; in place when y == x, the resampling layers) or
// fp16 (a Mosaic block under fp16 autocast, whose residual stream is fp16), the same fp32
// arithmetic as torch.nn.RMSNorm. The sum of squares is taken over the input values,
// each lane over its 16-byte chunks in order and the lanes by a fixed butterfly, so it is
// deterministic.
template <bool kF16In>
__global__ void __launch_bounds__(256) rms_apply_kernel(const uint16_t* x, __nv_bfloat16* y,
                                                        const float* __restrict__ w, long long rows, int D, float eps) {
  using In = Act<kF16In>;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint16_t* xr = x + row * D;
  __nv_bfloat16* yr = y + row * D;
  float ss = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = In::unpack(wd[i]);
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / static_cast<float>(D) + eps);
  for (int c = lane * 8; c < D; c += 256) {
    uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    uint32_t wd[4] = {v.x, v.y, v.z, v.w};
    float wt[8];
    if (w != nullptr) {
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + c)), w1 = __ldg(reinterpret_cast<const float4*>(w + c) + 1);
      wt[0] = w0.x; wt[1] = w0.y; wt[2] = w0.z; wt[3] = w0.w; wt[4] = w1.x; wt[5] = w1.y; wt[6] = w1.z; wt[7] = w1.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) wt[i] = 1.f;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = In::unpack(wd[i]);
      wd[i] = pack_bf16x2(f.x * r * wt[2 * i], f.y * r * wt[2 * i + 1]);
    }
    *reinterpret_cast<uint4*>(yr + c) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  }
}

// 16 RoPE frequencies p0 .. p0 + 15 of one table row (four 16-byte loads of each table).
__device__ __forceinline__ void load_rope16(float (&cs)[16], float (&sn)[16], const float* cos_row,
                                            const float* sin_row, int p0) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 c = __ldg(reinterpret_cast<const float4*>(cos_row + p0) + i);
    const float4 t = __ldg(reinterpret_cast<const float4*>(sin_row + p0) + i);
    cs[4 * i] = c.x; cs[4 * i + 1] = c.y; cs[4 * i + 2] = c.z; cs[4 * i + 3] = c.w;
    sn[4 * i] = t.x; sn[4 * i + 1] = t.y; sn[4 * i + 2] = t.z; sn[4 * i + 3] = t.w;
  }
}

// 32 output columns of one row -> packed bf16, rotated by RoPE with the chunk's table
// values already in registers (rot). The reference rounds the Linear output to bf16
// first, then rotates in fp32: out[2i] = x[2i] cos - x[2i+1] sin and out[2i+1] =
// x[2i+1] cos + x[2i] sin, each product and the sum rounded.
__device__ __forceinline__ void pack_chunk_tab(uint32_t (&packed)[16], const uint32_t (&acc)[32],
                                               const float (&cs)[16], const float (&sn)[16], bool rot) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float x0 = __uint_as_float(acc[2 * i]), x1 = __uint_as_float(acc[2 * i + 1]);
    bf16_round2(x0, x1);
    if (rot) {
      const float o0 = __fadd_rn(__fmul_rn(x0, cs[i]), __fmul_rn(-x1, sn[i]));
      const float o1 = __fadd_rn(__fmul_rn(x1, cs[i]), __fmul_rn(x0, sn[i]));
      x0 = o0;
      x1 = o1;
    }
    packed[i] = pack_bf16x2(x0, x1);
  }
}

// One instantiation per mode, so that each epilogue gets its own register allocation.
template <int kMode>
__global__ void __launch_bounds__(kPThreads, 1) proj_kernel(const __grid_constant__ ProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  ProjSmem& sm = *reinterpret_cast<ProjSmem*>(tiles + kPStages * kPStageBytes);
  uint8_t* stage_all = tiles + kPStages * kPStageBytes + ((sizeof(ProjSmem) + 15) / 16) * 16;
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm.acc_full[a], 1);
      mbar_init(&sm.acc_empty[a], 256);
    }
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x) {
      const int mt = t / p.n_tiles, nt = t % p.n_tiles;
      for (int kb = 0; kb < p.k_blocks; ++kb, ++g) {
        const int st = g % kPStages, r = g / kPStages;
        if (r > 0 && !warp_wait(&sm.empty[st], (r - 1) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        uint8_t* sa = tiles + st * kPStageBytes;
        uint8_t* sb = sa + kPABytes;
        mbar_arrive_expect_tx_elect(&sm.full[st], kPStageBytes);
        if (p.a3d) {
          const int f = kb / p.c_blocks, c = (kb - f * p.c_blocks) * kPBK;
          for (int i = 0; i < 2; ++i) tma_load_3d_elect(sa + i * kPBox, &p.tm_a, &sm.full[st], c, f, mt * kPBM + 64 * i);
        } else {
          for (int i = 0; i < 2; ++i)
            tma_load_2d_elect(sa + i * kPBox, &p.tm_a, &sm.full[st], kb * kPBK, mt * kPBM + 64 * i);
        }
        for (int i = 0; i < 4; ++i) tma_load_2d_elect(sb + i * kPBox, &p.tm_w, &sm.full[st], kb * kPBK, nt * kPBN + 64 * i);
      }
    }
    if (lane == 0) {
      for (int s = 0; s < kPStages && s < g; ++s) {
        const int g_last = s + kPStages * ((g - 1 - s) / kPStages);
        wait_noabort_p(&sm.full[s], (g_last / kPStages) & 1, p.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    const uint32_t idesc = make_idesc_bf16(kPBM, kPBN, false);
    const uint32_t sbase = smem_u32(tiles);
    int g = 0, it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, ++it) {
      const int a = it & 1;
      // The epilogue must have read this accumulator's previous tile.
      if (it >= 2) ok = warp_wait(&sm.acc_empty[a], ((it >> 1) - 1) & 1, abort_flag, p.status);
      tc_fence_after();
      for (int kb = 0; ok && kb < p.k_blocks; ++kb, ++g) {
        const int st = g % kPStages;
        if (!warp_wait(&sm.full[st], (g / kPStages) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = sw128_desc(sbase + st * kPStageBytes, 1024, 16);
        const uint64_t bd = sw128_desc(sbase + st * kPStageBytes + kPABytes, 1024, 16);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_ss_elect(tmem + 256u * a, ad + static_cast<uint64_t>(2 * ks), bd + static_cast<uint64_t>(2 * ks), idesc,
                       (kb > 0 || ks > 0) ? 1u : 0u);
        tc_commit_elect(&sm.empty[st]);
      }
      if (!ok) break;
      tc_commit_elect(&sm.acc_full[a]);
    }
    tc_commit_elect(&sm.drain);
    if (lane == 0) wait_noabort_p(&sm.drain, 0, p.status);
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- epilogue, one output row per thread
    const int half = (warp - 4) >> 2;  // warpgroup: columns [128 half, 128 half + 128) of each tile
    const int row = (warp & 3) * 32 + lane;
    uint8_t* stage = stage_all + (warp - 4) * 32 * kStagePitch;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int qcols = p.Hq * 64, kcols = p.Hk * 64;
    const int gbase = qcols + 2 * kcols;  // first gate-logit column (kQkv)
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, ++it) {
      const int a = it & 1;
      const int mt = t / p.n_tiles, nt = t % p.n_tiles;
      const int m = mt * kPBM + row;
      const bool live = m < p.M;
      const uint32_t tacc = tmem + lane_off + 256u * a;
      if constexpr (kMode == kSwiGLU) {
        // Tile nt holds x1 of hidden units [128 nt, 128 nt + 128) in columns 0-127 and x3
        // of the same units in columns 128-255; warpgroup `half` forms units
        // j0 + [0, 64), two chunks of 32. Rows are (s, b): member b = m % B.
        const int j0 = nt * 128 + 64 * half;
        const float rs = live && p.rscale != nullptr ? __ldg(p.rscale + m) : 1.0f;
        const __nv_bfloat16* nrow =
            live && p.noise != nullptr ? p.noise + static_cast<size_t>(m % p.B) * p.hidden + j0 : nullptr;
        uint32_t nw[2][16];
        load_words16(nw[0], nrow);
        load_words16(nw[1], nrow != nullptr ? nrow + 32 : nullptr);
        if (!bounded_wait(&sm.acc_full[a], (it >> 1) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          uint32_t a1[32], a3[32];
          tmem_ld32(tacc + 64 * half + 32 * k, a1);
          tmem_ld32(tacc + 128 + 64 * half + 32 * k, a3);
          tmem_ld_wait();
          reg_fence<32>(a1);
          reg_fence<32>(a3);
          uint32_t packed[16];
          pack_chunk_swiglu(packed, a1, a3, nw[k], rs);
          warp_store_rows(stage, packed, live ? p.out + static_cast<size_t>(m) * p.hidden + j0 + 32 * k : nullptr,
                          lane);
        }
        tc_fence_before();
        mbar_arrive(&sm.acc_empty[a]);
        continue;
      }
      if constexpr (kMode == kDown || kMode == kUp) {
        // The warpgroup's (up to) 4 chunks of 32 columns lie in one child block f
        // (out_dim % 128 == 0), so the output row and the bias row are fixed for the
        // tile. The bias / shortcut words of chunk k + 1 load while chunk k is stored,
        // and those of chunk 0 while the MMAs of this tile finish.
        const int cbase = nt * kPBN + 128 * half;
        const int nch = cbase >= p.N ? 0 : min(4, (p.N - cbase) / 32);
        const int n = kMode == kDown ? m : m / p.B;
        const int f = kMode == kDown ? 0 : cbase / p.out_dim;
        const long long orow = kMode == kDown ? static_cast<long long>(m) * p.B + p.member
                                              : (static_cast<long long>(n) * p.F + f) * p.B + (m - n * p.B);
        const size_t o0 = static_cast<size_t>(orow) * p.out_dim + (cbase - f * p.out_dim);
        const __nv_bfloat16* pos0 = p.pos + static_cast<size_t>(n) * p.N + cbase;
        const __nv_bfloat16* sc0 = p.shortcut != nullptr ? p.shortcut + o0 : nullptr;
        uint32_t pw[2][16], sw[2][16];
        if (live && nch > 0) load_chunk_res(pw[0], sw[0], pos0, sc0);
        if (!bounded_wait(&sm.acc_full[a], (it >> 1) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (k >= nch) break;
          if (live && k + 1 < nch)
            load_chunk_res(pw[(k + 1) & 1], sw[(k + 1) & 1], pos0 + 32 * (k + 1),
                           sc0 != nullptr ? sc0 + 32 * (k + 1) : nullptr);
          uint32_t acc[32];
          tmem_ld32(tacc + 32 * (4 * half + k), acc);
          tmem_ld_wait();
          reg_fence<32>(acc);
          uint32_t packed[16];
          pack_chunk_res(packed, acc, pw[k & 1], sw[k & 1], sc0 != nullptr);
          warp_store_rows(stage, packed, live ? p.out + o0 + 32 * k : nullptr, lane);
        }
        tc_fence_before();
        mbar_arrive(&sm.acc_empty[a]);
        continue;
      }
      if (!bounded_wait(&sm.acc_full[a], (it >> 1) & 1, abort_flag, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // kQkv visits the warpgroup's chunks in the order 0, 2, 1, 3: chunks 0 and 2 rotate
      // with RoPE frequencies 0-15 and chunks 1 and 3 with 16-31 (d0 = 0 or 32 of a head),
      // so each half of the row's table is loaded once per tile instead of twice.
      float cs[16], sn[16];
      int tab_p0 = -1;
#pragma unroll 1
      for (int k = 0; k < 4; ++k) {
        const int ci = 4 * half + (kMode == kQkv ? (k & 1) * 2 + (k >> 1) : k);
        const int c0 = nt * kPBN + 32 * ci;  // warp-uniform
        if (c0 >= p.N) {
          if (kMode == kQkv) continue;
          break;
        }
        if (kMode == kQkv && c0 == gbase + 32) continue;  // second gate chunk: taken with the first
        uint32_t acc[32];
        if (kMode == kPlain) {
          // A rows are (b, s) (attention output), out rows (s, b)
          const int b = m / p.S, s = m % p.S;
          const size_t o = (static_cast<size_t>(s) * p.B + b) * p.N + c0;
          uint32_t rw[16];
          if (p.shortcut != nullptr) load_words16(rw, live ? p.shortcut + o : nullptr);
          tmem_ld32(tacc + 32 * ci, acc);
          tmem_ld_wait();
          reg_fence<32>(acc);
          uint32_t packed[16];
          if (p.shortcut != nullptr && p.out_f16)
            pack_chunk_residual<true>(packed, acc, rw, 1.0f);
          else if (p.shortcut != nullptr)
            pack_chunk_residual<false>(packed, acc, rw, 1.0f);
          else
            pack_chunk(packed, acc);
          warp_store_rows(stage, packed, live ? p.out + o : nullptr, lane);
          continue;
        }
        if (kMode == kLinear) {
          const float rs = live && p.rscale != nullptr ? __ldg(p.rscale + m) : 1.0f;
          uint32_t rw[16];
          if (p.shortcut != nullptr) load_words16(rw, live ? p.shortcut + static_cast<size_t>(m) * p.N + c0 : nullptr);
          tmem_ld32(tacc + 32 * ci, acc);
          tmem_ld_wait();
          reg_fence<32>(acc);
          uint32_t packed[16];
          if (p.shortcut != nullptr && p.out_f16)
            pack_chunk_residual<true>(packed, acc, rw, rs);
          else if (p.shortcut != nullptr)
            pack_chunk_residual<false>(packed, acc, rw, rs);
          else
            pack_chunk(packed, acc, rs);
          // with a residual the output may alias it: every lane of the warp has read its
          // residual words before warp_store_rows writes any row
          warp_store_rows(stage, packed, live ? p.out + static_cast<size_t>(m) * p.N + c0 : nullptr, lane);
          continue;
        }
        const int s = m / p.B, b = m % p.B;  // x rows are (s, b)
        if (c0 < gbase) {
          tmem_ld32(tacc + 32 * ci, acc);
          tmem_ld_wait();
          reg_fence<32>(acc);
          __nv_bfloat16* dst;
          bool rot = false;
          int d0;
          if (c0 < qcols) {
            d0 = c0 % 64;
            dst = p.q + ((static_cast<size_t>(b) * p.S + s) * p.Hq + c0 / 64) * 64 + d0;
            rot = p.rope_cos != nullptr;
          } else if (c0 < qcols + kcols) {
            d0 = (c0 - qcols) % 64;
            dst = p.k + ((static_cast<size_t>(b) * p.S + s) * p.Hk + (c0 - qcols) / 64) * 64 + d0;
            rot = p.rope_cos != nullptr;
          } else {
            d0 = (c0 - qcols - kcols) % 64;
            dst = p.v + ((static_cast<size_t>(b) * p.S + s) * p.Hk + (c0 - qcols - kcols) / 64) * 64 + d0;
          }
          if (rot && live && tab_p0 != d0 / 2) {
            load_rope16(cs, sn, p.rope_cos + static_cast<size_t>(s) * 32, p.rope_sin + static_cast<size_t>(s) * 32,
                        d0 / 2);
            tab_p0 = d0 / 2;
          }
          uint32_t packed[16];
          pack_chunk_tab(packed, acc, cs, sn, rot && live);
          warp_store_rows(stage, packed, live ? dst : nullptr, lane);
        } else if (c0 == gbase) {
          // The 3 Hq gate logits (at most 64 columns, starting 64-aligned, so inside this
          // tile): logits are bf16 Linear outputs laid out (head, strategy); softmax over
          // the three strategies in fp32, rounded to bf16.
          uint32_t hi[32];
          tmem_ld32(tacc + 32 * ci, acc);
          tmem_ld32(tacc + 32 * ci + 32, hi);
          tmem_ld_wait();
          reg_fence<32>(acc);
          reg_fence<32>(hi);
          if (live && p.g != nullptr) {
#pragma unroll
            for (int h = 0; h < 21; ++h) {
              if (h >= p.Hq) break;
              float l[3];
#pragma unroll
              for (int j = 0; j < 3; ++j) {
                const int e = 3 * h + j;
                l[j] = bf16_round(__uint_as_float(e < 32 ? acc[e & 31] : hi[(e - 32) & 31]));
              }
              const float mx = fmaxf(fmaxf(l[0], l[1]), l[2]);
              const float e0 = expf(l[0] - mx), e1 = expf(l[1] - mx), e2 = expf(l[2] - mx);
              const float sum = e0 + e1 + e2;
              const size_t plane = static_cast<size_t>(p.B) * p.S * p.Hq;
              const size_t o = (static_cast<size_t>(b) * p.S + s) * p.Hq + h;
              p.g[o] = __float2bfloat16_rn(e0 / sum);
              p.g[plane + o] = __float2bfloat16_rn(e1 / sum);
              p.g[2 * plane + o] = __float2bfloat16_rn(e2 / sum);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.acc_empty[a]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int sm_count_p() {
  static int count[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (count[dev] == 0 && cudaDeviceGetAttribute(&count[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  return count[dev];
}

template <int kMode>
int set_proj_smem(int dev) {
  static bool done[64] = {};
  if (!done[dev]) {
    if (cudaFuncSetAttribute(proj_kernel<kMode>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kProjSmemBytes)) != cudaSuccess)
      return MOSAIC_ERR_CUDA;
    done[dev] = true;
  }
  return MOSAIC_OK;
}

template <int kMode>
void launch_proj_mode(const ProjParams& p, int grid, cudaStream_t stream) {
  proj_kernel<kMode><<<grid, kPThreads, kProjSmemBytes, stream>>>(p);
}

int launch_proj(ProjParams& p, cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOSAIC_ERR_CUDA;
  int rc = MOSAIC_ERR_INVALID_ARGUMENT;
  switch (p.mode) {
    case kQkv: rc = set_proj_smem<kQkv>(dev); break;
    case kPlain: rc = set_proj_smem<kPlain>(dev); break;
    case kLinear: rc = set_proj_smem<kLinear>(dev); break;
    case kDown: rc = set_proj_smem<kDown>(dev); break;
    case kUp: rc = set_proj_smem<kUp>(dev); break;
    case kSwiGLU: rc = set_proj_smem<kSwiGLU>(dev); break;
  }
  if (rc != MOSAIC_OK) return rc;
  const int sms = sm_count_p();
  if (sms <= 0) return MOSAIC_ERR_CUDA;
  p.m_tiles = (p.M + kPBM - 1) / kPBM;
  p.n_tiles = (p.N + kPBN - 1) / kPBN;
  p.tiles = p.m_tiles * p.n_tiles;
  p.k_blocks = p.K / kPBK;
  const int grid = p.tiles < sms ? p.tiles : sms;
  if (grid > 0) {
    switch (p.mode) {
      case kQkv: launch_proj_mode<kQkv>(p, grid, stream); break;
      case kPlain: launch_proj_mode<kPlain>(p, grid, stream); break;
      case kLinear: launch_proj_mode<kLinear>(p, grid, stream); break;
      case kDown: launch_proj_mode<kDown>(p, grid, stream); break;
      case kUp: launch_proj_mode<kUp>(p, grid, stream); break;
      case kSwiGLU: launch_proj_mode<kSwiGLU>(p, grid, stream); break;
    }
  }
  return cudaGetLastError() == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

}  // namespace

int launch_qkv_proj(const QkvProjLaunch& a, cudaStream_t stream) {
  ProjParams p;
  memset(&p, 0, sizeof(p));
  const int n = (a.Hq + 2 * a.Hk) * 64 + (a.gates ? 3 * a.Hq : 0);
  if (make_tmap_bf16_2d(&p.tm_a, a.x, static_cast<uint64_t>(a.S) * a.B, static_cast<uint64_t>(a.dim)) ||
      make_tmap_bf16_2d(&p.tm_w, a.w, static_cast<uint64_t>(n), static_cast<uint64_t>(a.dim)))
    return MOSAIC_ERR_CUDA;
  p.q = static_cast<__nv_bfloat16*>(a.q);
  p.k = static_cast<__nv_bfloat16*>(a.k);
  p.v = static_cast<__nv_bfloat16*>(a.v);
  p.g = static_cast<__nv_bfloat16*>(a.gates);
  p.rope_cos = a.rope_cos;
  p.rope_sin = a.rope_sin;
  p.status = a.status;
  p.mode = kQkv;
  p.M = a.S * a.B;
  p.K = a.dim;
  p.N = n;
  p.S = a.S;
  p.B = a.B;
  p.Hq = a.Hq;
  p.Hk = a.Hk;
  return launch_proj(p, stream);
}

int launch_linear(const LinearLaunch& a, cudaStream_t stream) {
  ProjParams p;
  memset(&p, 0, sizeof(p));
  if (make_tmap_bf16_2d(&p.tm_a, a.a, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.K)) ||
      make_tmap_bf16_2d(&p.tm_w, a.w, static_cast<uint64_t>(a.N), static_cast<uint64_t>(a.K)))
    return MOSAIC_ERR_CUDA;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.rscale = a.rscale;
  p.shortcut = static_cast<const __nv_bfloat16*>(a.residual);
  p.out_f16 = a.out_f16;
  p.status = a.status;
  p.mode = kLinear;
  p.M = a.M;
  p.K = a.K;
  p.N = a.N;
  return launch_proj(p, stream);
}

int launch_swiglu(const SwigluLaunch& a, cudaStream_t stream) {
  ProjParams p;
  memset(&p, 0, sizeof(p));
  if (make_tmap_bf16_2d(&p.tm_a, a.x, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.dim)) ||
      make_tmap_bf16_2d(&p.tm_w, a.w13, static_cast<uint64_t>(2) * a.hidden, static_cast<uint64_t>(a.dim)))
    return MOSAIC_ERR_CUDA;
  p.out = static_cast<__nv_bfloat16*>(a.h);
  p.rscale = a.rscale;
  p.noise = static_cast<const __nv_bfloat16*>(a.noise);
  p.status = a.status;
  p.mode = kSwiGLU;
  p.M = a.M;
  p.K = a.dim;
  p.N = 2 * a.hidden;
  p.hidden = a.hidden;
  p.B = a.B;
  return launch_proj(p, stream);
}

int launch_rms_apply(void* y, const float* w, long long rows, int D, float eps, cudaStream_t stream) {
  return launch_rms_norm(y, y, w, rows, D, eps, false, stream);
}

int launch_rms_norm(const void* x, void* y, const float* w, long long rows, int D, float eps, bool x_f16,
                    cudaStream_t stream) {
  if (rows == 0) return MOSAIC_OK;
  const unsigned grid = static_cast<unsigned>((rows * 32 + 255) / 256);
  if (x_f16)
    rms_apply_kernel<true><<<grid, 256, 0, stream>>>(static_cast<const uint16_t*>(x), static_cast<__nv_bfloat16*>(y),
                                                     w, rows, D, eps);
  else
    rms_apply_kernel<false><<<grid, 256, 0, stream>>>(static_cast<const uint16_t*>(x), static_cast<__nv_bfloat16*>(y),
                                                      w, rows, D, eps);
  return cudaGetLastError() == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int launch_healpix_down(const UpDownLaunch& a, cudaStream_t stream) {
  const long long rows = static_cast<long long>(a.n) * a.B;
  if (rows == 0) return MOSAIC_OK;
  for (int b = 0; b < a.B; ++b) {  // one GEMM per member: A = member b's children, read in place
    ProjParams p;
    memset(&p, 0, sizeof(p));
    const uint64_t row_bytes = static_cast<uint64_t>(a.B) * a.c_in * 2;
    if (make_tmap_bf16_3d(&p.tm_a, static_cast<const __nv_bfloat16*>(a.x) + static_cast<size_t>(b) * a.c_in,
                          static_cast<uint64_t>(a.c_in), static_cast<uint64_t>(a.F), static_cast<uint64_t>(a.n),
                          row_bytes, row_bytes * a.F) ||
        make_tmap_bf16_2d(&p.tm_w, a.w, static_cast<uint64_t>(a.c_out), static_cast<uint64_t>(a.F) * a.c_in))
      return MOSAIC_ERR_CUDA;
    p.a3d = 1;
    p.c_blocks = a.c_in / kPBK;
    p.out = static_cast<__nv_bfloat16*>(a.out);
    p.pos = static_cast<const __nv_bfloat16*>(a.pos);
    p.status = a.status;
    p.mode = kDown;
    p.M = a.n;
    p.K = a.F * a.c_in;
    p.N = a.c_out;
    p.B = a.B;
    p.F = a.F;
    p.out_dim = a.c_out;
    p.member = b;
    const int rc = launch_proj(p, stream);
    if (rc != MOSAIC_OK) return rc;
  }
  return launch_rms_apply(a.out, a.norm_w, rows, a.c_out, a.eps, stream);
}

int launch_healpix_up(const UpDownLaunch& a, cudaStream_t stream) {
  const long long rows = static_cast<long long>(a.n) * a.F * a.B;
  if (rows == 0) return MOSAIC_OK;
  ProjParams p;
  memset(&p, 0, sizeof(p));
  if (make_tmap_bf16_2d(&p.tm_a, a.x, static_cast<uint64_t>(a.n) * a.B, static_cast<uint64_t>(a.c_in)) ||
      make_tmap_bf16_2d(&p.tm_w, a.w, static_cast<uint64_t>(a.F) * a.c_out, static_cast<uint64_t>(a.c_in)))
    return MOSAIC_ERR_CUDA;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.pos = static_cast<const __nv_bfloat16*>(a.pos);
  p.shortcut = static_cast<const __nv_bfloat16*>(a.shortcut);
  p.status = a.status;
  p.mode = kUp;
  p.M = a.n * a.B;
  p.K = a.c_in;
  p.N = a.F * a.c_out;
  p.B = a.B;
  p.F = a.F;
  p.out_dim = a.c_out;
  const int rc = launch_proj(p, stream);
  if (rc != MOSAIC_OK) return rc;
  return launch_rms_apply(a.out, a.norm_w, rows, a.c_out, a.eps, stream);
}

int launch_out_proj(const OutProjLaunch& a, cudaStream_t stream) {
  ProjParams p;
  memset(&p, 0, sizeof(p));
  const int kdim = a.Hq * 64;
  if (make_tmap_bf16_2d(&p.tm_a, a.attn, static_cast<uint64_t>(a.S) * a.B, static_cast<uint64_t>(kdim)) ||
      make_tmap_bf16_2d(&p.tm_w, a.w, static_cast<uint64_t>(a.dim), static_cast<uint64_t>(kdim)))
    return MOSAIC_ERR_CUDA;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.shortcut = static_cast<const __nv_bfloat16*>(a.residual);
  p.out_f16 = a.out_f16;
  p.status = a.status;
  p.mode = kPlain;
  p.M = a.S * a.B;
  p.K = kdim;
  p.N = a.dim;
  p.S = a.S;
  p.B = a.B;
  p.Hq = a.Hq;
  return launch_proj(p, stream);
}

}  // namespace mosaic
