// Fused block-sparse attention engine for sm_100a (tcgen05 + TMEM + TMA).
//
// One CTA owns one (batch b, kv head h, 64-query tile) and all G = 4 query heads
// of that kv group. The four heads are packed into two M = 128 MMA tiles
// ("M-tiles": rows 0-63 = head 4h+2m, rows 64-127 = head 4h+2m+1), so every K/V
// tile that TMA brings into shared memory is used by 4 heads x 64 queries.
// Keys stream in tiles of 128 (two 64-row TMA boxes):
//   * local branch   (primitives.block_attention, primitives.py:28-32): the
//     window [w*win, (w+1)*win) that contains the query tile;
//   * selected branch (ops.mosaic_attn_fwd_kernel, ops.py:94-128): the 64-row
//     segments of blocks block_idx[b, n/bs, h, 0..K-1].
// Each branch keeps its own online-softmax state and its own TMEM accumulator,
// because the reference combines three separately normalised softmaxes
// linearly (primitives.py:89). The epilogue applies the gates and adds the
// coarse-attention row o_cmp[b, n/bs, head] (the repeat_interleave of
// primitives.py:78 becomes an index).
//
// Warp roles (320 threads): warp 0 issues TMA, warp 1 issues tcgen05.mma (one
// thread) and owns the TMEM allocation, warps 2-5 run the softmax + epilogue of
// M-tile 0 and warps 6-9 those of M-tile 1. The two M-tiles ping-pong on the
// tensor core: while one softmax warpgroup turns S into P, the MMA warp runs
// the other M-tile's P*V and Q*K^T.
//
// TMEM (512 columns, fp32): S/P of M-tile m at [128m, 128m+128) (P overwrites the
// first 64 columns of S as packed bf16 pairs), O_local of M-tile m at
// 256+128m, O_selected at 320+128m.
#include <cmath>
#include <cstring>

#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {
namespace {

constexpr int kQTile = 64;
constexpr int kStages = 4;
constexpr int kSegBytes = 64 * 128;       // one 64-row x 64-col bf16 box
constexpr int kTileBytes = 2 * kSegBytes;  // 128 rows
constexpr int kThreads = 320;
constexpr int kMaxSel = 1024;  // max selected blocks per query block
constexpr float kRescaleThreshold = 8.0f;  // log2 units: keep a stale max while p <= 2^8

struct EngineParams {
  CUtensorMap tm_q, tm_k, tm_v;
  const int64_t* block_idx;
  const __nv_bfloat16* gates;
  const __nv_bfloat16* o_cmp;
  __nv_bfloat16* out;
  float* lse;
  int* status;
  int B, Nq, Nk, Hq, Hk;
  int win, bs, K, nqb, nkb;
  int combine;
  float scale_log2;
};

struct EngineSmem {
  uint64_t q_full;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_final[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int sel[kMaxSel];
};

constexpr size_t kSmemBytes = 1024 /*align slack*/ + 2 * kTileBytes + 2 * kStages * kTileBytes + sizeof(EngineSmem);

// Geometry of key tile t (shared by the producer, the MMA issuer and the softmax).
struct KeyTile {
  int nseg;   // 1 or 2 boxes of 64 keys
  int valid;  // keys in the tile that take part (<= 64*nseg)
  int row0, row1;  // key rows (within the batch) of the two boxes
};

__device__ __forceinline__ KeyTile key_tile(const EngineParams& p, const int* sel, int t, int T_loc, int wstart,
                                            int wend) {
  KeyTile kt;
  if (t < T_loc) {
    const int start = wstart + t * 128;
    kt.valid = min(128, wend - start);
    kt.row0 = start;
    kt.row1 = start + 64;
  } else {
    const int pos = (t - T_loc) * 128;
    const int total = p.K * p.bs;
    kt.valid = min(128, total - pos);
    kt.row0 = sel[pos / p.bs] * p.bs + pos % p.bs;
    const int pos1 = pos + 64;
    kt.row1 = pos1 < total ? sel[pos1 / p.bs] * p.bs + pos1 % p.bs : 0;
  }
  kt.nseg = kt.valid > 64 ? 2 : 1;
  return kt;
}

// Online-softmax step for one 128-row S tile held in TMEM: each thread owns one
// row. Reads NK scores, updates (m_run, l_run), rescales this row's O accumulator
// when the running max grows by more than kRescaleThreshold, and writes
// P = exp2(S*c - m) as packed bf16 pairs over the first NK/2 columns of S.
template <int NK>
__device__ __forceinline__ void softmax_tile(uint32_t tS, uint32_t tO, int valid, bool first, float c,
                                             float& m_run, float& l_run) {
  uint32_t s[NK];
#pragma unroll
  for (int i = 0; i < NK / 32; ++i) tmem_ld32(tS + 32 * i, s + 32 * i);
  tmem_ld_wait();
  reg_fence<NK>(s);
  if (valid < NK) {
#pragma unroll
    for (int i = 0; i < NK; ++i)
      if (i >= valid) s[i] = __float_as_uint(-INFINITY);
  }
  float mx0 = __uint_as_float(s[0]), mx1 = __uint_as_float(s[1]);
#pragma unroll
  for (int i = 2; i < NK; i += 2) {
    mx0 = fmaxf(mx0, __uint_as_float(s[i]));
    mx1 = fmaxf(mx1, __uint_as_float(s[i + 1]));
  }
  const float m_new = fmaxf(m_run, fmaxf(mx0, mx1) * c);
  float m_use = m_run, alpha = 1.0f;
  bool need = false;
  if (first) {
    m_use = m_new;
  } else if (m_new > m_run + kRescaleThreshold) {
    need = true;
    m_use = m_new;
    alpha = ex2_approx(m_run - m_new);
  }
  if (__any_sync(0xffffffffu, need)) {
    // Rare path; 8 columns at a time so that the 128 live scores do not spill.
#pragma unroll 1
    for (int c8 = 0; c8 < 64; c8 += 8) {
      uint32_t o[8];
      tmem_ld8(tO + c8, o);
      tmem_ld_wait();
      reg_fence<8>(o);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
      tmem_st8(tO + c8, o);
    }
  }
  l_run *= alpha;
  const float nm = -m_use;
  float sum0 = 0.f, sum1 = 0.f;
  // P pairs are packed in place over the scores they came from (s[i] <- s[2i], s[2i+1]).
#pragma unroll
  for (int i = 0; i < NK / 2; ++i) {
    const float p0 = ex2_approx(fmaf(__uint_as_float(s[2 * i]), c, nm));
    const float p1 = ex2_approx(fmaf(__uint_as_float(s[2 * i + 1]), c, nm));
    sum0 += p0;
    sum1 += p1;
    s[i] = pack_bf16x2(p0, p1);
  }
#pragma unroll
  for (int h = 0; h < NK / 64; ++h) tmem_st32(tS + 32 * h, s + 32 * h);
  tmem_st_wait();
  l_run += sum0 + sum1;
  m_run = m_use;
}

__device__ __forceinline__ bool wait_noabort(uint64_t* bar, uint32_t parity, int* status) {
  int dummy = 0;
  return bounded_wait(bar, parity, &dummy, status);
}

__global__ void __launch_bounds__(kThreads, 1) bsa_engine_kernel(const __grid_constant__ EngineParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = tiles;
  uint8_t* sK = tiles + 2 * kTileBytes;
  uint8_t* sV = sK + kStages * kTileBytes;
  EngineSmem& sm = *reinterpret_cast<EngineSmem*>(sV + kStages * kTileBytes);
  volatile int* abort_flag = &sm.abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int n0 = qt * kQTile;
  const int G = p.Hq / p.Hk;

  int T_loc = 0, wstart = 0, wend = 0;
  if (p.win > 0) {
    wstart = (n0 / p.win) * p.win;
    wend = min(wstart + p.win, p.Nk);
    T_loc = (wend - wstart + 127) / 128;
  }
  const int T_slc = p.K > 0 ? (p.K * p.bs + 127) / 128 : 0;
  const int T = T_loc + T_slc;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int m = 0; m < 2; ++m) {
      mbar_init(&sm.s_full[m], 1);
      mbar_init(&sm.p_full[m], 128);
      mbar_init(&sm.o_final[m], 1);
    }
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && p.K > 0) {
    // Stage this query block's selected kv blocks; out-of-range entries are
    // reported and clamped so that no load leaves the batch.
    const int qb = n0 / p.bs;
    const int64_t* src = p.block_idx + ((static_cast<int64_t>(b) * p.nqb + qb) * p.Hk + h) * p.K;
    for (int s = lane; s < p.K; s += 32) {
      int64_t v = src[s];
      if (v < 0 || v >= p.nkb) {
        if (p.status) atomicOr(p.status, MOSAIC_STATUS_BAD_INDEX);
        v = 0;
      }
      sm.sel[s] = static_cast<int>(v);
    }
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
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_k);
      prefetch_tmap(&p.tm_v);
      mbar_arrive_expect_tx(&sm.q_full, 4 * kSegBytes);
      for (int m = 0; m < 2; ++m)
        for (int u = 0; u < 2; ++u)
          tma_load_2d(sQ + m * kTileBytes + u * kSegBytes, &p.tm_q, &sm.q_full, (h * G + 2 * m + u) * 64,
                      b * p.Nq + n0);
      int issued = 0;
      for (int t = 0; t < T; ++t) {
        const int st = t % kStages, r = t / kStages;
        if (r > 0 && !bounded_wait(&sm.kv_empty[st], (r - 1) & 1, abort_flag, p.status)) break;
        const KeyTile kt = key_tile(p, sm.sel, t, T_loc, wstart, wend);
        mbar_arrive_expect_tx(&sm.kv_full[st], kt.nseg * 2 * kSegBytes);
        uint8_t* dk = sK + st * kTileBytes;
        uint8_t* dv = sV + st * kTileBytes;
        tma_load_2d(dk, &p.tm_k, &sm.kv_full[st], h * 64, b * p.Nk + kt.row0);
        tma_load_2d(dv, &p.tm_v, &sm.kv_full[st], h * 64, b * p.Nk + kt.row0);
        if (kt.nseg == 2) {
          tma_load_2d(dk + kSegBytes, &p.tm_k, &sm.kv_full[st], h * 64, b * p.Nk + kt.row1);
          tma_load_2d(dv + kSegBytes, &p.tm_v, &sm.kv_full[st], h * 64, b * p.Nk + kt.row1);
        }
        issued = t + 1;
      }
      // Drain: every TMA write into shared memory must land before the CTA exits.
      wait_noabort(&sm.q_full, 0, p.status);
      for (int s = 0; s < kStages && s < issued; ++s) {
        const int t_last = s + kStages * ((issued - 1 - s) / kStages);
        wait_noabort(&sm.kv_full[s], (t_last / kStages) & 1, p.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s64 = make_idesc_bf16(128, 64, false);
      const uint32_t idesc_s128 = make_idesc_bf16(128, 128, false);
      const uint32_t idesc_pv = make_idesc_bf16(128, 64, true);
      const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);
      bool ok = bounded_wait(&sm.q_full, 0, abort_flag, p.status);
      tc_fence_after();
      int prev_nseg = 0;
      for (int t = 0; ok && t <= T; ++t) {
        const int st = t % kStages;
        int nseg = 0;
        if (t < T) {
          if (!bounded_wait(&sm.kv_full[st], (t / kStages) & 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          nseg = key_tile(p, sm.sel, t, T_loc, wstart, wend).nseg;
        }
        for (int m = 0; m < 2; ++m) {
          const uint32_t tS = tmem + 128 * m;
          if (t > 0) {
            if (!bounded_wait(&sm.p_full[m], (t - 1) & 1, abort_flag, p.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const int pt = t - 1;
            const uint32_t tO = tmem + 256 + 128 * m + (pt < T_loc ? 0 : 64);
            const uint32_t acc0 = (pt == 0 || pt == T_loc) ? 0u : 1u;
            const uint64_t vdesc = sw128_desc(sVa + (pt % kStages) * kTileBytes, 1024, 16384);
            for (int ks = 0; ks < prev_nseg * 4; ++ks)
              mma_ts(tO, tS + ks * 8, vdesc + static_cast<uint64_t>(ks * 128), idesc_pv, ks > 0 ? 1u : acc0);
          }
          if (t < T) {
            const uint64_t qdesc = sw128_desc(sQa + m * kTileBytes, 1024, 16);
            const uint64_t kdesc = sw128_desc(sKa + st * kTileBytes, 1024, 16);
            const uint32_t idesc = nseg == 2 ? idesc_s128 : idesc_s64;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              mma_ss(tS, qdesc + static_cast<uint64_t>(2 * ks), kdesc + static_cast<uint64_t>(2 * ks), idesc,
                     ks > 0 ? 1u : 0u);
            tc_commit(&sm.s_full[m]);
          }
        }
        if (!ok) break;
        if (t > 0) tc_commit(&sm.kv_empty[(t - 1) % kStages]);
        prev_nseg = nseg;
      }
      if (ok) {
        tc_commit(&sm.o_final[0]);
        tc_commit(&sm.o_final[1]);
      }
      tc_commit(&sm.drain);
      wait_noabort(&sm.drain, 0, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int wg = (warp - 2) >> 2;  // M-tile
    const int qd = warp & 3;         // TMEM lane quadrant this warp can access
    const int row = qd * 32 + lane;  // row of the M-tile
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t tS = tmem + lane_off + 128 * wg;
    const uint32_t tOl = tmem + lane_off + 256 + 128 * wg;
    const uint32_t tOs = tOl + 64;
    const int head = h * G + 2 * wg + (row >> 6);
    const int n = n0 + (row & 63);
    const bool live = n < p.Nq;

    // Gates of this output row (the reference's weight_ba_cmp_slc[:, b, n, head]).
    float c0 = 0.f, c1 = 0.f, c2 = 0.f;
    if (p.combine == kCombineLocal) {
      c0 = 1.f;
    } else if (p.combine == kCombineSel) {
      c2 = 1.f;
    } else if (live) {
      const size_t plane = static_cast<size_t>(p.B) * p.Nq * p.Hq;
      const size_t gi = (static_cast<size_t>(b) * p.Nq + n) * p.Hq + head;
      const float w0 = __bfloat162float(p.gates[gi]);
      const float w1 = __bfloat162float(p.gates[plane + gi]);
      const float w2 = __bfloat162float(p.gates[2 * plane + gi]);
      if (p.combine == kCombineGated) {
        c0 = w0;
        c1 = w1;
        c2 = w2;
      } else if (p.combine == kCombineNoCmp) {
        const float ws = w0 + w2 + 1e-8f;
        c0 = w0 / ws;
        c2 = w2 / ws;
      } else {  // kCombineNoSlc
        const float ws = w0 + w1 + 1e-8f;
        c0 = w0 / ws;
        c1 = w1 / ws;
      }
    }

    float m_run = -INFINITY, l_run = 0.f;
    float l_loc = 1.f, l_slc = 1.f, m_slc = 0.f;
    bool ok = true;
    for (int t = 0; t < T; ++t) {
      if (t == T_loc && t > 0) {
        l_loc = l_run;
        m_run = -INFINITY;
        l_run = 0.f;
      }
      if (!bounded_wait(&sm.s_full[wg], t & 1, abort_flag, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const KeyTile kt = key_tile(p, sm.sel, t, T_loc, wstart, wend);
      const bool first = (t == 0) || (t == T_loc);
      const uint32_t tO = t < T_loc ? tOl : tOs;
      if (kt.nseg == 2)
        softmax_tile<128>(tS, tO, kt.valid, first, p.scale_log2, m_run, l_run);
      else
        softmax_tile<64>(tS, tO, kt.valid, first, p.scale_log2, m_run, l_run);
      tc_fence_before();
      mbar_arrive(&sm.p_full[wg]);
    }
    if (T_slc > 0) {
      l_slc = l_run;
      m_slc = m_run;
    } else {
      l_loc = l_run;
    }

    if (ok) ok = bounded_wait(&sm.o_final[wg], 0, abort_flag, p.status);
    tc_fence_after();
    if (ok) {
      const float f0 = T_loc > 0 ? c0 / l_loc : 0.f;
      const float f2 = T_slc > 0 ? c2 / l_slc : 0.f;
      const uint4* cmp_row =
          (live && c1 != 0.f)
              ? reinterpret_cast<const uint4*>(p.o_cmp + ((static_cast<size_t>(b) * p.nqb + n / p.bs) * p.Hq + head) * 64)
              : nullptr;
      uint4* dst = reinterpret_cast<uint4*>(p.out + ((static_cast<size_t>(b) * p.Nq + (live ? n : 0)) * p.Hq + head) * 64);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
        if (T_loc > 0) {
          uint32_t o[32];
          tmem_ld32(tOl + 32 * half, o);
          tmem_ld_wait();
          reg_fence<32>(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(o[i]) * f0;
        }
        if (T_slc > 0) {
          uint32_t o[32];
          tmem_ld32(tOs + 32 * half, o);
          tmem_ld_wait();
          reg_fence<32>(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = fmaf(__uint_as_float(o[i]), f2, acc[i]);
        }
        if (cmp_row != nullptr) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 u = __ldg(cmp_row + 4 * half + i);
            const __nv_bfloat162* bv = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f2v = __bfloat1622float2(bv[j]);
              acc[8 * i + 2 * j] = fmaf(c1, f2v.x, acc[8 * i + 2 * j]);
              acc[8 * i + 2 * j + 1] = fmaf(c1, f2v.y, acc[8 * i + 2 * j + 1]);
            }
          }
        }
        if (live) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 u;
            u.x = pack_bf16x2(acc[8 * i + 0], acc[8 * i + 1]);
            u.y = pack_bf16x2(acc[8 * i + 2], acc[8 * i + 3]);
            u.z = pack_bf16x2(acc[8 * i + 4], acc[8 * i + 5]);
            u.w = pack_bf16x2(acc[8 * i + 6], acc[8 * i + 7]);
            dst[4 * half + i] = u;
          }
        }
      }
      if (live && p.lse != nullptr && T_slc > 0)
        p.lse[(static_cast<size_t>(b) * p.Nq + n) * p.Hq + head] = m_slc + log2f(l_slc);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int launch_engine(const EngineLaunch& a, cudaStream_t stream) {
  EngineParams p;
  memset(&p, 0, sizeof(p));
  if (make_tmap_bf16_2d(&p.tm_q, a.q, static_cast<uint64_t>(a.B) * a.Nq, static_cast<uint64_t>(a.Hq) * 64) ||
      make_tmap_bf16_2d(&p.tm_k, a.k, static_cast<uint64_t>(a.B) * a.Nk, static_cast<uint64_t>(a.Hk) * 64) ||
      make_tmap_bf16_2d(&p.tm_v, a.v, static_cast<uint64_t>(a.B) * a.Nk, static_cast<uint64_t>(a.Hk) * 64))
    return MOSAIC_ERR_CUDA;
  p.block_idx = a.block_idx;
  p.gates = static_cast<const __nv_bfloat16*>(a.gates);
  p.o_cmp = static_cast<const __nv_bfloat16*>(a.o_cmp);
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.lse = a.lse;
  p.status = a.status;
  p.B = a.B;
  p.Nq = a.Nq;
  p.Nk = a.Nk;
  p.Hq = a.Hq;
  p.Hk = a.Hk;
  p.win = a.win;
  p.bs = a.bs > 0 ? a.bs : 64;
  p.K = a.K;
  p.nqb = a.Nq / p.bs;
  p.nkb = a.Nk / p.bs;
  p.combine = a.combine;
  p.scale_log2 = a.softmax_scale * 1.4426950408889634f;

  // The shared-memory opt-in is a per-device function attribute: set it once per device.
  static bool attr_done[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOSAIC_ERR_CUDA;
  if (!attr_done[dev]) {
    if (cudaFuncSetAttribute(bsa_engine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes)) != cudaSuccess)
      return MOSAIC_ERR_CUDA;
    attr_done[dev] = true;
  }
  dim3 grid((a.Nq + kQTile - 1) / kQTile, a.Hk, a.B);
  bsa_engine_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

size_t engine_max_selected() { return kMaxSel; }

}  // namespace mosaic
