// Fused block-sparse attention engine for sm_100a (tcgen05 + TMEM + TMA).
//
// A work unit is one (batch b, kv head h, group of four query heads, 64-query tile):
// query heads h*G + 4*grp + 0..3 of the G = Hq / Hk heads that share kv head h
// (G = 8 makes two groups per kv head). The grid is persistent (one CTA per SM) and
// CTA i walks units i, i + grid, ... with Q double-buffered so that the next unit's
// Q loads while the current one finishes. The four head slots are packed into two
// M = 128 MMA tiles ("M-tiles": rows 0-63 = slot 2m, rows 64-127 = slot 2m+1), so
// every K/V tile that TMA brings into shared memory is used by 4 heads x 64 queries.
// With G = 1 or 2 the slots past the last head of the group load zeros (an
// out-of-range TMA column) and write nothing.
// Keys stream in tiles of 64 (one TMA box each for K and V, 8-stage ring):
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
// Warp roles (384 threads): warp 0 issues TMA, warps 1 and 2 issue the
// tcgen05.mma of M-tile 0 and 1 (converged warps, one elected lane; warp 1 also
// owns the TMEM allocation), warp 3 idles, warps 4-7 run the softmax + epilogue
// of M-tile 0 and warps 8-11 those of M-tile 1.
//
// Pipeline: S is double-buffered per M-tile, so Q*K^T of tile t+2 is issued as
// soon as P*V of tile t has been issued, and a softmax warpgroup never waits for
// the tensor core between tiles; the two M-tiles interleave on the tensor core.
// The softmax splits its exponentials between MUFU (ex2.approx) and a software
// exp2 on the FMA pipe, because at head_dim 64 the MUFU rate, not the tensor
// core, is the first limit.
//
// In the full forward this kernel is launched with programmatic stream
// serialization after the top-k kernel (EngineParams::pdl): its CTAs start while
// top-k and the coarse attention finish, run the local tiles of their first unit,
// and wait (griddepcontrol.wait) only before reading block indices (TMA warp) and
// coarse-attention rows (softmax warps). The top-k kernel completes only after the
// coarse attention, so one wait covers both.
//
// TMEM (512 columns, fp32): S/P buffer b of M-tile m at 64*(2m+b) (P overwrites
// the first 32 columns of its S buffer as packed 16-bit pairs and feeds P*V from
// TMEM), O_local of M-tile m at 256+128m, O_selected at 320+128m.
//
// Activation type: bf16, or fp16 (the reference's dtype under fp16 autocast). The
// kernel is instantiated for both; with fp16, Q, K, V and P enter the tensor core
// as fp16 (kind::f16 with f16 operands, fp32 accumulation) and the gates, coarse
// rows and output are fp16.
#include <cmath>
#include <cstring>

#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {

#ifdef MOSAIC_TRACE
// Development timeline (off in the library build): clock64() stamps of one CTA's
// pipeline events during its MOSAIC_TRACE_IT-th work unit, read back by a tracing
// build's host code.
__device__ long long g_engine_trace[4096];
#ifndef MOSAIC_TRACE_IT
#define MOSAIC_TRACE_IT 0
#endif
#define MOSAIC_TRACE_AT(cond, slot) \
  do {                              \
    if (cond) g_engine_trace[(slot)] = clock64(); \
  } while (0)
#else
#define MOSAIC_TRACE_IT 0
#define MOSAIC_TRACE_AT(cond, slot) \
  do {                              \
    (void)(cond);                   \
  } while (0)
#endif

namespace {

constexpr int kQTile = 64;
constexpr int kStages = 8;
constexpr int kBoxBytes = 64 * 128;        // one 64-row x 64-col bf16 box (8 KB)
constexpr int kQTileBytes = 2 * kBoxBytes;  // one M-tile of Q: 128 rows
constexpr int kThreads = 384;
constexpr int kMaxSel = 1024;  // max selected blocks per query block
// Of every kPolyDen pairs of scores, the last kPolyNum take the software exp2
// (FMA pipe) and the others ex2.approx (MUFU), so both pipes share the work.
#ifndef MOSAIC_POLY_NUM
#define MOSAIC_POLY_NUM 3
#endif
constexpr int kPolyDen = 8;
constexpr int kPolyNum = MOSAIC_POLY_NUM;
struct EngineParams {
  CUtensorMap tm_q, tm_k, tm_v;
  const int64_t* block_idx;
  const uint16_t* gates;  // 16-bit values of the activation type
  const uint16_t* o_cmp;
  uint16_t* out;
  float* lse;
  int* status;
  int B, Nq, Nk, Hq, Hk;
  int win, bs, K, nqb, nkb;
  int combine;
  float scale_log2;
  int G;        // query heads per kv head
  int ngroups;  // groups of four query heads per kv head: ceil(G / 4)
  int qtiles;   // 64-query tiles per (batch, kv head)
  int units;    // B * Hk * ngroups * qtiles work units
  int pdl;      // launched with programmatic serialization: wait for the previous grids before reading
                // block_idx and o_cmp
};

// One work unit: (batch b, kv head h, head group grp, 64-query tile starting at n0)
// and its key tiles.
struct Unit {
  int b, h, grp, n0;
  int wstart, wend;  // local window
  int T_loc, T;      // local tiles, all tiles
};

// Q column (elements) of head slot j of a unit: slots past the group's last head
// read at column Hq * 64, outside the tensor, which TMA fills with zeros.
__device__ __forceinline__ int q_column(const Unit& w, int j, int G, int Hq) {
  const int jj = w.grp * 4 + j;
  return jj < G ? (w.h * G + jj) * 64 : Hq * 64;
}

__device__ __forceinline__ Unit decode_unit(const EngineParams& p, int u) {
  Unit w;
  const int qt = u % p.qtiles;
  int rest = u / p.qtiles;
  w.grp = rest % p.ngroups;
  rest /= p.ngroups;
  w.h = rest % p.Hk;
  w.b = rest / p.Hk;
  w.n0 = qt * kQTile;
  w.T_loc = 0;
  w.wstart = w.wend = 0;
  if (p.win > 0) {
    w.wstart = (w.n0 / p.win) * p.win;
    w.wend = min(w.wstart + p.win, p.Nk);
    w.T_loc = (w.wend - w.wstart + 63) / 64;
  }
  w.T = w.T_loc + (p.K > 0 ? (p.K * p.bs) / 64 : 0);
  return w;
}

struct EngineSmem {
  uint64_t q_full[2];   // Q double buffer: loaded
  uint64_t q_empty[2];  // Q double buffer: every S of the unit issued (both MMA warps)
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2][2];  // [M-tile][S buffer]
  // [M-tile][S buffer]: one per buffer, because a softmax warpgroup may finish
  // tiles t and t+1 before the MMA warp consumes P(t); it can never get two tiles
  // ahead on the same buffer (S(t+2) is issued only after P(t)*V(t)).
  uint64_t p_full[2][2];
  uint64_t o_done[2];   // per P*V
  uint64_t o_final[2];  // per work unit: its last P*V has completed
  uint64_t o_empty[2];  // per work unit: the epilogue has read O
  uint64_t drain[2];
  uint32_t tmem_base;
  int abort_flag;
  int sel[kMaxSel];
};

constexpr size_t kSmemBytes = 1024 /*align slack*/ + 4 * kQTileBytes + 2 * kStages * kBoxBytes + sizeof(EngineSmem);

// TMEM columns (fp32, 128 lanes): S/P buffer b of M-tile m at 64*(2m+b);
// O_local of M-tile m at 256+128m, O_selected at 320+128m.
__device__ __forceinline__ uint32_t col_s(int m, int b) { return 64u * (2 * m + b); }
__device__ __forceinline__ uint32_t col_ol(int m) { return 256u + 128u * m; }
__device__ __forceinline__ uint32_t col_os(int m) { return 320u + 128u * m; }

// Key tile t = 64 keys: local-window tiles first, then one tile per 64-row
// segment of the selected blocks (block size is a multiple of 64).
struct KeyTile {
  int row;    // first key row within the batch
  int valid;  // keys of the tile that take part (< 64 only at the end of a short window)
};

__device__ __forceinline__ KeyTile key_tile(const EngineParams& p, const int* sel, int t, int T_loc, int wstart,
                                            int wend) {
  KeyTile kt;
  if (t < T_loc) {
    kt.row = wstart + 64 * t;
    kt.valid = min(64, wend - kt.row);
  } else {
    const int pos = (t - T_loc) * 64;
    kt.row = sel[pos / p.bs] * p.bs + pos % p.bs;
    kt.valid = 64;
  }
  return kt;
}

// exp2 of 64 scores against max m, packed in place as 32 pairs of the activation
// type (s[i] <- s[2i], s[2i+1]); returns the fp32 row sum. Of every kPolyDen pairs
// the last kPolyNum use the software exp2, the others ex2.approx.
#ifndef MOSAIC_NACC
#define MOSAIC_NACC 8
#endif
template <bool kF16>
__device__ __forceinline__ float exp_pack_tile(uint32_t (&s)[64], float c, float m) {
  const uint64_t c2 = f2_pack(c, c);
  const uint64_t nm2 = f2_pack(-m, -m);
  constexpr int kAcc = MOSAIC_NACC;  // independent partial sums (packed pairs)
  uint64_t acc[kAcc];
#pragma unroll
  for (int i = 0; i < kAcc; ++i) acc[i] = 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const uint64_t x = f2_fma(f2_pack(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), c2, nm2);
    uint64_t e;
    if ((i % kPolyDen) >= kPolyDen - kPolyNum) {
      e = exp2_poly2<true>(x);  // x = s*c - m_run is not bounded above (stale max)
    } else {
      float x0, x1;
      f2_unpack(x, x0, x1);
      e = f2_pack(ex2_approx(x0), ex2_approx(x1));
    }
    acc[i % kAcc] = f2_add(acc[i % kAcc], e);
    float e0, e1;
    f2_unpack(e, e0, e1);
    s[i] = Act<kF16>::pack(e0, e1);
  }
#pragma unroll
  for (int w = kAcc / 2; w > 0; w /= 2)
#pragma unroll
    for (int i = 0; i < w; ++i) acc[i] = f2_add(acc[i], acc[i + w]);
  float a0, a1;
  f2_unpack(acc[0], a0, a1);
  return a0 + a1;
}

__device__ __forceinline__ void load_scores(uint32_t tS, uint32_t (&s)[64], int valid) {
  tmem_ld32(tS, s);
  tmem_ld32(tS + 32, s + 32);
  tmem_ld_wait();
  reg_fence<64>(s);
  if (valid < 64) {
#pragma unroll
    for (int i = 0; i < 64; ++i)
      if (i >= valid) s[i] = __float_as_uint(-INFINITY);
  }
}

// Online-softmax step of one 64-key tile; each thread owns one row of the M-tile.
// The common path exponentiates against the running max m_run without looking at
// this tile's max: the result is exact after the final normalisation as long as
// no p grows too large, which the tile sum bounds (sum <= 2^14 => every p <= 2^14,
// far inside bf16/fp32 range). A row whose sum exceeds that (its max grew), the
// first tile of a branch, and any non-finite sum take the exact path: reload S,
// take the row max, rescale this row's O accumulator (after the previous P*V has
// landed, `o_done`) and l, and exponentiate again. P is written as 32 packed
// 16-bit pairs over the first 32 columns of the S buffer.
template <bool kF16>
__device__ __forceinline__ bool softmax_tile(uint32_t tS, uint32_t tO, int valid, bool first, float c,
                                             float& m_run, float& l_run, uint64_t* o_done, uint32_t o_parity,
                                             volatile int* abort_flag, int* status, int tslot) {
  constexpr float kSumLimit = 16384.0f;
  uint32_t s[64];
  load_scores(tS, s, valid);
  MOSAIC_TRACE_AT(tslot >= 0, 3000 + tslot * 4 + 0);
  float sum = 0.f;
  bool exact = first;
  if (!first) {
    sum = exp_pack_tile<kF16>(s, c, m_run);
    exact = !(sum <= kSumLimit);  // also catches NaN / inf
  }
  MOSAIC_TRACE_AT(tslot >= 0, 3000 + tslot * 4 + 1);
  bool ok = true;
  if (__any_sync(0xffffffffu, exact)) {
    // Exact path for the rows that need it (the warp runs it together).
    load_scores(tS, s, valid);
    float mx[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float a = fmax3(__uint_as_float(s[j]), __uint_as_float(s[j + 8]), __uint_as_float(s[j + 16]));
      a = fmax3(a, __uint_as_float(s[j + 24]), __uint_as_float(s[j + 32]));
      a = fmax3(a, __uint_as_float(s[j + 40]), __uint_as_float(s[j + 48]));
      mx[j] = fmaxf(a, __uint_as_float(s[j + 56]));
    }
    const float rmax = fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], fmax3(mx[5], mx[6], mx[7])));
    const float m_new = first ? rmax * c : fmaxf(m_run, rmax * c);
    const float alpha = first ? 1.0f : ex2_approx(m_run - m_new);
    const bool rescale = exact && !first;
    if (__any_sync(0xffffffffu, rescale)) {
      // The previous P*V must have landed in O before O is scaled.
      ok = bounded_wait(o_done, o_parity, abort_flag, status);
      tc_fence_after();
#pragma unroll 1
      for (int c8 = 0; c8 < 64; c8 += 8) {
        uint32_t o[8];
        tmem_ld8(tO + c8, o);
        tmem_ld_wait();
        reg_fence<8>(o);
        const float f = rescale ? alpha : 1.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
        tmem_st8(tO + c8, o);
      }
    }
    if (exact) {
      if (!first) l_run *= alpha;
      m_run = m_new;
    }
    const float sum2 = exp_pack_tile<kF16>(s, c, m_run);  // rows not on the exact path recompute the same values
    if (exact) sum = sum2;
  }
  tmem_st32(tS, s);
  MOSAIC_TRACE_AT(tslot >= 0, 3000 + tslot * 4 + 2);
  tmem_st_wait();
  MOSAIC_TRACE_AT(tslot >= 0, 3000 + tslot * 4 + 3);
  l_run += sum;
  return ok;
}

__device__ __forceinline__ bool wait_noabort(uint64_t* bar, uint32_t parity, int* status) {
  int dummy = 0;
  return bounded_wait(bar, parity, &dummy, status);
}

template <bool kF16>
__global__ void __launch_bounds__(kThreads, 1) bsa_engine_kernel(const __grid_constant__ EngineParams p) {
  using A = Act<kF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = tiles;  // two buffers of 2 M-tiles
  uint8_t* sK = tiles + 4 * kQTileBytes;
  uint8_t* sV = sK + kStages * kBoxBytes;
  EngineSmem& sm = *reinterpret_cast<EngineSmem*>(sV + kStages * kBoxBytes);
  volatile int* abort_flag = &sm.abort_flag;
  // A kernel launched after this one with programmatic stream serialization (the
  // top-k kernel after the coarse attention) may start right away: it does not
  // read anything this kernel writes.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool traced_cta = blockIdx.x == 5;
  MOSAIC_TRACE_AT(traced_cta && threadIdx.x == 0, 2000);
  const int G = p.Hq / p.Hk;

  if (threadIdx.x == 0) {
    for (int qb = 0; qb < 2; ++qb) {
      mbar_init(&sm.q_full[qb], 1);
      mbar_init(&sm.q_empty[qb], 2);  // both MMA warps
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 2);  // released by both MMA warps
    }
    for (int m = 0; m < 2; ++m) {
      mbar_init(&sm.s_full[m][0], 1);
      mbar_init(&sm.s_full[m][1], 1);
      mbar_init(&sm.p_full[m][0], 128);
      mbar_init(&sm.p_full[m][1], 128);
      mbar_init(&sm.o_done[m], 1);
      mbar_init(&sm.o_final[m], 1);
      mbar_init(&sm.o_empty[m], 128);
      mbar_init(&sm.drain[m], 1);
    }
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

  // Every role walks the same units in the same order; `g` counts key tiles
  // across units so that ring stages, S buffers and barrier phases continue.
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (converged warp)
    if (lane == 0) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_k);
      prefetch_tmap(&p.tm_v);
    }
    int g = 0, it = 0;
    bool ok = true, dep_done = !p.pdl;
    // This query block's selected kv blocks; out-of-range entries are reported and
    // clamped so that no load leaves the batch. Only this warp reads sel[].
    auto load_sel = [&](const Unit& w) {
      const int qb = w.n0 / p.bs;
      const int64_t* src = p.block_idx + ((static_cast<int64_t>(w.b) * p.nqb + qb) * p.Hk + w.h) * p.K;
      __syncwarp();
      for (int s = lane; s < p.K; s += 32) {
        int64_t v = src[s];
        if (v < 0 || v >= p.nkb) {
          if (p.status) atomicOr(p.status, MOSAIC_STATUS_BAD_INDEX);
          v = 0;
        }
        sm.sel[s] = static_cast<int>(v);
      }
      __syncwarp();
    };
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++it) {
      const Unit w = decode_unit(p, u);
      // Once the grids before this one are complete, the indices are read up front;
      // until then (the first unit of a kernel launched with programmatic
      // serialization after the top-k kernel) only after the local tiles are
      // queued, so that the local branch overlaps the end of top-k.
      const bool sel_now = p.K > 0 && dep_done;
      if (sel_now) load_sel(w);
      const int qbuf = it & 1;
      if (it >= 2 && !warp_wait(&sm.q_empty[qbuf], ((it - 2) >> 1) & 1, abort_flag, p.status)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx_elect(&sm.q_full[qbuf], 4 * kBoxBytes);
      for (int m = 0; m < 2; ++m)
        for (int v = 0; v < 2; ++v)
          tma_load_2d_elect(sQ + (2 * qbuf + m) * kQTileBytes + v * kBoxBytes, &p.tm_q, &sm.q_full[qbuf],
                            q_column(w, 2 * m + v, G, p.Hq), w.b * p.Nq + w.n0);
      for (int t = 0; t < w.T; ++t, ++g) {
        if (t == w.T_loc && p.K > 0 && !sel_now) {
          asm volatile("griddepcontrol.wait;" ::: "memory");
          dep_done = true;
          load_sel(w);
        }
        const int st = g % kStages, r = g / kStages;
        if (r > 0 && !warp_wait(&sm.kv_empty[st], (r - 1) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        const KeyTile kt = key_tile(p, sm.sel, t, w.T_loc, w.wstart, w.wend);
        mbar_arrive_expect_tx_elect(&sm.kv_full[st], 2 * kBoxBytes);
        tma_load_2d_elect(sK + st * kBoxBytes, &p.tm_k, &sm.kv_full[st], w.h * 64, w.b * p.Nk + kt.row);
        tma_load_2d_elect(sV + st * kBoxBytes, &p.tm_v, &sm.kv_full[st], w.h * 64, w.b * p.Nk + kt.row);
      }
    }
    // Drain: every TMA write into shared memory must land before the CTA exits.
    if (lane == 0) {
      for (int qb = 0; qb < 2 && qb < it; ++qb) {
        const int last_it = qb + 2 * ((it - 1 - qb) / 2);
        wait_noabort(&sm.q_full[qb], (last_it >> 1) & 1, p.status);
      }
      for (int s = 0; s < kStages && s < g; ++s) {
        const int g_last = s + kStages * ((g - 1 - s) / kStages);
        wait_noabort(&sm.kv_full[s], (g_last / kStages) & 1, p.status);
      }
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issuers (converged warps)
    // Warp 1 issues every MMA of M-tile 0 and warp 2 those of M-tile 1, so the two
    // issue chains overlap on the tensor core.
    const int m = warp - 1;
    const uint32_t idesc_s = make_idesc(128, 64, false, A::kMmaFmt);
    const uint32_t idesc_pv = make_idesc(128, 64, true, A::kMmaFmt);
    const uint32_t sKa = smem_u32(sK), sVa = smem_u32(sV), sQa = smem_u32(sQ);
    // S_m(gt) = Q_m K(gt)^T into S buffer gt%2 of M-tile m
    auto issue_s = [&](uint64_t qdesc, int gt) {
      const uint64_t kdesc = sw128_desc(sKa + (gt % kStages) * kBoxBytes, 1024, 16);
      const uint32_t tS = tmem + col_s(m, gt & 1);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_ss_elect(tS, qdesc + static_cast<uint64_t>(2 * ks), kdesc + static_cast<uint64_t>(2 * ks), idesc_s,
                     ks > 0 ? 1u : 0u);
      tc_commit_elect(&sm.s_full[m][gt & 1]);
    };
    int g = 0, it = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++it) {
      const Unit w = decode_unit(p, u);
      const int qbuf = it & 1;
      const uint64_t qdesc = sw128_desc(sQa + (2 * qbuf + m) * kQTileBytes, 1024, 16);
      ok = warp_wait(&sm.q_full[qbuf], (it >> 1) & 1, abort_flag, p.status);
      tc_fence_after();
      for (int j = 0; ok && j < 2 && j < w.T; ++j) {
        ok = warp_wait(&sm.kv_full[(g + j) % kStages], ((g + j) / kStages) & 1, abort_flag, p.status);
        tc_fence_after();
        if (ok) issue_s(qdesc, g + j);
      }
      // The epilogue of the previous unit must have read O before P*V overwrites it.
      if (ok && it > 0) {
        ok = warp_wait(&sm.o_empty[m], (it - 1) & 1, abort_flag, p.status);
        tc_fence_after();
      }
      for (int t = 0; ok && t < w.T; ++t) {
        const int gt = g + t;
        const uint32_t col_o_off = t < w.T_loc ? 0u : 64u;
        const uint32_t acc0 = (t == 0 || t == w.T_loc) ? 0u : 1u;
        const uint64_t vdesc = sw128_desc(sVa + (gt % kStages) * kBoxBytes, 1024, 16384);
        MOSAIC_TRACE_AT(traced_cta && it == MOSAIC_TRACE_IT && lane == 0 && t < 64, 1024 + (m * 64 + t) * 3 + 0);
        if (!warp_wait(&sm.p_full[m][gt & 1], (gt >> 1) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        MOSAIC_TRACE_AT(traced_cta && it == MOSAIC_TRACE_IT && lane == 0 && t < 64, 1024 + (m * 64 + t) * 3 + 1);
        tc_fence_after();
        const uint32_t tO = tmem + col_ol(m) + col_o_off;
        const uint32_t tP = tmem + col_s(m, gt & 1);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_ts_elect(tO, tP + ks * 8, vdesc + static_cast<uint64_t>(ks * 128), idesc_pv, ks > 0 ? 1u : acc0);
        tc_commit_elect(&sm.o_done[m]);
        if (t + 2 < w.T) {
          if (!warp_wait(&sm.kv_full[(gt + 2) % kStages], ((gt + 2) / kStages) & 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(qdesc, gt + 2);
        }
        tc_commit_elect(&sm.kv_empty[gt % kStages]);
        MOSAIC_TRACE_AT(traced_cta && it == MOSAIC_TRACE_IT && lane == 0 && t < 64, 1024 + (m * 64 + t) * 3 + 2);
      }
      if (!ok) break;
      tc_commit_elect(&sm.q_empty[qbuf]);  // every S of this unit has been issued
      tc_commit_elect(&sm.o_final[m]);
      g += w.T;
    }
    tc_commit_elect(&sm.drain[m]);
    if (lane == 0) wait_noabort(&sm.drain[m], 0, p.status);
    __syncwarp();
  } else if (warp == 3) {
    // idle warp (keeps the softmax warpgroups aligned to TMEM lane quadrants)
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int wg = (warp - 4) >> 2;  // M-tile
    const int qd = warp & 3;         // TMEM lane quadrant this warp can access
    const int row = qd * 32 + lane;  // row of the M-tile
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t tOl = tmem + lane_off + col_ol(wg);
    const uint32_t tOs = tmem + lane_off + col_os(wg);
    int g = 0, it = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++it) {
      const Unit w = decode_unit(p, u);
      const int T_slc = w.T - w.T_loc;
      const int slot = w.grp * 4 + 2 * wg + (row >> 6);  // query head within the kv group
      const int head = w.h * G + min(slot, G - 1);
      const int n = w.n0 + (row & 63);
      const bool live = n < p.Nq && slot < G;

      // Gates of this output row (the reference's weight_ba_cmp_slc[:, b, n, head]).
      float c0 = 0.f, c1 = 0.f, c2 = 0.f;
      if (p.combine == kCombineLocal) {
        c0 = 1.f;
      } else if (p.combine == kCombineSel) {
        c2 = 1.f;
      } else if (live) {
        const size_t plane = static_cast<size_t>(p.B) * p.Nq * p.Hq;
        const size_t gi = (static_cast<size_t>(w.b) * p.Nq + n) * p.Hq + head;
        const float w0 = A::from_bits(p.gates[gi]);
        const float w1 = A::from_bits(p.gates[plane + gi]);
        const float w2 = A::from_bits(p.gates[2 * plane + gi]);
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
      for (int t = 0; t < w.T; ++t) {
        const int gt = g + t;
        if (t == w.T_loc && t > 0) {
          l_loc = l_run;
          m_run = -INFINITY;
          l_run = 0.f;
        }
        const bool rec = traced_cta && it == MOSAIC_TRACE_IT && row == 0 && t < 64;
        MOSAIC_TRACE_AT(rec, (wg * 64 + t) * 5 + 0);
        if (!bounded_wait(&sm.s_full[wg][gt & 1], (gt >> 1) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        MOSAIC_TRACE_AT(rec, (wg * 64 + t) * 5 + 1);
        tc_fence_after();
        const int valid = t < w.T_loc ? min(64, w.wend - (w.wstart + 64 * t)) : 64;
        const bool first = (t == 0) || (t == w.T_loc);
        const uint32_t tS = tmem + lane_off + col_s(wg, gt & 1);
        ok = softmax_tile<kF16>(tS, t < w.T_loc ? tOl : tOs, valid, first, p.scale_log2, m_run, l_run, &sm.o_done[wg],
                          (gt - 1) & 1, abort_flag, p.status, rec ? wg * 64 + t : -1);
        MOSAIC_TRACE_AT(rec, (wg * 64 + t) * 5 + 4);
        tc_fence_before();
        mbar_arrive(&sm.p_full[wg][gt & 1]);
        if (!ok) break;
      }
      if (!ok) break;
      if (T_slc > 0) {
        l_slc = l_run;
        m_slc = m_run;
      } else {
        l_loc = l_run;
      }

      // The coarse-attention rows come from a kernel that may still run when this
      // one starts (programmatic serialization): wait for it before the first read.
      // The wait returns at once after its first completion, and in a kernel launched
      // without programmatic serialization; it carries the row pointer, so the loads
      // below cannot move above it.
      const uint16_t* o_cmp = p.o_cmp;
      asm volatile("griddepcontrol.wait;" : "+l"(o_cmp));
      // Start the coarse-attention row loads before waiting for the last P*V (plain
      // loads: with programmatic serialization the rows are written while this
      // kernel runs, so they are not read-only for its lifetime).
      const uint4* cmp_row =
          (live && c1 != 0.f)
              ? reinterpret_cast<const uint4*>(o_cmp + ((static_cast<size_t>(w.b) * p.nqb + n / p.bs) * p.Hq + head) * 64)
              : nullptr;
      uint4 cmpv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) cmpv[i] = cmp_row != nullptr ? cmp_row[i] : make_uint4(0, 0, 0, 0);

      MOSAIC_TRACE_AT(traced_cta && it == MOSAIC_TRACE_IT && row == 0, 2002 + wg);
      if (!bounded_wait(&sm.o_final[wg], it & 1, abort_flag, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float f0 = w.T_loc > 0 ? c0 / l_loc : 0.f;
      const float f2 = T_slc > 0 ? c2 / l_slc : 0.f;
      uint4* dst =
          reinterpret_cast<uint4*>(p.out + ((static_cast<size_t>(w.b) * p.Nq + (live ? n : 0)) * p.Hq + head) * 64);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
        if (w.T_loc > 0) {
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
            const uint32_t* bv = reinterpret_cast<const uint32_t*>(&cmpv[4 * half + i]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f2v = A::unpack(bv[j]);
              acc[8 * i + 2 * j] = fmaf(c1, f2v.x, acc[8 * i + 2 * j]);
              acc[8 * i + 2 * j + 1] = fmaf(c1, f2v.y, acc[8 * i + 2 * j + 1]);
            }
          }
        }
        if (live) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 v;
            v.x = A::pack(acc[8 * i + 0], acc[8 * i + 1]);
            v.y = A::pack(acc[8 * i + 2], acc[8 * i + 3]);
            v.z = A::pack(acc[8 * i + 4], acc[8 * i + 5]);
            v.w = A::pack(acc[8 * i + 6], acc[8 * i + 7]);
            dst[4 * half + i] = v;
          }
        }
      }
      // O has been read: the next unit's first P*V may overwrite it.
      tc_fence_before();
      mbar_arrive(&sm.o_empty[wg]);
      MOSAIC_TRACE_AT(traced_cta && it == MOSAIC_TRACE_IT && row == 0, 2006 + wg);
      if (live && p.lse != nullptr && T_slc > 0)
        p.lse[(static_cast<size_t>(w.b) * p.Nq + n) * p.Hq + head] = m_slc + log2f(l_slc);
      g += w.T;
    }
  }

  MOSAIC_TRACE_AT(traced_cta && (threadIdx.x == 128 || threadIdx.x == 256), 2004 + (threadIdx.x == 256));
  tc_fence_before();
  __syncthreads();
  MOSAIC_TRACE_AT(traced_cta && threadIdx.x == 0, 2001);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int launch_engine(const EngineLaunch& a, cudaStream_t stream) {
  EngineParams p;
  memset(&p, 0, sizeof(p));
  if (make_tmap_2d(&p.tm_q, a.q, static_cast<uint64_t>(a.B) * a.Nq, static_cast<uint64_t>(a.Hq) * 64, a.f16) ||
      make_tmap_2d(&p.tm_k, a.k, static_cast<uint64_t>(a.B) * a.Nk, static_cast<uint64_t>(a.Hk) * 64, a.f16) ||
      make_tmap_2d(&p.tm_v, a.v, static_cast<uint64_t>(a.B) * a.Nk, static_cast<uint64_t>(a.Hk) * 64, a.f16))
    return MOSAIC_ERR_CUDA;
  p.block_idx = a.block_idx;
  p.gates = static_cast<const uint16_t*>(a.gates);
  p.o_cmp = static_cast<const uint16_t*>(a.o_cmp);
  p.out = static_cast<uint16_t*>(a.out);
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
  p.G = a.Hq / a.Hk;
  p.ngroups = (p.G + 3) / 4;
  p.qtiles = (a.Nq + kQTile - 1) / kQTile;
  p.units = a.B * a.Hk * p.ngroups * p.qtiles;
  p.pdl = a.after_topk ? 1 : 0;

  // The shared-memory opt-in is a per-device function attribute: set it once per
  // device and instantiation.
  static bool attr_done[2][64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOSAIC_ERR_CUDA;
  if (!attr_done[a.f16][dev]) {
    if (cudaFuncSetAttribute(a.f16 ? bsa_engine_kernel<true> : bsa_engine_kernel<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes)) != cudaSuccess)
      return MOSAIC_ERR_CUDA;
    attr_done[a.f16][dev] = true;
  }
  // Persistent: one CTA per SM (TMEM and shared memory allow no more), each
  // walking work units blockIdx.x, blockIdx.x + gridDim.x, ...
  static int sm_count[64] = {};
  if (sm_count[dev] == 0 &&
      cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return MOSAIC_ERR_CUDA;
  const int grid = p.units < sm_count[dev] ? p.units : sm_count[dev];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.after_topk ? 1 : 0;
  const cudaError_t e = a.f16 ? cudaLaunchKernelEx(&cfg, bsa_engine_kernel<true>, p)
                              : cudaLaunchKernelEx(&cfg, bsa_engine_kernel<false>, p);
  return e == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

size_t engine_max_selected() { return kMaxSel; }

}  // namespace mosaic
