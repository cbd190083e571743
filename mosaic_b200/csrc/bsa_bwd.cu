// Backward of the selected-block attention for sm_100a: the gradients that
// ops.MosaicAttnFunction.backward (ops.py:542-554) computes through
// ops.mosaic_attn_bwd (ops.py:436-507) and its two Triton kernels.
//
// With c = scale * log2(e), S = q.k (fp32), P = exp2(S c - lse) (lse in log2 units,
// as the forward writes it), dP = dO.v and D = rowsum(O * dO):
//   dS = P (dP - D)
//   dQ = scale * sum over the selected keys of bf16(dS) k            (ops.py:184-274)
//   dK = scale * sum over the selecting queries of bf16(dS) q        (ops.py:305-433)
//   dV =         sum over the selecting queries of bf16(P) dO
// dQ loops over every selection of the query block (a block selected twice counts
// twice, as in the forward); dK and dV take each selecting query block once (the
// reference's boolean block mask, ops.mosaic_block_mask at ops.py:277-297).
//
// Kernels, in launch order:
//   delta      D per (row, head)                                        HBM-bound
//   idx_*      the inverted block index: for every kv block the ascending, distinct
//              q blocks that selected it (count, scan, fill, sort), and per 128-key
//              tile the size of the union of its two 64-key segments' lists
//   dq         per (b, kv head, 64-query tile): S = Q K^T and dP = dO V^T on the
//              tensor core into TMEM, dS = P (dP - D) written back into TMEM as bf16,
//              dQ += dS K from TMEM (the 4 query heads as two 128-row M-tiles)
//   dkv        per (b, kv head, 128-key tile): S^T = K Q^T and dP^T = V dO^T, P^T and
//              dS^T in TMEM, dV += P^T dO and dK += dS^T Q, over 128-row chunks
//              (64 queries x 2 heads) of the q blocks that selected the tile
// Every wait is bounded (no kernel can hang); no TMA multicast.
#include <cstring>

#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {
namespace {

constexpr int kBox = 64 * 128;  // one 64-row x 64-col bf16 box (8 KB)

__device__ __forceinline__ bool wait_noabort_b(uint64_t* bar, uint32_t parity, int* status) {
  int dummy = 0;
  return bounded_wait(bar, parity, &dummy, status);
}

// 32 lanes x 16 consecutive 32-bit TMEM columns <- 16 registers per thread.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Four consecutive fp32 values from shared memory (16-byte aligned).
__device__ __forceinline__ float4 lds4(const float* ptr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(smem_u32(ptr)));
  return v;
}

// P^T and dS^T of one key row over 32 query columns, packed in place as 16 bf16
// pairs: p = exp2(s c - lse), ds = p (dp - D), with nlse = -lse and ndl = -D read
// from shared memory. Of every 8 pairs the last 3 take the software exp2 on the FMA
// pipe and the others ex2.approx, which balances the two pipes (the same split as
// the forward softmax). s[i] / dp[i] are read at pair i/2 <= i, before pair i is
// written, so packing in place is safe.
__device__ __forceinline__ void p_ds_quarter(uint32_t (&s)[32], uint32_t (&dp)[32], const float* nlse,
                                             const float* ndl, float c) {
  constexpr int kPolyDen = 8, kPolyNum = 3;
  const uint64_t c2 = f2_pack(c, c);
#pragma unroll
  for (int q = 0; q < 4; ++q) {  // 8 columns: two 16-byte loads of each of nlse, ndl
    const float4 la = lds4(nlse + 8 * q), lb = lds4(nlse + 8 * q + 4);
    const float4 da = lds4(ndl + 8 * q), db = lds4(ndl + 8 * q + 4);
    const uint64_t nl[4] = {f2_pack(la.x, la.y), f2_pack(la.z, la.w), f2_pack(lb.x, lb.y), f2_pack(lb.z, lb.w)};
    const uint64_t nd[4] = {f2_pack(da.x, da.y), f2_pack(da.z, da.w), f2_pack(db.x, db.y), f2_pack(db.z, db.w)};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = 4 * q + k;
      const uint64_t x = f2_fma(f2_pack(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), c2, nl[k]);
      uint64_t e;
      if ((i % kPolyDen) >= kPolyDen - kPolyNum) {
        e = exp2_poly2(x);  // x = s*c - lse <= 0 up to rounding: lse is the forward's log-sum of these keys
      } else {
        float x0, x1;
        f2_unpack(x, x0, x1);
        e = f2_pack(ex2_approx(x0), ex2_approx(x1));
      }
      const uint64_t d =
          f2_mul(e, f2_add(f2_pack(__uint_as_float(dp[2 * i]), __uint_as_float(dp[2 * i + 1])), nd[k]));
      float e0, e1, d0, d1;
      f2_unpack(e, e0, e1);
      f2_unpack(d, d0, d1);
      s[i] = pack_bf16x2(e0, e1);
      dp[i] = pack_bf16x2(d0, d1);
    }
  }
}

// ============================================================================ D
// D[r] = sum_d O[r, d] dO[r, d] in fp32; 8 threads per 64-value row (coalesced
// 16-byte loads), reduced with shuffles.
__global__ void delta_kernel(const uint4* o, const uint4* go, float* D, long long rows) {
  const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long r = t >> 3;
  float s = 0.f;
  if (r < rows) {
    const uint4 a = __ldg(o + t), b = __ldg(go + t);
    const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fx = __bfloat1622float2(x[j]), fy = __bfloat1622float2(y[j]);
      s = fmaf(fx.x, fy.x, s);
      s = fmaf(fx.y, fy.y, s);
    }
  }
  s += __shfl_xor_sync(0xffffffffu, s, 4);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  if (r < rows && (t & 7) == 0) D[r] = s;
}

// ============================================================================ inverted index
// For (b, h) = bh: offs[bh * (nkb + 1) + c] .. [c + 1] delimit, inside
// list[bh * nkb * K ...], the q blocks that selected kv block c.

__device__ __forceinline__ bool first_occurrence(const int64_t* row, int s) {
  const int64_t c = row[s];
  for (int s2 = 0; s2 < s; ++s2)
    if (row[s2] == c) return false;
  return true;
}

// One thread per (b, q block, h) row of block_indices.
__global__ void idx_count_kernel(const int64_t* idx, int* count, int B, int nqb, int Hk, int K, int nkb,
                                 int* status) {
  const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= static_cast<long long>(B) * nqb * Hk) return;
  const int h = static_cast<int>(t % Hk);
  const int b = static_cast<int>(t / (static_cast<long long>(Hk) * nqb));
  const int64_t* row = idx + t * K;
  for (int s = 0; s < K; ++s) {
    const int64_t c = row[s];
    if (c < 0 || c >= nkb) {
      if (status) atomicOr(status, MOSAIC_STATUS_BAD_INDEX);
      continue;
    }
    if (first_occurrence(row, s)) atomicAdd(&count[(static_cast<size_t>(b) * Hk + h) * nkb + c], 1);
  }
}

// One 1024-thread CTA per (b, h): offs = exclusive prefix sum of count (nkb + 1 entries).
__global__ void __launch_bounds__(1024) idx_scan_kernel(const int* count, int* offs, int nkb) {
  __shared__ int warp_sum[32];
  const int bh = blockIdx.x;
  const int* cnt = count + static_cast<size_t>(bh) * nkb;
  int* off = offs + static_cast<size_t>(bh) * (nkb + 1);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int per = (nkb + 1023) / 1024;
  const int c0 = min(static_cast<int>(threadIdx.x) * per, nkb), c1 = min(c0 + per, nkb);
  int s = 0;
  for (int c = c0; c < c1; ++c) s += cnt[c];
  int incl = s;  // inclusive scan of the per-thread sums within the warp
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += x;
  }
  if (lane == 31) warp_sum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = warp_sum[lane];
    int wi = w;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, wi, d);
      if (lane >= d) wi += x;
    }
    warp_sum[lane] = wi - w;  // exclusive prefix of the warp totals
  }
  __syncthreads();
  int run = warp_sum[warp] + incl - s;
  for (int c = c0; c < c1; ++c) {
    off[c] = run;
    run += cnt[c];
  }
  if (threadIdx.x == 1023) off[nkb] = warp_sum[31] + incl;
}

__global__ void idx_fill_kernel(const int64_t* idx, const int* offs, int* cursor, int* list, int B, int nqb, int Hk,
                                int K, int nkb) {
  const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= static_cast<long long>(B) * nqb * Hk) return;
  const int h = static_cast<int>(t % Hk);
  const int i = static_cast<int>((t / Hk) % nqb);
  const int b = static_cast<int>(t / (static_cast<long long>(Hk) * nqb));
  const size_t bh = static_cast<size_t>(b) * Hk + h;
  const int64_t* row = idx + t * K;
  for (int s = 0; s < K; ++s) {
    const int64_t c = row[s];
    if (c < 0 || c >= nkb || !first_occurrence(row, s)) continue;
    const int pos = atomicAdd(&cursor[bh * nkb + c], 1);
    list[bh * static_cast<size_t>(nkb) * K + offs[bh * (nkb + 1) + c] + pos] = i;
  }
}

// One 128-thread CTA per list: rank sort (entries are distinct) from `list` into
// `sorted`, so that dK / dV accumulate their chunks in ascending q-block order
// whatever order the atomics of idx_fill produced.
constexpr int kSortCap = 2048;
__global__ void __launch_bounds__(128) idx_sort_kernel(const int* offs, const int* list, int* sorted, int nkb,
                                                       int K) {
  __shared__ int buf[kSortCap];
  const int bh = blockIdx.x / nkb, c = blockIdx.x % nkb;
  const size_t base = static_cast<size_t>(bh) * nkb * K;
  const int o0 = offs[static_cast<size_t>(bh) * (nkb + 1) + c], o1 = offs[static_cast<size_t>(bh) * (nkb + 1) + c + 1];
  const int n = o1 - o0;
  const int* src = list + base + o0;
  const bool in_smem = n <= kSortCap;
  if (in_smem) {
    for (int e = threadIdx.x; e < n; e += blockDim.x) buf[e] = src[e];
    __syncthreads();
  }
  const int* v = in_smem ? buf : src;
  for (int e = threadIdx.x; e < n; e += blockDim.x) {
    const int x = v[e];
    int rank = 0;
    for (int j = 0; j < n; ++j) rank += v[j] < x ? 1 : 0;
    sorted[base + o0 + rank] = x;
  }
}

// The q blocks of a 128-key tile: the ascending union of the lists of the kv
// blocks of its two 64-key segments, with a mask of which segments each selected.
struct UnionWalk {
  const int* a;
  const int* c;
  int na, nc, ia, ic;
  __device__ bool next(int& qb, int& mask) {
    if (ia >= na && ic >= nc) return false;
    const int x = ia < na ? a[ia] : 0x7FFFFFFF, y = ic < nc ? c[ic] : 0x7FFFFFFF;
    if (x == y) {
      qb = x;
      mask = 3;
      ++ia;
      ++ic;
    } else if (x < y) {
      qb = x;
      mask = 1;
      ++ia;
    } else {
      qb = y;
      mask = 2;
      ++ic;
    }
    return true;
  }
};

struct KeyTile {
  int b, h, key0;
  int blk0, blk1;  // kv blocks of the two segments (blk1 = -1: the tile ends at the sequence end)
};

__device__ __forceinline__ KeyTile decode_key_tile(int u, int ktiles, int Hk, int N, int bs) {
  KeyTile k;
  const int kt = u % ktiles, rest = u / ktiles;
  k.h = rest % Hk;
  k.b = rest / Hk;
  k.key0 = kt * 128;
  k.blk0 = k.key0 / bs;
  k.blk1 = k.key0 + 64 < N ? (k.key0 + 64) / bs : -1;
  return k;
}

__device__ __forceinline__ UnionWalk make_walk(const int* offs_all, const int* list_all, const KeyTile& k, int Hk,
                                               int nkb, int K) {
  UnionWalk w;
  const size_t bh = static_cast<size_t>(k.b) * Hk + k.h;
  const int* offs = offs_all + bh * (nkb + 1);
  const int* base = list_all + bh * static_cast<size_t>(nkb) * K;
  w.a = base + offs[k.blk0];
  w.na = offs[k.blk0 + 1] - offs[k.blk0];
  if (k.blk1 >= 0 && k.blk1 != k.blk0) {
    w.c = base + offs[k.blk1];
    w.nc = offs[k.blk1 + 1] - offs[k.blk1];
  } else {
    w.c = w.a;
    w.nc = k.blk1 >= 0 ? w.na : 0;  // both segments in one block: every entry pairs with itself
  }
  w.ia = w.ic = 0;
  return w;
}

// One thread per 128-key tile: the number of q blocks in its union.
__global__ void idx_union_kernel(const int* offs, const int* sorted, int* ucount, int units, int ktiles, int Hk,
                                 int N, int bs, int nkb, int K) {
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= units) return;
  const KeyTile kt = decode_key_tile(u, ktiles, Hk, N, bs);
  UnionWalk w = make_walk(offs, sorted, kt, Hk, nkb, K);
  int n = 0, qb, mk;
  while (w.next(qb, mk)) ++n;
  ucount[u] = n;
}

// ============================================================================ dQ
constexpr int kThreadsBwd = 384;  // warp 0 TMA, warp 1 MMA, warps 2-3 idle, warps 4-11 rows
constexpr int kStagesDq = 8;
constexpr int kMaxSelB = 1024;

struct DqParams {
  CUtensorMap tm_q, tm_do, tm_k, tm_v;
  const int64_t* block_idx;
  const float* lse;
  const float* delta;
  __nv_bfloat16* dq;
  int* status;
  int B, N, Hq, Hk, bs, K, nqb, nkb;
  float scale, scale_log2;
  int ngroups;  // groups of four query heads per kv head: ceil(G / 4)
  int qtiles, units;
};

// A dq unit: (batch b, kv head h, head group grp, 64-query tile qt) with the query
// heads h*G + 4*grp + 0..3 (slots past the group's last head are empty: their Q and
// dO load as zeros and their dQ is not written).
struct DqUnit {
  int b, h, grp, qt;
};

__device__ __forceinline__ DqUnit decode_dq_unit(const DqParams& p, int u) {
  DqUnit w;
  w.qt = u % p.qtiles;
  int rest = u / p.qtiles;
  w.grp = rest % p.ngroups;
  rest /= p.ngroups;
  w.h = rest % p.Hk;
  w.b = rest / p.Hk;
  return w;
}

struct DqSmem {
  uint64_t kv_full[kStagesDq], kv_empty[kStagesDq];
  uint64_t qs_full, qs_empty;  // the shared-memory staging buffer of the next unit's Q / dO
  uint64_t qt_full[2], sp_full[2], ds_full[2], dq_done[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int sel[kMaxSelB];
};

constexpr size_t kDqSmemBytes = 1024 + 8 * kBox /*Q, dO staging*/ + 2 * kStagesDq * kBox /*K, V*/ + sizeof(DqSmem);

// TMEM of M-tile m (query heads 2m, 2m+1 of the group) at 256m: S (64 columns; dS
// overwrites its first 32 as bf16 pairs), dP at +64, dQ at +128, and the unit's Q and
// dO rows as bf16 pairs at +192 and +224: the A operands of S = Q K^T and dP = dO V^T,
// written once per unit by the row threads from a shared-memory staging buffer that
// the producer fills for the next unit while the current one runs, so those MMAs read
// only K / V from shared memory.
__global__ void __launch_bounds__(kThreadsBwd, 1) dq_kernel(const __grid_constant__ DqParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = tiles;                   // staging: boxes j = 0..3 (head j of the group)
  uint8_t* sDO = tiles + 4 * kBox;       // same layout
  uint8_t* sK = tiles + 8 * kBox;        // stages
  uint8_t* sV = sK + kStagesDq * kBox;   // stages
  DqSmem& sm = *reinterpret_cast<DqSmem*>(sV + kStagesDq * kBox);
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.Hq / p.Hk;
  const int spb = p.bs / 64;
  const int T = p.K * spb;  // 64-key tiles per unit

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesDq; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    mbar_init(&sm.qs_full, 1);
    mbar_init(&sm.qs_empty, 256);
    for (int m = 0; m < 2; ++m) {
      mbar_init(&sm.qt_full[m], 128);
      mbar_init(&sm.sp_full[m], 1);
      mbar_init(&sm.ds_full[m], 128);
      mbar_init(&sm.dq_done[m], 1);
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
    // Per unit: its Q / dO boxes into the staging buffer (free once the rows copied the
    // previous unit's into TMEM, at that unit's start), then its K / V tiles.
    int g = 0, nq = 0;  // K/V tiles and Q/dO stagings issued
    bool ok = true;
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
      const DqUnit un = decode_dq_unit(p, u);
      const int qt = un.qt, h = un.h, b = un.b;
      const int qb = qt * 64 / p.bs;
      const int64_t* src = p.block_idx + ((static_cast<int64_t>(b) * p.nqb + qb) * p.Hk + h) * p.K;
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
      if (nq > 0 && !warp_wait(&sm.qs_empty, (nq - 1) & 1, abort_flag, p.status)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx_elect(&sm.qs_full, 8 * kBox);
      for (int j = 0; j < 4; ++j) {
        // an empty slot reads at column Hq * 64, outside the tensor: TMA fills zeros
        const int jj = un.grp * 4 + j;
        const int col = jj < G ? (h * G + jj) * 64 : p.Hq * 64, row = b * p.N + qt * 64;
        tma_load_2d_elect(sQ + j * kBox, &p.tm_q, &sm.qs_full, col, row);
        tma_load_2d_elect(sDO + j * kBox, &p.tm_do, &sm.qs_full, col, row);
      }
      ++nq;
      for (int t = 0; t < T; ++t, ++g) {
        const int st = g % kStagesDq, r = g / kStagesDq;
        if (r > 0 && !warp_wait(&sm.kv_empty[st], (r - 1) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        const int krow = sm.sel[t / spb] * p.bs + (t % spb) * 64;
        mbar_arrive_expect_tx_elect(&sm.kv_full[st], 2 * kBox);
        tma_load_2d_elect(sK + st * kBox, &p.tm_k, &sm.kv_full[st], h * 64, b * p.N + krow);
        tma_load_2d_elect(sV + st * kBox, &p.tm_v, &sm.kv_full[st], h * 64, b * p.N + krow);
      }
    }
    // Drain: every TMA write into shared memory lands before the CTA exits.
    if (lane == 0) {
      if (nq > 0) wait_noabort_b(&sm.qs_full, (nq - 1) & 1, p.status);
      for (int s = 0; s < kStagesDq && s < g; ++s) {
        const int g_last = s + kStagesDq * ((g - 1 - s) / kStagesDq);
        wait_noabort_b(&sm.kv_full[s], (g_last / kStagesDq) & 1, p.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (both M-tiles)
    // Software-pipelined: once the rows of M-tile m have turned tile t into dS, the
    // warp issues dQ_m(t) and then S_m / dP_m of tile t + 1, so one warpgroup works on
    // tile t + 1 while the other finishes tile t.
    const uint32_t id_s = make_idesc_bf16(128, 64, false);   // B = K / V tile, K-major
    const uint32_t id_dq = make_idesc_bf16(128, 64, true);   // B = K tile as [keys x d], MN-major
    const uint32_t sKa = smem_u32(sK), sVa = smem_u32(sV);
    // S_m = Q_m K^T and dP_m = dO_m V^T of the tile in stage st (Q_m, dO_m from TMEM)
    auto issue_sdp = [&](int m, int st) {
      const uint64_t kd = sw128_desc(sKa + st * kBox, 1024, 16);
      const uint64_t vd = sw128_desc(sVa + st * kBox, 1024, 16);
      const uint32_t tM = tmem + 256u * m;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_ts_elect(tM, tM + 192u + 8u * ks, kd + static_cast<uint64_t>(2 * ks), id_s, ks > 0 ? 1u : 0u);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_ts_elect(tM + 64u, tM + 224u + 8u * ks, vd + static_cast<uint64_t>(2 * ks), id_s, ks > 0 ? 1u : 0u);
      tc_commit_elect(&sm.sp_full[m]);
    };
    int g = 0, it = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++it) {
      // qt_full: the rows have written this unit's Q / dO into TMEM, after reading the
      // previous unit's dQ (so dQ may be overwritten too).
      ok = warp_wait(&sm.qt_full[0], it & 1, abort_flag, p.status) &&
           warp_wait(&sm.qt_full[1], it & 1, abort_flag, p.status) &&
           warp_wait(&sm.kv_full[g % kStagesDq], (g / kStagesDq) & 1, abort_flag, p.status);
      tc_fence_after();
      if (!ok) break;
      issue_sdp(0, g % kStagesDq);
      issue_sdp(1, g % kStagesDq);
      for (int t = 0; ok && t < T; ++t) {
        const int gt = g + t, st = gt % kStagesDq;
        const uint64_t kmn = sw128_desc(sKa + st * kBox, 1024, 16384);
        for (int m = 0; ok && m < 2; ++m) {
          ok = warp_wait(&sm.ds_full[m], gt & 1, abort_flag, p.status);
          tc_fence_after();
          if (!ok) break;
          const uint32_t tM = tmem + 256u * m;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            mma_ts_elect(tM + 128u, tM + 8u * ks, kmn + static_cast<uint64_t>(ks * 128), id_dq,
                         (t > 0 || ks > 0) ? 1u : 0u);
          if (t == T - 1) {
            tc_commit_elect(&sm.dq_done[m]);  // also: every MMA of the unit reading Q_m / dO_m is issued
          } else {
            if (m == 0) {
              ok = warp_wait(&sm.kv_full[(gt + 1) % kStagesDq], ((gt + 1) / kStagesDq) & 1, abort_flag, p.status);
              tc_fence_after();
              if (!ok) break;
            }
            // S_m / dP_m of the next tile overwrite the dS that the dQ_m MMAs above read;
            // tcgen05.mma executes in issue order, so those reads come first.
            issue_sdp(m, (gt + 1) % kStagesDq);
          }
        }
        if (ok) tc_commit_elect(&sm.kv_empty[st]);
      }
      if (!ok) break;
      g += T;
    }
    tc_commit_elect(&sm.drain);
    if (lane == 0) wait_noabort_b(&sm.drain, 0, p.status);
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- dS and the dQ epilogue, one query row per thread
    const int wg = (warp - 4) >> 2, qd = warp & 3;
    const int row = qd * 32 + lane;
    const uint32_t tM = tmem + (static_cast<uint32_t>(qd * 32) << 16) + 256u * wg;
    int g = 0, it = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++it) {
      const DqUnit un = decode_dq_unit(p, u);
      const int qt = un.qt, h = un.h, b = un.b;
      const int slot = un.grp * 4 + 2 * wg + (row >> 6);  // query head within the kv group
      const bool live = slot < G;
      const int head = h * G + min(slot, G - 1);
      const int n = qt * 64 + (row & 63);
      const size_t ri = (static_cast<size_t>(b) * p.N + n) * p.Hq + head;
      // an empty slot's row has Q = dO = 0, so lse = D = 0 make its dS zero
      const float lse_r = live ? p.lse[ri] : 0.f, d_r = live ? p.delta[ri] : 0.f;
      {
        // This row of Q and of dO, from the staging buffer (a 128-byte-swizzled TMA box:
        // 16-byte chunk c of box row r sits at chunk c ^ (r & 7)), into TMEM. Every MMA
        // of the previous unit has completed: its epilogue below waited for dq_done,
        // committed after the last of them.
        if (!bounded_wait(&sm.qs_full, it & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        const int r = row & 63;
        const uint8_t* qrow = sQ + (2 * wg + (row >> 6)) * kBox + r * 128;
        const uint8_t* orow = sDO + (2 * wg + (row >> 6)) * kBox + r * 128;
        uint32_t qa[32], oa[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 x = *reinterpret_cast<const uint4*>(qrow + ((c ^ (r & 7)) << 4));
          const uint4 y = *reinterpret_cast<const uint4*>(orow + ((c ^ (r & 7)) << 4));
          qa[4 * c] = x.x; qa[4 * c + 1] = x.y; qa[4 * c + 2] = x.z; qa[4 * c + 3] = x.w;
          oa[4 * c] = y.x; oa[4 * c + 1] = y.y; oa[4 * c + 2] = y.z; oa[4 * c + 3] = y.w;
        }
        mbar_arrive(&sm.qs_empty);
        tmem_st32(tM + 192, qa);
        tmem_st32(tM + 224, oa);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sm.qt_full[wg]);
      }
      for (int t = 0; t < T; ++t) {
        if (!bounded_wait(&sm.sp_full[wg], (g + t) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t s[64], dp[64];
        tmem_ld32(tM, s);
        tmem_ld32(tM + 32, s + 32);
        tmem_ld32(tM + 64, dp);
        tmem_ld32(tM + 96, dp + 32);
        tmem_ld_wait();
        reg_fence<64>(s);
        reg_fence<64>(dp);
        // s[i] is read at step i/2 <= i, so packing in place never overwrites an unread value
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float p0 = ex2_approx(__uint_as_float(s[2 * i]) * p.scale_log2 - lse_r);
          const float p1 = ex2_approx(__uint_as_float(s[2 * i + 1]) * p.scale_log2 - lse_r);
          s[i] = pack_bf16x2(p0 * (__uint_as_float(dp[2 * i]) - d_r), p1 * (__uint_as_float(dp[2 * i + 1]) - d_r));
        }
        tmem_st32(tM, s);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sm.ds_full[wg]);
      }
      if (!ok) break;
      if (T > 0) {
        if (!bounded_wait(&sm.dq_done[wg], it & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      uint4* dst = reinterpret_cast<uint4*>(p.dq + ri * 64);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t o[32];
        if (T > 0) {
          tmem_ld32(tM + 128 + 32 * half, o);
          tmem_ld_wait();
          reg_fence<32>(o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(o[8 * i + 0]) * p.scale, __uint_as_float(o[8 * i + 1]) * p.scale);
          w.y = pack_bf16x2(__uint_as_float(o[8 * i + 2]) * p.scale, __uint_as_float(o[8 * i + 3]) * p.scale);
          w.z = pack_bf16x2(__uint_as_float(o[8 * i + 4]) * p.scale, __uint_as_float(o[8 * i + 5]) * p.scale);
          w.w = pack_bf16x2(__uint_as_float(o[8 * i + 6]) * p.scale, __uint_as_float(o[8 * i + 7]) * p.scale);
          if (live) dst[4 * half + i] = w;
        }
      }
      g += T;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================ dK, dV
constexpr int kStagesKv = 4;
constexpr int kChunkBytes = 4 * kBox;  // Q chunk (2 boxes) + dO chunk (2 boxes)

struct DkvParams {
  CUtensorMap tm_q, tm_do;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const int* offs;
  const int* list;
  const int* ucount;  // q blocks per 128-key tile
  const float* lse;
  const float* delta;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int* status;
  int B, N, Hq, Hk, bs, K, nkb;
  float scale, scale_log2;
  int ktiles, units;
};

struct DkvSmem {
  uint64_t ch_full[kStagesKv], ch_empty[kStagesKv];
  uint64_t kvt_full, sp_full[2], ps_full[2], acc_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int mask[kStagesKv];  // per chunk: bit s set = the q block selected key segment s
  alignas(16) float nlse[kStagesKv][128];  // -lse of the chunk's 128 query rows
  alignas(16) float ndl[kStagesKv][128];   // -D of the chunk's 128 query rows
};

constexpr size_t kDkvSmemBytes = 1024 + kStagesKv * kChunkBytes + sizeof(DkvSmem);

// TMEM (lanes = the 128 keys of the tile): S^T at 0 and dP^T at 128, 128 columns each
// (one per query row of the chunk: 64 queries of head 2j, then 64 of head 2j+1).
// Column half hf of S^T is overwritten by P^T as bf16 pairs at 64 hf + [0, 32), of
// dP^T by dS^T at 128 + 64 hf + [0, 32). dV accumulates at 256, dK at 320. The tile's
// K and V rows sit at 384 and 416 as bf16 pairs, written once per unit by the row
// threads: the A operands of S^T = K Q^T and dP^T = V dO^T, which therefore read only
// Q / dO from shared memory.
__global__ void __launch_bounds__(kThreadsBwd, 1) dkv_kernel(const __grid_constant__ DkvParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sC = tiles;  // stages: Q chunk (2 boxes) then dO chunk (2 boxes)
  DkvSmem& sm = *reinterpret_cast<DkvSmem*>(sC + kStagesKv * kChunkBytes);
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.Hq / p.Hk;
  // chunks per q block: 64-query sub-tiles x head pairs (with an odd G the last pair
  // has one head; its second half loads zeros and takes lse = D = 0, adding nothing)
  const int HP = (G + 1) / 2;
  const int per_qb = (p.bs / 64) * HP;

  if (threadIdx.x == 0) {
    mbar_init(&sm.kvt_full, 256);
    for (int s = 0; s < kStagesKv; ++s) {
      mbar_init(&sm.ch_full[s], 1);
      mbar_init(&sm.ch_empty[s], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&sm.sp_full[h], 1);
      mbar_init(&sm.ps_full[h], 128);
    }
    mbar_init(&sm.acc_full, 1);
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

  // Units whose tile no q block selected have no chunks: every role skips their
  // pipeline (the row threads write zero gradients), so the barriers only count
  // units with chunks ("live" units).
  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    int gc = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
      if (p.ucount[u] == 0) continue;
      const KeyTile kt = decode_key_tile(u, p.ktiles, p.Hk, p.N, p.bs);
      UnionWalk walk = make_walk(p.offs, p.list, kt, p.Hk, p.nkb, p.K);
      int qb, mk;
      while (ok && walk.next(qb, mk)) {
        for (int cq = 0; cq < per_qb; ++cq, ++gc) {
          const int hp = cq % HP, qs = cq / HP;
          const bool second = 2 * hp + 1 < G;
          const int st = gc % kStagesKv, r = gc / kStagesKv;
          if (r > 0 && !warp_wait(&sm.ch_empty[st], (r - 1) & 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          const int nbase = qb * p.bs + qs * 64;
          const int head0 = kt.h * G + 2 * hp;
          float lv[4], dv[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int e = lane + 32 * j;
            const size_t ri = (static_cast<size_t>(kt.b) * p.N + nbase + (e & 63)) * p.Hq + head0 + (e >> 6);
            const bool row_live = (e >> 6) == 0 || second;
            lv[j] = row_live ? p.lse[ri] : 0.f;
            dv[j] = row_live ? p.delta[ri] : 0.f;
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sm.nlse[st][lane + 32 * j] = -lv[j];
            sm.ndl[st][lane + 32 * j] = -dv[j];
          }
          if (lane == 0) sm.mask[st] = mk;
          __syncwarp();
          mbar_arrive_expect_tx_elect(&sm.ch_full[st], kChunkBytes);
          uint8_t* dst = sC + st * kChunkBytes;
          for (int v = 0; v < 2; ++v) {
            const int col = (v == 0 || second) ? (head0 + v) * 64 : p.Hq * 64;  // outside the tensor: zeros
            tma_load_2d_elect(dst + v * kBox, &p.tm_q, &sm.ch_full[st], col, kt.b * p.N + nbase);
            tma_load_2d_elect(dst + (2 + v) * kBox, &p.tm_do, &sm.ch_full[st], col, kt.b * p.N + nbase);
          }
        }
      }
    }
    if (lane == 0) {
      for (int s = 0; s < kStagesKv && s < gc; ++s) {
        const int g_last = s + kStagesKv * ((gc - 1 - s) / kStagesKv);
        wait_noabort_b(&sm.ch_full[s], (g_last / kStagesKv) & 1, p.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // Each chunk is two halves h (the 64 query rows of head 2j + h). Once warpgroup h
    // has turned half h of chunk c into P^T / dS^T, the warp issues its dV / dK MMAs and
    // then S^T / dP^T of half h of chunk c + 1, so one warpgroup works on chunk c + 1
    // while the other finishes chunk c.
    const uint32_t id_s = make_idesc_bf16(128, 64, false);
    const uint32_t id_acc = make_idesc_bf16(128, 64, true);
    const uint32_t sCa = smem_u32(sC);
    // S^T_h = K Q_h^T and dP^T_h = V dO_h^T of the chunk in stage st (K, V from TMEM)
    auto issue_ss = [&](int h, int st) {
      const uint32_t cq = sCa + st * kChunkBytes + h * kBox, cdo = cq + 2 * kBox;
      const uint64_t qk = sw128_desc(cq, 1024, 16), dok = sw128_desc(cdo, 1024, 16);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_ts_elect(tmem + 64u * h, tmem + 384u + 8u * ks, qk + static_cast<uint64_t>(2 * ks), id_s,
                     ks > 0 ? 1u : 0u);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_ts_elect(tmem + 128u + 64u * h, tmem + 416u + 8u * ks, dok + static_cast<uint64_t>(2 * ks), id_s,
                     ks > 0 ? 1u : 0u);
      tc_commit_elect(&sm.sp_full[h]);
    };
    // dV += P^T_h dO_h and dK += dS^T_h Q_h (P^T_h / dS^T_h as bf16 pairs in TMEM)
    auto issue_ts = [&](int h, int st, bool first) {
      const uint32_t cq = sCa + st * kChunkBytes + h * kBox, cdo = cq + 2 * kBox;
      const uint64_t qmn = sw128_desc(cq, 1024, 16384), domn = sw128_desc(cdo, 1024, 16384);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_ts_elect(tmem + 256, tmem + 64u * h + 8u * ks, domn + static_cast<uint64_t>(ks * 128), id_acc,
                     (first && ks == 0) ? 0u : 1u);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_ts_elect(tmem + 320, tmem + 128u + 64u * h + 8u * ks, qmn + static_cast<uint64_t>(ks * 128), id_acc,
                     (first && ks == 0) ? 0u : 1u);
    };
    int gc = 0, live = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
      const int nch = p.ucount[u] * per_qb;
      if (nch == 0) continue;
      // kvt_full: the rows have written this tile's K / V into TMEM, after reading the
      // previous live unit's dK / dV (so those may be overwritten too).
      ok = warp_wait(&sm.kvt_full, live & 1, abort_flag, p.status) &&
           warp_wait(&sm.ch_full[gc % kStagesKv], (gc / kStagesKv) & 1, abort_flag, p.status);
      tc_fence_after();
      if (!ok) break;
      issue_ss(0, gc % kStagesKv);
      issue_ss(1, gc % kStagesKv);
      for (int c = 0; ok && c < nch; ++c) {
        const int g = gc + c, st = g % kStagesKv;
        for (int h = 0; ok && h < 2; ++h) {
          ok = warp_wait(&sm.ps_full[h], g & 1, abort_flag, p.status);
          tc_fence_after();
          if (!ok) break;
          issue_ts(h, st, c == 0 && h == 0);
          if (c + 1 < nch) {
            // S^T_h / dP^T_h of the next chunk overwrite the P^T_h / dS^T_h that the
            // MMAs above read; tcgen05.mma executes in issue order.
            if (h == 0) {
              ok = warp_wait(&sm.ch_full[(g + 1) % kStagesKv], ((g + 1) / kStagesKv) & 1, abort_flag, p.status);
              tc_fence_after();
              if (!ok) break;
            }
            issue_ss(h, (g + 1) % kStagesKv);
          }
        }
        if (ok) tc_commit_elect(&sm.ch_empty[st]);  // every read of this chunk's stage is issued
      }
      if (!ok) break;
      tc_commit_elect(&sm.acc_full);  // every MMA of the unit, K / V reads included
      ++live;
      gc += nch;
    }
    tc_commit_elect(&sm.drain);
    if (lane == 0) wait_noabort_b(&sm.drain, 0, p.status);
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- P^T / dS^T, one key row x one column half per thread;
    // epilogue: warpgroup 0 writes dV, warpgroup 1 dK
    const int hf = (warp - 4) >> 2, qd = warp & 3;
    const int kr = qd * 32 + lane;  // key row of the tile = TMEM lane
    const int seg = kr >> 6;
    const uint32_t tT = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    int gc = 0, live = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
      const KeyTile kt = decode_key_tile(u, p.ktiles, p.Hk, p.N, p.bs);
      const int nch = p.ucount[u] * per_qb;
      const int key = kt.key0 + kr;
      if (nch > 0) {
        // This key's K row (warpgroup 0) or V row (warpgroup 1) into TMEM. Every MMA of
        // the previous live unit has completed: its epilogue below waited for acc_full.
        uint32_t kv[32];
        if (key < p.N) {
          const uint4* src = reinterpret_cast<const uint4*>(
              (hf == 0 ? p.k : p.v) + ((static_cast<size_t>(kt.b) * p.N + key) * p.Hk + kt.h) * 64);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 x = __ldg(src + i);
            kv[4 * i] = x.x; kv[4 * i + 1] = x.y; kv[4 * i + 2] = x.z; kv[4 * i + 3] = x.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) kv[i] = 0u;
        }
        tmem_st32(tT + 384 + 32 * hf, kv);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sm.kvt_full);
      }
      for (int c = 0; c < nch; ++c, ++gc) {
        const int st = gc % kStagesKv;
        // ch_full orders the producer's lse / D / mask writes before these reads
        if (!bounded_wait(&sm.ch_full[st], (gc / kStagesKv) & 1, abort_flag, p.status) ||
            !bounded_wait(&sm.sp_full[hf], gc & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const bool on = (sm.mask[st] >> seg) & 1;
        // Two 32-column quarters of this half; quarter j's P^T / dS^T pairs land in
        // columns 16j..16j+15 of the half, which quarter 0 has already read.
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t s[32], dp[32];
          tmem_ld32(tT + 64 * hf + 32 * j, s);
          tmem_ld32(tT + 128 + 64 * hf + 32 * j, dp);
          tmem_ld_wait();
          reg_fence<32>(s);
          reg_fence<32>(dp);
          if (on) {
            p_ds_quarter(s, dp, sm.nlse[st] + 64 * hf + 32 * j, sm.ndl[st] + 64 * hf + 32 * j, p.scale_log2);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) s[i] = dp[i] = 0u;
          }
          tmem_st16(tT + 64 * hf + 16 * j, s);
          tmem_st16(tT + 128 + 64 * hf + 16 * j, dp);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sm.ps_full[hf]);
      }
      if (!ok) break;
      uint32_t o[64];
      if (nch > 0) {
        if (!bounded_wait(&sm.acc_full, live & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_ld32(tT + 256 + 64 * hf, o);
        tmem_ld32(tT + 256 + 64 * hf + 32, o + 32);
        tmem_ld_wait();
        reg_fence<64>(o);
        ++live;
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) o[i] = 0u;
      }
      if (key < p.N) {
        const float f = hf == 0 ? 1.0f : p.scale;
        __nv_bfloat16* out = hf == 0 ? p.dv : p.dk;
        uint4* dst = reinterpret_cast<uint4*>(out + ((static_cast<size_t>(kt.b) * p.N + key) * p.Hk + kt.h) * 64);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(o[8 * i + 0]) * f, __uint_as_float(o[8 * i + 1]) * f);
          w.y = pack_bf16x2(__uint_as_float(o[8 * i + 2]) * f, __uint_as_float(o[8 * i + 3]) * f);
          w.z = pack_bf16x2(__uint_as_float(o[8 * i + 4]) * f, __uint_as_float(o[8 * i + 5]) * f);
          w.w = pack_bf16x2(__uint_as_float(o[8 * i + 6]) * f, __uint_as_float(o[8 * i + 7]) * f);
          dst[i] = w;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <typename F>
int set_smem(F* fn, size_t bytes, bool* done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOSAIC_ERR_CUDA;
  if (!done[dev]) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) !=
        cudaSuccess)
      return MOSAIC_ERR_CUDA;
    done[dev] = true;
  }
  return MOSAIC_OK;
}

int sm_count_cached() {
  static int count[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (count[dev] == 0 && cudaDeviceGetAttribute(&count[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  return count[dev];
}

}  // namespace

int sparse_bwd_max_selected() { return kMaxSelB; }

SparseBwdWorkspace sparse_bwd_workspace(int B, int N, int Hq, int Hk, int bs, int K) {
  SparseBwdWorkspace w;
  const size_t nkb = bs > 0 ? static_cast<size_t>(N) / bs : 0;
  const size_t bh = static_cast<size_t>(B) * Hk;
  const size_t units = bh * ((static_cast<size_t>(N) + 127) / 128);
  auto r256 = [](size_t x) { return (x + 255) & ~size_t(255); };
  size_t off = 0;
  w.delta = off;  off += r256(static_cast<size_t>(B) * N * Hq * sizeof(float));
  w.count = off;  off += r256(bh * nkb * sizeof(int));
  w.cursor = off; off += r256(bh * nkb * sizeof(int));
  w.offs = off;   off += r256(bh * (nkb + 1) * sizeof(int));
  w.list = off;   off += r256(bh * nkb * K * sizeof(int));
  w.sorted = off; off += r256(bh * nkb * K * sizeof(int));
  w.ucount = off; off += r256(units * sizeof(int));
  w.total = off;
  return w;
}

int launch_sparse_bwd(const SparseBwdLaunch& a, cudaStream_t stream) {
  const int B = a.B, N = a.N, Hq = a.Hq, Hk = a.Hk, bs = a.bs, K = a.K;
  const int nkb = N / bs;
  const SparseBwdWorkspace ws = sparse_bwd_workspace(B, N, Hq, Hk, bs, K);
  uint8_t* w = static_cast<uint8_t*>(a.workspace);
  float* delta = reinterpret_cast<float*>(w + ws.delta);
  int* count = reinterpret_cast<int*>(w + ws.count);
  int* cursor = reinterpret_cast<int*>(w + ws.cursor);
  int* offs = reinterpret_cast<int*>(w + ws.offs);
  int* list = reinterpret_cast<int*>(w + ws.list);
  int* sorted = reinterpret_cast<int*>(w + ws.sorted);
  int* ucount = reinterpret_cast<int*>(w + ws.ucount);
  const size_t bh = static_cast<size_t>(B) * Hk;
  const int ktiles = (N + 127) / 128;
  const int kv_units = static_cast<int>(bh) * ktiles;

  // D
  const long long rows = static_cast<long long>(B) * N * Hq;
  delta_kernel<<<static_cast<unsigned>((rows * 8 + 255) / 256), 256, 0, stream>>>(
      static_cast<const uint4*>(a.out), static_cast<const uint4*>(a.grad_out), delta, rows);
  // inverted index
  if (cudaMemsetAsync(count, 0, bh * nkb * sizeof(int), stream) != cudaSuccess ||
      cudaMemsetAsync(cursor, 0, bh * nkb * sizeof(int), stream) != cudaSuccess)
    return MOSAIC_ERR_CUDA;
  const long long qrows = static_cast<long long>(B) * nkb * Hk;
  const unsigned qgrid = static_cast<unsigned>((qrows + 255) / 256);
  idx_count_kernel<<<qgrid, 256, 0, stream>>>(a.block_idx, count, B, nkb, Hk, K, nkb, a.status);
  idx_scan_kernel<<<static_cast<unsigned>(bh), 1024, 0, stream>>>(count, offs, nkb);
  idx_fill_kernel<<<qgrid, 256, 0, stream>>>(a.block_idx, offs, cursor, list, B, nkb, Hk, K, nkb);
  idx_sort_kernel<<<static_cast<unsigned>(bh * nkb), 128, 0, stream>>>(offs, list, sorted, nkb, K);
  idx_union_kernel<<<static_cast<unsigned>((kv_units + 127) / 128), 128, 0, stream>>>(
      offs, sorted, ucount, kv_units, ktiles, Hk, N, bs, nkb, K);
  if (cudaGetLastError() != cudaSuccess) return MOSAIC_ERR_CUDA;

  const int sms = sm_count_cached();
  if (sms <= 0) return MOSAIC_ERR_CUDA;
  const float scale = a.softmax_scale;
  const float scale_log2 = scale * 1.4426950408889634f;
  CUtensorMap tm_q, tm_do, tm_k, tm_v;
  if (make_tmap_bf16_2d(&tm_q, a.q, static_cast<uint64_t>(B) * N, static_cast<uint64_t>(Hq) * 64) ||
      make_tmap_bf16_2d(&tm_do, a.grad_out, static_cast<uint64_t>(B) * N, static_cast<uint64_t>(Hq) * 64) ||
      make_tmap_bf16_2d(&tm_k, a.k, static_cast<uint64_t>(B) * N, static_cast<uint64_t>(Hk) * 64) ||
      make_tmap_bf16_2d(&tm_v, a.v, static_cast<uint64_t>(B) * N, static_cast<uint64_t>(Hk) * 64))
    return MOSAIC_ERR_CUDA;
  const __nv_bfloat16* kb = static_cast<const __nv_bfloat16*>(a.k);
  const __nv_bfloat16* vb = static_cast<const __nv_bfloat16*>(a.v);
  // dQ
  {
    DqParams p;
    memset(&p, 0, sizeof(p));
    p.tm_q = tm_q; p.tm_do = tm_do; p.tm_k = tm_k; p.tm_v = tm_v;
    p.block_idx = a.block_idx;
    p.lse = a.lse;
    p.delta = delta;
    p.dq = static_cast<__nv_bfloat16*>(a.grad_q);
    p.status = a.status;
    p.B = B; p.N = N; p.Hq = Hq; p.Hk = Hk; p.bs = bs; p.K = K;
    p.nqb = nkb; p.nkb = nkb;
    p.scale = scale; p.scale_log2 = scale_log2;
    p.ngroups = (Hq / Hk + 3) / 4;
    p.qtiles = N / 64;
    p.units = B * Hk * p.ngroups * p.qtiles;
    static bool done[64] = {};
    int rc = set_smem(dq_kernel, kDqSmemBytes, done);
    if (rc) return rc;
    const int grid = p.units < sms ? p.units : sms;
    if (grid > 0) dq_kernel<<<grid, kThreadsBwd, kDqSmemBytes, stream>>>(p);
    if (cudaGetLastError() != cudaSuccess) return MOSAIC_ERR_CUDA;
  }
  // dK, dV
  {
    DkvParams p;
    memset(&p, 0, sizeof(p));
    p.tm_q = tm_q; p.tm_do = tm_do;
    p.k = kb; p.v = vb;
    p.offs = offs;
    p.list = sorted;
    p.ucount = ucount;
    p.lse = a.lse;
    p.delta = delta;
    p.dk = static_cast<__nv_bfloat16*>(a.grad_k);
    p.dv = static_cast<__nv_bfloat16*>(a.grad_v);
    p.status = a.status;
    p.B = B; p.N = N; p.Hq = Hq; p.Hk = Hk; p.bs = bs; p.K = K; p.nkb = nkb;
    p.scale = scale; p.scale_log2 = scale_log2;
    p.ktiles = ktiles;
    p.units = kv_units;
    static bool done[64] = {};
    int rc = set_smem(dkv_kernel, kDkvSmemBytes, done);
    if (rc) return rc;
    const int grid = p.units < sms ? p.units : sms;
    if (grid > 0) dkv_kernel<<<grid, kThreadsBwd, kDkvSmemBytes, stream>>>(p);
    if (cudaGetLastError() != cudaSuccess) return MOSAIC_ERR_CUDA;
  }
  return MOSAIC_OK;
}

}  // namespace mosaic
