// Block scores + top-k block selection on the tensor core (tcgen05), for the
// shapes where the score matrix is large (it grows as nb^2: 0.9 GFLOP at Nside 64,
// 232 GFLOP at Nside 256).
//
// Same arithmetic as topk.cu and the reference attn_topk (primitives.py:35-51):
// S_j = q_cmp[:, :, j] . k_cmp[:, :, j // G]^T in fp32, rounded to the activation
// type (bf16, or fp16 under the reference's fp16 autocast); the mean over the
// STRIDED head group j = g*Hk + h (fp32 sum of the rounded scores, divided by G,
// rounded again); the K largest per row with ties to the lower block index
// (32-bit keys: order-preserving 16-bit float bits << 16 | 65535 - block).
//
// One CTA = 128 query blocks (one M = 128 MMA tile) of one (b, h). Keys stream in
// tiles of 64 blocks: TMA brings the G kv-head rows of the tile, one elected lane
// of the MMA warp issues S_g = Q_g K_g^T for the G head slots into a TMEM buffer
// (G x 64 columns, double-buffered), and eight epilogue warps round, average and
// select: two threads per row, each owning one 32-key half of every tile and its
// own best list; the two lists of a row are merged once at the end (the K best of
// a union are the K best of the two partial K-best lists). Selection keeps each row's best keys sorted in
// registers (KP >= K of them, KP a multiple of 8; keeping more than K changes
// nothing in the first K); a key of the current tile is appended to a shared-memory
// buffer only if it beats the KP-th best, and after the tile the few appended keys
// go through a branch-free insertion network in a loop the warp runs together.
//
// Every wait is bounded (MOSAIC_STATUS_TIMEOUT on expiry, then the CTA drains and
// returns); there is no TMA multicast.
#include <cstring>

#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {

#ifdef MOSAIC_TRACE
// Development timeline (off in the library build), shared with the engine's.
extern __device__ long long g_engine_trace[4096];
#define TOPK_TRACE_AT(cond, slot) \
  do {                            \
    if (cond) g_engine_trace[(slot)] = clock64(); \
  } while (0)
#else
#define TOPK_TRACE_AT(cond, slot) \
  do {                            \
    (void)(cond);                 \
  } while (0)
#endif

namespace {

constexpr int kRowsTc = 128;    // query blocks per CTA
constexpr int kKeysTc = 64;     // key blocks per tile
constexpr int kStagesTc = 4;
constexpr int kMaxGTc = 4;
constexpr int kMaxKTc = 32;
constexpr int kThreadsTc = 384; // warp 0 TMA, warp 1 MMA, warps 2-3 idle, warps 4-11 epilogue
constexpr int kBox = 64 * 128;  // one 64-row x 64-col bf16 box

struct TopkTcParams {
  CUtensorMap tm_q, tm_k;
  int64_t* idx;
  int* status;
  int B, nb, Hq, Hk, K, G;
};

struct TopkTcSmem {
  uint64_t q_full;
  uint64_t kv_full[kStagesTc];
  uint64_t kv_empty[kStagesTc];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  // per (key half, row): one tile's new candidates, and at the end the row's
  // partial best list (+1: rows start in different banks)
  uint32_t cand[2][kRowsTc][32 + 1];
};

constexpr size_t kTcSmemBytes =
    1024 + kMaxGTc * 2 * kBox + kStagesTc * kMaxGTc * kBox + sizeof(TopkTcSmem);

template <bool kF16>
__device__ __forceinline__ uint32_t order_key_tc(float t, int block) {
  uint32_t u = Act<kF16>::bits(t);
  if (u == 0x8000u) u = 0;  // -0 ties with +0, as in torch.topk
  const uint32_t ord = (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
  return (ord << 16) | (0xFFFFu - static_cast<uint32_t>(block));
}

// Inserts key into the descending register list L[0..KP) (dropping the smallest):
// L'[p] = key > L[p-1] ? L[p-1] : max(L[p], key), from the bottom up.
template <int KP>
__device__ __forceinline__ void insert_sorted(uint32_t (&L)[KP], uint32_t key) {
#pragma unroll
  for (int p = KP - 1; p > 0; --p) L[p] = key > L[p - 1] ? L[p - 1] : max(L[p], key);
  L[0] = max(L[0], key);
}

__device__ __forceinline__ void g_na_max_trace(int t, int v) {
#ifdef MOSAIC_TRACE
  g_engine_trace[2000 + 10 + t] = v;
#else
  (void)t;
  (void)v;
#endif
}

__device__ __forceinline__ bool wait_noabort_tc(uint64_t* bar, uint32_t parity, int* status) {
  int dummy = 0;
  return bounded_wait(bar, parity, &dummy, status);
}

template <int KP, int G, bool kF16>
__global__ void __launch_bounds__(kThreadsTc, 1) topk_tc_kernel(const __grid_constant__ TopkTcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = tiles;                           // G slots x 2 boxes (128 rows)
  uint8_t* sK = tiles + kMaxGTc * 2 * kBox;      // stages x G slots x 1 box (64 keys)
  TopkTcSmem& sm = *reinterpret_cast<TopkTcSmem*>(sK + kStagesTc * kMaxGTc * kBox);
  volatile int* abort_flag = &sm.abort_flag;
  // The next kernel of the stream (the attention engine) reads the indices this
  // kernel writes, so it is not released early.

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i0 = blockIdx.x * kRowsTc, h = blockIdx.y, b = blockIdx.z;
  const int T = (p.nb + kKeysTc - 1) / kKeysTc;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStagesTc; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&sm.s_full[j], 1);
      mbar_init(&sm.s_free[j], 256);  // the 8 epilogue warps
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
  bool epi_ok = false;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_k);
    }
    // Q of the G head slots g*Hk + h: rows i0 .. i0+127 (out-of-range rows read 0)
    mbar_arrive_expect_tx_elect(&sm.q_full, G * 2 * kBox);
    for (int g = 0; g < G; ++g)
      for (int r = 0; r < 2; ++r)
        tma_load_2d_elect(sQ + (2 * g + r) * kBox, &p.tm_q, &sm.q_full, (g * p.Hk + h) * 64,
                          b * p.nb + i0 + 64 * r);
    bool ok = true;
    for (int t = 0; ok && t < T; ++t) {
      const int st = t % kStagesTc, r = t / kStagesTc;
      if (r > 0 && !warp_wait(&sm.kv_empty[st], (r - 1) & 1, abort_flag, p.status)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx_elect(&sm.kv_full[st], G * kBox);
      for (int g = 0; g < G; ++g)
        tma_load_2d_elect(sK + (st * kMaxGTc + g) * kBox, &p.tm_k, &sm.kv_full[st], ((g * p.Hk + h) / G) * 64,
                          b * p.nb + t * kKeysTc);
    }
    // every TMA write into shared memory must land before the CTA exits
    if (lane == 0) {
      wait_noabort_tc(&sm.q_full, 0, p.status);
      for (int s = 0; s < kStagesTc && s < T; ++s) {
        const int t_last = s + kStagesTc * ((T - 1 - s) / kStagesTc);
        wait_noabort_tc(&sm.kv_full[s], (t_last / kStagesTc) & 1, p.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    const uint32_t idesc = make_idesc(128, kKeysTc, false, Act<kF16>::kMmaFmt);
    const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK);
    bool ok = warp_wait(&sm.q_full, 0, abort_flag, p.status);
    tc_fence_after();
    for (int t = 0; ok && t < T; ++t) {
      const int st = t % kStagesTc, buf = t & 1;
      if (t >= 2 && !warp_wait(&sm.s_free[buf], ((t - 2) >> 1) & 1, abort_flag, p.status)) {
        ok = false;
        break;
      }
      if (!warp_wait(&sm.kv_full[st], (t / kStagesTc) & 1, abort_flag, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int g = 0; g < G; ++g) {
        const uint64_t qd = sw128_desc(sQa + 2 * g * kBox, 1024, 16);
        const uint64_t kd = sw128_desc(sKa + (st * kMaxGTc + g) * kBox, 1024, 16);
        const uint32_t tS = tmem + 256u * buf + 64u * g;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_ss_elect(tS, qd + static_cast<uint64_t>(2 * ks), kd + static_cast<uint64_t>(2 * ks), idesc,
                       ks > 0 ? 1u : 0u);
      }
      tc_commit_elect(&sm.s_full[buf]);
      tc_commit_elect(&sm.kv_empty[st]);
      TOPK_TRACE_AT(blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && lane == 0 && t < 96, 3600 + t);
    }
    tc_commit_elect(&sm.drain);
    if (lane == 0) wait_noabort_tc(&sm.drain, 0, p.status);
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- epilogue: two threads per row
    const int qd = warp & 3;              // TMEM lane quadrant of the warp
    const int ch = (warp - 4) >> 2;       // key half of every tile this warp owns
    const int row = qd * 32 + lane;
    const int i = i0 + row;
    const bool live = i < p.nb;
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    uint32_t* cand = sm.cand[ch][row];  // this tile's keys that beat the KP-th best
    constexpr float kInvG = 1.0f / static_cast<float>(G);  // G in {1, 2, 4}: t / G == t * (1/G) exactly
    uint32_t L[KP];  // best keys, descending (0 = empty: every real key is > 0)
#pragma unroll
    for (int q = 0; q < KP; ++q) L[q] = 0;
    bool ok = true;
    for (int t = 0; ok && t < T; ++t) {
      const int buf = t & 1;
      const bool rec = blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && row == 0 && ch == 0 && t < 96;
      TOPK_TRACE_AT(rec, 2500 + 5 * t + 0);
      if (!bounded_wait(&sm.s_full[buf], (t >> 1) & 1, abort_flag, p.status)) {
        ok = false;
        break;
      }
      TOPK_TRACE_AT(rec, 2500 + 5 * t + 1);
      tc_fence_after();
      // fp32 sum over the head slots of the bf16-rounded scores; the next slot's
      // TMEM load is in flight while this slot's values are added
      float tsum[32];
      uint32_t va[32], vb[32];
      const uint32_t tS = tmem + lane_off + 256u * buf + 32u * ch;
      tmem_ld32(tS, va);
      tmem_ld_wait();
      reg_fence<32>(va);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        uint32_t(&cur)[32] = (g & 1) ? vb : va;
        uint32_t(&nxt)[32] = (g & 1) ? va : vb;
        if (g + 1 < G) tmem_ld32(tS + 64u * (g + 1), nxt);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float r = Act<kF16>::round(__uint_as_float(cur[j]));
          tsum[j] = g == 0 ? r : tsum[j] + r;
        }
        if (g + 1 < G) {
          tmem_ld_wait();
          reg_fence<32>(nxt);
        }
      }
      // S of this tile has been read: the MMA warp may reuse the buffer
      tc_fence_before();
      mbar_arrive(&sm.s_free[buf]);
      TOPK_TRACE_AT(rec, 2500 + 5 * t + 2);
      // append this half-tile's keys that beat the KP-th best so far; each key's
      // slot is the number of qualifying keys before it (no serial counter)
      const uint32_t thr = L[KP - 1];
      const int key0 = t * kKeysTc + 32 * ch;
      uint32_t keys[32];
      uint32_t mask = 0;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        keys[j] = order_key_tc<kF16>(tsum[j] * kInvG, key0 + j);
        const bool take = live && key0 + j < p.nb && keys[j] > thr;
        mask |= static_cast<uint32_t>(take) << j;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if ((mask >> j) & 1) cand[__popc(mask & ((1u << j) - 1))] = keys[j];
      const int na = __popc(mask);
      // merge them; the warp runs the longest merge together
      const int na_max = __reduce_max_sync(0xffffffffu, na);
      TOPK_TRACE_AT(rec, 2500 + 5 * t + 3);
      if (rec) g_na_max_trace(t, na_max);
      for (int a = 0; a < na_max; ++a) {
        const uint32_t key = a < na ? cand[a] : 0u;  // 0 changes nothing
        insert_sorted<KP>(L, key);
      }
      TOPK_TRACE_AT(rec, 2500 + 5 * t + 4);
    }
    // this half's best list, for the merge after the CTA barrier
#pragma unroll
    for (int q = 0; q < KP; ++q) cand[q] = L[q];
    epi_ok = ok;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  // the K best of a row = the K best of its two half lists (both descending)
  if (warp >= 4 && warp < 8 && epi_ok && !*abort_flag) {
    const int row = (warp & 3) * 32 + lane;
    const int i = i0 + row;
    if (i < p.nb) {
      const uint32_t* A = sm.cand[0][row];
      const uint32_t* Bl = sm.cand[1][row];
      int ia = 0, ib = 0;
      int64_t* dst = p.idx + ((static_cast<size_t>(b) * p.nb + i) * p.Hk + h) * p.K;
      for (int q = 0; q < p.K; ++q) {
        const uint32_t a = ia < KP ? A[ia] : 0u, c = ib < KP ? Bl[ib] : 0u;
        const uint32_t x = a > c ? a : c;
        if (a > c) ++ia; else ++ib;
        dst[q] = static_cast<int64_t>(0xFFFFu - (x & 0xFFFFu));
      }
    }
  }
  // Complete only after the coarse attention launched before this kernel, so that
  // a kernel waiting on this grid also sees the coarse-attention output.
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <int KP, int G, bool kF16>
int launch_kp(const TopkTcParams& p, const TopkLaunch& a, cudaStream_t stream) {
  static bool attr_done[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOSAIC_ERR_CUDA;
  if (!attr_done[dev]) {
    if (cudaFuncSetAttribute(topk_tc_kernel<KP, G, kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kTcSmemBytes)) != cudaSuccess)
      return MOSAIC_ERR_CUDA;
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.nb + kRowsTc - 1) / kRowsTc, a.Hk, a.B);
  cfg.blockDim = dim3(kThreadsTc);
  cfg.dynamicSmemBytes = kTcSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.overlap_previous ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, topk_tc_kernel<KP, G, kF16>, p) == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

template <int G, bool kF16>
int launch_g(const TopkTcParams& p, const TopkLaunch& a, cudaStream_t stream) {
  switch ((a.K + 7) / 8) {
    case 1: return launch_kp<8, G, kF16>(p, a, stream);
    case 2: return launch_kp<16, G, kF16>(p, a, stream);
    case 3: return launch_kp<24, G, kF16>(p, a, stream);
    case 4: return launch_kp<32, G, kF16>(p, a, stream);
    default: return MOSAIC_ERR_UNSUPPORTED;
  }
}

template <bool kF16>
int launch_typed(const TopkTcParams& p, const TopkLaunch& a, cudaStream_t stream) {
  return p.G == 4 ? launch_g<4, kF16>(p, a, stream)
                  : p.G == 2 ? launch_g<2, kF16>(p, a, stream) : launch_g<1, kF16>(p, a, stream);
}

}  // namespace

bool topk_tc_supported(const TopkLaunch& a) {
  const int G = a.Hk > 0 ? a.Hq / a.Hk : 0;
  return (G == 1 || G == 2 || G == 4) && a.K >= 1 && a.K <= kMaxKTc && a.nb <= 65535;
}

int launch_topk_tc(const TopkLaunch& a, cudaStream_t stream) {
  TopkTcParams p;
  memset(&p, 0, sizeof(p));
  if (make_tmap_2d(&p.tm_q, a.q_cmp, static_cast<uint64_t>(a.B) * a.nb, static_cast<uint64_t>(a.Hq) * 64, a.f16) ||
      make_tmap_2d(&p.tm_k, a.k_cmp, static_cast<uint64_t>(a.B) * a.nb, static_cast<uint64_t>(a.Hk) * 64, a.f16))
    return MOSAIC_ERR_CUDA;
  p.idx = a.idx;
  p.status = a.status;
  p.B = a.B;
  p.nb = a.nb;
  p.Hq = a.Hq;
  p.Hk = a.Hk;
  p.K = a.K;
  p.G = a.Hq / a.Hk;
  return a.f16 ? launch_typed<true>(p, a, stream) : launch_typed<false>(p, a, stream);
}

}  // namespace mosaic
