// Block scores + top-k block selection for Mosaic's selected branch.
//
// Reference attn_topk (primitives.py:35-51):
//   k = k_cmp.repeat_interleave(G, dim=2)              -> q head j uses kv head j // G
//   S_j = q_cmp[:, :, j] @ k[:, :, j]^T                (matmul in the activation type, bf16
//                                                       or fp16 under autocast: fp32 sum,
//                                                       result rounded to that type)
//   T_h = mean_g S_{g*Hk + h}                          ('b (g h) t k -> b h t k': a STRIDED
//                                                       head group; fp32 sum, rounded again)
//   idx[b, i, h, :] = topk(T_h[i, :], K, largest)      (int64)
// The strided group is what the reference computes even though the sparse kernel
// then uses idx[..., h, :] for the contiguous heads h*G .. h*G+G-1 (ops.py:49);
// this kernel reproduces it on purpose.
//
// Each score becomes the 32-bit key (order-preserving 16-bit float bits << 16) |
// (65535 - block): keys are unique, their order is score descending with ties to
// the lower block index (torch.topk's usual order), and the top-K of a row is
// exactly the K largest keys.
//
// One CTA = 16 query blocks of one (b, h), 16 warps. The keys stream in chunks of
// up to kChunk blocks:
//   A) scores of the chunk -> shared memory (mma.sync m16n8k16; each warp owns
//      whole 8-key column groups for all G heads, so the strided-group mean needs
//      no cross-warp reduction);
//   B) warp r owns row r: the keys of the chunk and its running top list reach a
//      threshold (the K-th largest of the lanes' maxima) that every top-K key
//      clears; the few that do are ranked against each other (K <= 32). Otherwise
//      a binary search on the key value (warp reductions) finds the K-th largest,
//      keeps the keys >= it and sorts them.
// The work is tiny (0.9 GFLOP of scores at Nside 64); the kernel is latency-bound,
// so the point of this layout is to keep many independent loads and warps in flight.
#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {
namespace {

constexpr int kRows = 16;
constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kChunk = 1024;  // key blocks scored per pass
constexpr int kMaxG = 8;
constexpr int kMaxK = 128;
constexpr int kTcMinBlocks = 2048;

struct TopkParams {
  const uint16_t* q_cmp;  // bf16 or fp16 bits
  const uint16_t* k_cmp;
  int64_t* idx;
  int B, nb, Hq, Hk, K, G;
};

struct TopkSmem {
  uint16_t qs[kMaxG][kRows][64];       // 16 KB
  uint32_t keys[kRows][kChunk];        // 64 KB
  uint32_t top[kRows][kMaxK];          // 8 KB  running top list per row (sorted descending)
  uint32_t buf[kWarps][kMaxK];         // 8 KB  per-warp selection buffers
};

// Logical k index of the m16n8k16 fragments -> physical head-dim index. Thread
// (lane & 3) == gc holds logical k in {16ks + 2gc + {0,1,8,9}} (ks = 0..3); they map
// to the contiguous physical range [16gc, 16gc + 16).
__device__ __forceinline__ int perm_d(int kk) {
  const int ks = kk >> 4, w = kk & 15;
  const int gc = (w & 7) >> 1;
  const int q = (w & 1) | ((w >> 3) << 1);  // e in {0,1,8,9} -> 0..3
  return 16 * gc + 4 * ks + q;
}

// The score rounded to the activation type, as a key whose unsigned order is the
// score order; bf16 and fp16 are both sign-magnitude, so one transform serves both.
template <bool kF16>
__device__ __forceinline__ uint32_t order_key(float t, int block) {
  uint32_t u = Act<kF16>::bits(t);
  if (u == 0x8000u) u = 0;  // -0 ties with +0, as in torch.topk
  const uint32_t ord = (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
  return (ord << 16) | (0xFFFFu - static_cast<uint32_t>(block));
}

template <bool kF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (kF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// A fragments of the 16 rows for head slot g (loaded once per chunk).
// For G > 4 the fragments would not fit the register budget next to the B
// fragments, so they are cached for G <= 4 only.
constexpr int kCachedG = 4;
template <int G>
struct AFrags {
  uint32_t a[G <= kCachedG ? G : 1][4][4];
};

template <int G>
__device__ __forceinline__ void load_afrags(const TopkSmem& sm, AFrags<G>& f, int lane) {
  if (G > kCachedG) return;
  const int gr = lane >> 2, gc = (lane & 3) * 2;
#pragma unroll
  for (int g = 0; g < (G <= kCachedG ? G : 1); ++g)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      f.a[g][ks][0] = *reinterpret_cast<const uint32_t*>(&sm.qs[g][gr][ks * 16 + gc]);
      f.a[g][ks][1] = *reinterpret_cast<const uint32_t*>(&sm.qs[g][gr + 8][ks * 16 + gc]);
      f.a[g][ks][2] = *reinterpret_cast<const uint32_t*>(&sm.qs[g][gr][ks * 16 + gc + 8]);
      f.a[g][ks][3] = *reinterpret_cast<const uint32_t*>(&sm.qs[g][gr + 8][ks * 16 + gc + 8]);
    }
}

// Scores of key group [kb0, kb0+8) for the CTA's 16 rows into keys[][col0..col0+8).
template <int G, bool kF16>
__device__ __forceinline__ void score_group(const TopkParams& p, TopkSmem& sm, const AFrags<G>& f, int b, int h,
                                            int kb0, int col0, int lane) {
  const int gr = lane >> 2, gq = lane & 3;
  const int key = kb0 + gr;
  // physical head-dim range [16 gq, 16 gq + 16) of this thread's key row = its whole B fragment
  uint4 raw[G][2];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int kv = (g * p.Hk + h) / G;
    const uint4* src =
        reinterpret_cast<const uint4*>(p.k_cmp + ((static_cast<size_t>(b) * p.nb + key) * p.Hk + kv) * 64 + 16 * gq);
    raw[g][0] = key < p.nb ? __ldg(src) : make_uint4(0, 0, 0, 0);
    raw[g][1] = key < p.nb ? __ldg(src + 1) : make_uint4(0, 0, 0, 0);
  }
  float tacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(raw[g]);  // 8 words: (ks, q-pair)
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      if (G <= kCachedG) {
        mma_16816<kF16>(d, f.a[G <= kCachedG ? g : 0][ks], w[2 * ks], w[2 * ks + 1]);
      } else {
        const int gr = lane >> 2, gc = gq * 2;
        uint32_t a[4];
        a[0] = *reinterpret_cast<const uint32_t*>(&sm.qs[g][gr][ks * 16 + gc]);
        a[1] = *reinterpret_cast<const uint32_t*>(&sm.qs[g][gr + 8][ks * 16 + gc]);
        a[2] = *reinterpret_cast<const uint32_t*>(&sm.qs[g][gr][ks * 16 + gc + 8]);
        a[3] = *reinterpret_cast<const uint32_t*>(&sm.qs[g][gr + 8][ks * 16 + gc + 8]);
        mma_16816<kF16>(d, a, w[2 * ks], w[2 * ks + 1]);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) tacc[e] += Act<kF16>::round(d[e]);
  }
  const float fg = static_cast<float>(G);
  const int gc = gq * 2;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int r = gr + (e >= 2 ? 8 : 0);
    const int c = gc + (e & 1);
    const int kb = kb0 + c;
    sm.keys[r][col0 + c] = kb < p.nb ? order_key<kF16>(__fdiv_rn(tacc[e], fg), kb) : 0u;
  }
}

// Warp-wide: the K-th largest of the distinct candidate keys held in registers
// (lane l holds candidates l, l+32, ...; absent ones are 0, below every real key),
// by binary search on the key value: 32 steps, each a count of the keys >= mid
// reduced over the warp. No shared-memory atomics, so skewed score distributions
// cost nothing extra.
template <int NV>
__device__ __forceinline__ uint32_t kth_largest(const uint32_t (&v)[NV], int K) {
  uint32_t lo = 0, hi = 0xFFFFFFFFu;  // invariant: count(>= lo) >= K, count(>= hi + 1) < K
#pragma unroll 1
  for (int step = 0; step < 32 && lo < hi; ++step) {
    const uint32_t mid = lo + ((hi - lo) >> 1) + 1;
    uint32_t cnt = 0;
#pragma unroll
    for (int i = 0; i < NV; ++i) cnt += v[i] >= mid ? 1u : 0u;
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    if (cnt >= static_cast<uint32_t>(K))
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

// Warp-wide exact top-K (K <= 32) of the distinct candidate keys in registers, written
// to top[0..K) sorted descending; returns false (nothing written) when the shortcut
// does not apply and the caller must take the binary search. Every key of the top K
// is at least theta = the K-th largest of the 32 lanes' maxima (the K lanes with the
// largest maxima hold at least K keys >= theta), and on score-like data only a few
// dozen keys reach theta: they are compacted into buf and each one's rank is the
// number of larger candidates. Costs ~4 instructions per candidate instead of the
// search's 32 passes over all of them.
template <int NV>
__device__ __forceinline__ bool topk_by_threshold(const uint32_t (&v)[NV], int K, uint32_t* buf, uint32_t* top,
                                                  int lane) {
  constexpr int kCap = kMaxK;  // buf entries
  if (K > 32) return false;
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < NV; ++i) m = max(m, v[i]);
  int above = 0;  // lanes whose maximum is larger than this lane's
#pragma unroll
  for (int j = 0; j < 32; ++j) above += __shfl_sync(0xffffffffu, m, j) > m ? 1 : 0;
  const uint32_t theta = __reduce_min_sync(0xffffffffu, above < K ? m : 0xFFFFFFFFu);
  int base = 0;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const bool keep = v[i] >= theta && v[i] != 0u;
    const unsigned bal = __ballot_sync(0xffffffffu, keep);
    const int at = base + __popc(bal & ((1u << lane) - 1u));
    if (keep && at < kCap) buf[at] = v[i];
    base += __popc(bal);
  }
  if (base > kCap || base < K) return false;  // warp-uniform
  __syncwarp();
  for (int e = lane; e < base; e += 32) {
    const uint32_t x = buf[e];
    int rank = 0;
    for (int j = 0; j < base; ++j) rank += buf[j] > x ? 1 : 0;
    if (rank < K) top[rank] = x;
  }
  __syncwarp();
  return true;
}

template <int G, bool kF16>
__global__ void __launch_bounds__(kThreads, 1) topk_kernel(const TopkParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  TopkSmem& sm = *reinterpret_cast<TopkSmem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i0 = blockIdx.x * kRows, h = blockIdx.y, b = blockIdx.z;
  // The attention kernel after this one may start its local branch now; it waits
  // (griddepcontrol.wait) for this grid's completion before it reads the indices.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // q_cmp rows of the strided group {h, h+Hk, ...}, stored with the head dimension
  // permuted by perm_d() so that every thread's B-fragment values of a key row are
  // 32 contiguous bytes (the dot products are invariant to a shared permutation).
  for (int e = threadIdx.x; e < G * kRows * 64; e += kThreads) {
    const int g = e / (kRows * 64), r = (e / 64) % kRows, kk = e % 64;
    const int i = i0 + r;
    uint16_t val = 0;  // +0 in both types
    if (i < p.nb) val = p.q_cmp[((static_cast<size_t>(b) * p.nb + i) * p.Hq + g * p.Hk + h) * 64 + perm_d(kk)];
    sm.qs[g][r][kk] = val;
  }
  int count = 0;  // entries of the running top list (same in every warp)
  __syncthreads();

  for (int c0 = 0; c0 < p.nb; c0 += kChunk) {
    const int width = min(kChunk, p.nb - c0);
    // ---- A: scores of this chunk
    {
      AFrags<G> f;
      load_afrags<G>(sm, f, lane);
      for (int grp = warp; grp * 8 < width; grp += kWarps)
        score_group<G, kF16>(p, sm, f, b, h, c0 + grp * 8, grp * 8, lane);
    }
    __syncthreads();

    // ---- B: warp `warp` merges row `warp`
    const int r = warp;
    uint32_t* top = sm.top[r];
    uint32_t* row = sm.keys[r];
    const int K = p.K;
    constexpr int NV = (kChunk + kMaxK) / 32;  // candidates per lane
    uint32_t v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < width ? row[e] : (e - width < count ? top[e - width] : 0u);
    }
    uint32_t* buf = sm.buf[warp];
    if (!topk_by_threshold<NV>(v, K, buf, top, lane)) {
      const uint32_t kth = kth_largest<NV>(v, K);
      // keep the keys >= kth (exactly K of them) in an unsorted buffer ...
      int base = 0;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const bool keep = v[i] >= kth && v[i] != 0u;
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        if (keep) buf[base + __popc(bal & ((1u << lane) - 1u))] = v[i];
        base += __popc(bal);
      }
      __syncwarp();
      // ... and write them to the top list sorted descending (rank = number of larger keys)
      for (int e = lane; e < K; e += 32) {
        const uint32_t x = buf[e];
        int rank = 0;
        for (int j = 0; j < K; ++j) rank += buf[j] > x ? 1 : 0;
        top[rank] = x;
      }
    }
    count = K;
    __syncthreads();
  }

  // ---- write indices
  for (int e = threadIdx.x; e < kRows * p.K; e += kThreads) {
    const int r = e / p.K, s = e % p.K;
    const int i = i0 + r;
    if (i < p.nb)
      p.idx[((static_cast<size_t>(b) * p.nb + i) * p.Hk + h) * p.K + s] =
          static_cast<int64_t>(0xFFFFu - (sm.top[r][s] & 0xFFFFu));
  }
  // Complete only after the coarse attention launched before this kernel, so that
  // a kernel waiting on this grid also sees the coarse-attention output.
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <int G, bool kF16>
int launch_g(const TopkParams& p, cudaStream_t stream, bool overlap) {
  const size_t smem = sizeof(TopkSmem);
  static bool attr_done[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOSAIC_ERR_CUDA;
  if (!attr_done[dev]) {
    if (cudaFuncSetAttribute(topk_kernel<G, kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return MOSAIC_ERR_CUDA;
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.nb + kRows - 1) / kRows, p.Hk, p.B);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, topk_kernel<G, kF16>, p) == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

}  // namespace

int launch_topk(const TopkLaunch& a, cudaStream_t stream) {
  // The score matrix grows as nb^2: from a few thousand blocks on, the tensor-core
  // kernel (topk_tc.cu) wins; below, this one's 16-row CTAs fill the GPU better.
  if (a.B > 0 && a.nb >= kTcMinBlocks && topk_tc_supported(a)) return launch_topk_tc(a, stream);
  TopkParams p;
  p.q_cmp = static_cast<const uint16_t*>(a.q_cmp);
  p.k_cmp = static_cast<const uint16_t*>(a.k_cmp);
  p.idx = a.idx;
  p.B = a.B;
  p.nb = a.nb;
  p.Hq = a.Hq;
  p.Hk = a.Hk;
  p.K = a.K;
  p.G = a.Hq / a.Hk;
  if (p.K > kMaxK || p.K > p.nb || p.nb > 65535) return MOSAIC_ERR_UNSUPPORTED;
  switch (p.G * 2 + (a.f16 ? 1 : 0)) {
    case 2: return launch_g<1, false>(p, stream, a.overlap_previous);
    case 3: return launch_g<1, true>(p, stream, a.overlap_previous);
    case 4: return launch_g<2, false>(p, stream, a.overlap_previous);
    case 5: return launch_g<2, true>(p, stream, a.overlap_previous);
    case 8: return launch_g<4, false>(p, stream, a.overlap_previous);
    case 9: return launch_g<4, true>(p, stream, a.overlap_previous);
    case 6: return launch_g<3, false>(p, stream, a.overlap_previous);
    case 7: return launch_g<3, true>(p, stream, a.overlap_previous);
    case 10: return launch_g<5, false>(p, stream, a.overlap_previous);
    case 11: return launch_g<5, true>(p, stream, a.overlap_previous);
    case 12: return launch_g<6, false>(p, stream, a.overlap_previous);
    case 13: return launch_g<6, true>(p, stream, a.overlap_previous);
    case 14: return launch_g<7, false>(p, stream, a.overlap_previous);
    case 15: return launch_g<7, true>(p, stream, a.overlap_previous);
    case 16: return launch_g<8, false>(p, stream, a.overlap_previous);
    case 17: return launch_g<8, true>(p, stream, a.overlap_previous);
    default: return MOSAIC_ERR_UNSUPPORTED;
  }
}

}  // namespace mosaic
