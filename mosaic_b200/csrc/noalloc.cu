// mosaic_bsa_fwd_noalloc: the full forward without a caller-supplied workspace.
//
// Who needs it: callers that cannot hand the library device scratch memory. A
// foreign-language host (Go, Java, C) that binds the C ABI directly usually has
// no device allocator of its own, and an inference service that reserves its
// memory budget once at start-up must not call cudaMalloc / cudaFree per request
// (those calls can synchronise the whole device and fragment the reserved pool).
// For them this entry point keeps its scratch in a fixed device array that is
// part of the library image itself.
//
// The scratch: `g_bsa_scratch`, kNoAllocScratchBytes (8 MiB) per device. Every
// GPU that loads this library holds that array until the process exits. It holds
// the pooled q/k/v, the coarse-attention rows and the block indices of one call,
// so it covers B * (N / bs) * (2*Hq + 2*Hk) * 128 + B * (N / bs) * Hk * K * 8
// bytes (3.4 MB at Nside 64 with B = 1; B = 2 still fits). Larger calls are
// rejected with MOSAIC_ERR_WORKSPACE before anything runs. RoPE-on-the-fly is not
// offered here (its rotated copies of q and k would not fit a modest array).
//
// Sharing: all calls on a device use the same array and it keeps whatever the
// last call wrote. Every region is fully overwritten before it is read within a
// call, so nothing has to start at zero and nothing is cleared. Two calls whose
// kernels overlap on the GPU (different streams, or different host threads on one
// device) race on the array and corrupt each other's results: serialise them.
//
// Set-up: the first call on each device looks up the array's device address with
// cudaGetSymbolAddress (with that device current) and caches it; later calls
// reuse the cached address. Make that first call before any stream capture. The
// cache lives as long as the process: cudaDeviceReset destroys the context the
// address belongs to, so a process that resets a device must not call this entry
// point on that device afterwards.
// Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <mutex>

#include "kernels.h"
#include "ptx.cuh"

namespace mosaic {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_bsa_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_bsa_scratch on the current device (looked up once per device).
// In host code the name g_bsa_scratch is only a stand-in for the symbol; it must
// never be passed to a kernel.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MOSAIC_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_bsa_scratch) != cudaSuccess || p == nullptr) return MOSAIC_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return MOSAIC_OK;
}

}  // namespace
}  // namespace mosaic

extern "C" {

int mosaic_bsa_fwd_noalloc(const MosaicBsaArgs* args, void* stream) {
  if (args == nullptr) return MOSAIC_ERR_INVALID_ARGUMENT;
  if (args->rope_cos != nullptr || args->rope_sin != nullptr) return MOSAIC_ERR_UNSUPPORTED;
  const int K = args->block_attn_only ? 0 : args->sparse_block_count;
  const int bs = args->sparse_block_size > 0 ? args->sparse_block_size : 64;
  const size_t need = mosaic_bsa_workspace_bytes(args->batch, args->seq_len, args->num_q_heads,
                                                 args->num_kv_heads, args->head_dim, bs, K, 0);
  if (need > mosaic::kNoAllocScratchBytes) return MOSAIC_ERR_WORKSPACE;
  if (args->batch == 0 || args->seq_len == 0) return MOSAIC_OK;
  MosaicBsaArgs a = *args;
  void* scratch = nullptr;
  const bool needs_scratch = !a.block_attn_only;
  if (needs_scratch) {
    const int rc = mosaic::scratch_address(&scratch);
    if (rc != MOSAIC_OK) return rc;
  }
  a.workspace = scratch;
  a.workspace_bytes = needs_scratch ? mosaic::kNoAllocScratchBytes : 0;
  return mosaic_bsa_fwd(&a, stream);
}

}  // extern "C"
