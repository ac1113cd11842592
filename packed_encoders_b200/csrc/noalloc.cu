// pe_b200_attn_fwd_noalloc: packed attention for callers that cannot hand this library any
// device memory of their own.
//
// The regular entry point (pe_b200_attn_fwd) needs a caller-provided workspace for the tile
// schedule and the device error word. Some callers cannot provide one: a plugin whose host
// framework gives it only a stream and the tensors (no allocator, no workspace slot), a binding
// from a language runtime that has no CUDA allocation API of its own, or a server that reserves
// all device memory at start-up and forbids allocation on the request path. For them, this
// entry point keeps that scratch in a fixed array in the library's own device memory.
//
// Limits and rules:
//   * the array holds kNoAllocScratchBytes (1 MiB): the 256-byte schedule header plus 65,520
//     work-item slots, i.e. calls need n_seq + total_q / 128 + 2 <= 65,520; larger calls are
//     rejected with PE_B200_ERR_SCRATCH_LIMIT before anything is enqueued;
//   * every GPU that loads the library holds the 1 MiB until the process exits;
//   * the first call on a device looks up the array's device address on that device (with the
//     device current) and caches it; make that first call before any stream capture;
//   * all calls share the one array: calls whose kernels overlap on the GPU (different streams
//     without ordering, or several host threads) race on it and must be serialised by the
//     caller. The schedule header is cleared by every call, so nothing stale carries over.
//   * no cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/pe_b200_attn.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;

// The scratch itself. In host code `g_noalloc_scratch` is only a host-side stand-in for the
// symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of the scratch on the current device, looked up once per device.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return PE_B200_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    cudaError_t st = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (st != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();  // do not leave the lookup failure as the thread's last error
      return PE_B200_ERR_CUDA;
    }
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return PE_B200_OK;
}

}  // namespace

extern "C" int pe_b200_attn_fwd_noalloc(const PeB200AttnParams* p, void* stream) {
  if (!p) return PE_B200_ERR_NULL;
  size_t need = 0;
  int st = pe_b200_attn_workspace_size(p, &need);
  if (st != PE_B200_OK) return st;
  if (need > kNoAllocScratchBytes) return PE_B200_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  st = scratch_for_current_device(&scratch);
  if (st != PE_B200_OK) return st;
  PeB200AttnParams q = *p;
  q.workspace = scratch;
  q.workspace_bytes = kNoAllocScratchBytes;
  return pe_b200_attn_fwd(&q, stream);
}
