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
//   * the array holds kNoAllocScratchBytes (1 MiB); a call fits when pe_b200_attn_workspace_size
//     reports at most that. Without rotary tables that is n_seq + total_q / 128 + 2 <= 65,520
//     (a 256-byte header plus 16-byte work items); a call with rotary tables also keeps its
//     rotated q and k there, so only small rotary calls fit. Larger calls are rejected with
//     PE_B200_ERR_SCRATCH_LIMIT before anything is enqueued;
//   * every GPU that loads the library holds the 1 MiB until the process exits;
//   * the first call on a device (and the first after that device's context was destroyed and
//     re-created, e.g. by cudaDeviceReset) looks up the array's device address with the device
//     current and caches it per context; make that first call before any stream capture;
//   * all calls share the one array: calls whose kernels overlap on the GPU (different streams
//     without ordering, or several host threads) race on it and must be serialised by the
//     caller. The schedule header and error word are cleared by every call, so nothing stale
//     carries over;
//   * pe_b200_noalloc_error_word reads the device error word of the last call on the current
//     device (bounded-wait timeout, schedule overflow, malformed cu_seqlens);
//   * no cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda.h>
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
struct ScratchSlot {
  unsigned long long ctx_id = 0;  // the context the address belongs to (0: none yet)
  void* ptr = nullptr;
};
ScratchSlot g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the current context (cuCtxGetId, through the runtime's driver entry points); 0 if
// it cannot be read, in which case the cached address is trusted for the device.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(fn);
    cudaGetLastError();
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx && get_id(ctx, &id) == CUDA_SUCCESS) return id;
  return 0;
}

// Device address of the scratch on the current device, looked up once per device and context.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return PE_B200_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& slot = g_scratch[dev];
  if (slot.ptr == nullptr || slot.ctx_id != current_context_id()) {
    void* ptr = nullptr;
    cudaError_t st = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);  // creates the context if needed
    if (st != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();  // do not leave the lookup failure as the thread's last error
      return PE_B200_ERR_CUDA;
    }
    slot.ptr = ptr;
    slot.ctx_id = current_context_id();
  }
  *out = slot.ptr;
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

extern "C" int pe_b200_noalloc_error_word(int* out, void* stream) {
  if (!out) return PE_B200_ERR_NULL;
  void* scratch = nullptr;
  int st = scratch_for_current_device(&scratch);
  if (st != PE_B200_OK) return st;
  // The error word is the second int of the schedule header at the start of the scratch. One
  // copy on the caller's stream (ordered after the calls enqueued there), then wait for it.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(out, static_cast<const char*>(scratch) + sizeof(int), sizeof(int), cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    cudaGetLastError();
    return PE_B200_ERR_CUDA;
  }
  return PE_B200_OK;
}
