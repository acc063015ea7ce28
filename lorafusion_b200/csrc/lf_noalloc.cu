// Forward entry point that needs no caller-provided scratch and allocates nothing.
//
// Some hosts hand an operator only its input and output device buffers: plugin interfaces of
// inference engines that plan all device memory up front and give plugins no allocator, or
// processes that run under a fixed device-memory budget where a per-call workspace allocation
// would fail or fragment the pool.  Those callers cannot provide the forward's workspace.  This
// entry point keeps that scratch in a fixed-size array that the library itself declares in
// device memory, so the caller passes inputs and outputs only.
//
// Cost of the convenience: every GPU that loads this library reserves LF_NOALLOC_SCRATCH_BYTES
// for the array until the process exits, whether or not this entry point is used.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/lorafusion_b200.h"
#include "lf_internal.cuh"

namespace {

constexpr size_t kScratchBytes = LF_NOALLOC_SCRATCH_BYTES;

// Shared by every call on a device; it keeps whatever the last call wrote.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[64];  // device address of g_noalloc_scratch, per device ordinal
bool g_scratch_known[64];

}  // namespace

extern "C" int lf_forward_noalloc(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                                  void* y_dev, lf_stream_t stream) {
  if (!prob || !info) return LF_ERR_INVALID_ARG;
  // the fixed sections must fit; the K-split tail of the GEMM uses as much of the rest as it can
  if (lf::forward_min_workspace_bytes(info) > kScratchBytes) return LF_ERR_CAPACITY;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LF_ERR_CUDA;
  void* scratch = nullptr;
  {
    // First call on a device: look up the array's device address with that device current.
    // Host code must not use the symbol itself as a pointer: on the host it only names a
    // host-side stand-in for the device array.
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_known[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return LF_ERR_CUDA;
      g_scratch_addr[dev] = p;
      g_scratch_known[dev] = true;
    }
    scratch = g_scratch_addr[dev];
  }
  // The forward writes every scratch element it later reads (masked zeros included), so the
  // previous call's contents need no clearing.
  return lf_forward(prob, info, table_dev, y_dev, scratch, kScratchBytes, stream);
}
