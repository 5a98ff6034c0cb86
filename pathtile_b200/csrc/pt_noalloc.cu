// pt_noalloc.cu -- deterministic filter gradient that allocates nothing.
//
// Who needs it: callers that hand this library device pointers but are not
// allowed to allocate device memory themselves, for example a serving or
// training runtime that reserves its whole memory budget up front and owns
// every allocation through its own pool, or a real-time loop that must not call
// cudaMalloc/cudaFree in steady state because those calls can block on, or
// synchronise, the device.  The regular deterministic path (pt_dk) needs a
// caller-provided workspace for its per-CTA partial sums; this entry point uses
// a fixed scratch array that lives in the library's own device image instead.
//
// The scratch array is a file-scope __device__ array of PT_DK_NOALLOC_SCRATCH_BYTES
// (8 MiB).  Every GPU that loads the library holds it until the process exits.
// Host code cannot use the array's name as a device address, so the first call
// on each device (with that device current) resolves the address with
// cudaGetSymbolAddress and caches it; make that first call before any stream
// capture.  All calls share the one array: calls whose executions overlap on
// the GPU (different streams, or different host threads on one device) race on
// it and must be serialised by the caller.  Nothing in the array needs to start
// at zero: pass 1 writes every partial that pass 2 reads, and the tensor-core
// dK marks each CTA's partial slots unused before it waits on anything, so a
// CTA that gives up after a timed-out wait never lets pass 2 read what an
// earlier call left.  Whenever pt_device_error reports a non-zero word, the
// dK of the calls since it was last cleared is undefined.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "pathtile_b200.h"

namespace {

static __device__ __align__(256) unsigned char g_pt_dk_noalloc_scratch[PT_DK_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxNoallocDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxNoallocDevices] = {};

// Device address of the scratch array on the current device (set-up on first use).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return PT_ERR_CUDA;
  if (dev < 0 || dev >= kMaxNoallocDevices) return PT_ERR_DEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_pt_dk_noalloc_scratch);
    if (e != cudaSuccess || !p) return PT_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return PT_OK;
}

}  // namespace

extern "C" int pt_dk_noalloc(const float* dy, const float* x, float* dk, int B, int H, int L, int K,
                             int accumulate, void* stream) {
  if (B > 0) {
    const size_t need = pt_dk_workspace_bytes(B, H, L, K);
    if (need == 0) {
      // Same argument checks as pt_dk report the precise reason.
      return pt_dk(dy, x, dk, B, H, L, K, PT_DK_DETERMINISTIC, nullptr, 0, stream);
    }
    if (need > PT_DK_NOALLOC_SCRATCH_BYTES) return PT_ERR_SCRATCH_LIMIT;
  }
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != PT_OK) return rc;
  return pt_dk(dy, x, dk, B, H, L, K, accumulate ? PT_DK_DETERMINISTIC_ACCUMULATE : PT_DK_DETERMINISTIC,
               scratch, PT_DK_NOALLOC_SCRATCH_BYTES, stream);
}
