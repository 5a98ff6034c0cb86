// pt_cl.h -- channels-last ([B, L, H]) depthwise Conv1D kernels (host launchers).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

namespace pt {
namespace cl {

// y[b, t, h] = sum_j k[h, j] x[b, t + j - K/2, h] (FWD), or the input gradient
// dx[b, t, h] = sum_j k[h, K-1-j] dy[b, t + j - (K-1-K/2), h] (rev != 0).
cudaError_t launch_conv(const float* in, const float* k, float* out, int B, int L, int H, int K, bool rev,
                        cudaStream_t stream);

// Deterministic filter gradient: per-CTA partials [slices][H][K] in ws, then a
// fixed-order sum over slices into dk (= or += when accumulate != 0).
size_t dk_workspace_bytes(int B, int L, int H, int K, int sm_count);
cudaError_t launch_dk(const float* dy, const float* x, float* dk, int B, int L, int H, int K, int accumulate,
                      void* ws, int sm_count, cudaStream_t stream);

}  // namespace cl
}  // namespace pt
