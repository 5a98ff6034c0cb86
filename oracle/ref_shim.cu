// ref_shim.cu -- TEST INFRASTRUCTURE ONLY.  Host launchers for the reference's
// own warp-tiled CUDA kernels, so the unmodified reference kernels can run on a
// B200 as a comparison point (parity cross-check and timing), never as part of
// the product.  The kernel source is not in this repository: build_oracle.py
// extracts CUDA_TEMPLATE from the reference's kernels/warp_tiled_ampere.py,
// substitutes the reference's default launch constants (WARPS_PER_BLOCK=16,
// BWDK_BTILE=64, BWDK_BLOCK=128; kernels/warp_tiled_ampere.py:71-74, 668-672)
// and writes it to _ref/ref_warptile_kernels.cu, which this file includes.
// Launch geometry follows AmpereWarpRuntime (kernels/warp_tiled_ampere.py:
// 742-743 and 807-808).
#include <cuda_runtime.h>

#include REF_KERNELS_FILE

namespace {
constexpr int kRefWarps = 16;
constexpr int kRefBtile = 64;
constexpr int kRefBlock = 128;
}  // namespace

extern "C" {

int ref_fwd(const float* x, const float* k, float* y, int B, int H, int L, int K, void* stream) {
  dim3 grid((B + kRefWarps - 1) / kRefWarps, H, 1);
  dwconv1d_warptile_fwd<<<grid, kRefWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(x, k, y, B, H, L, K);
  return static_cast<int>(cudaGetLastError());
}

int ref_dx(const float* gy, const float* k, float* gx, int B, int H, int L, int K, void* stream) {
  dim3 grid((B + kRefWarps - 1) / kRefWarps, H, 1);
  dwconv1d_warptile_bwd_input<<<grid, kRefWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(gy, k, gx, B, H,
                                                                                                L, K);
  return static_cast<int>(cudaGetLastError());
}

// gk must be zero-filled by the caller (atomic accumulation, as in the reference).
int ref_dk(const float* gy, const float* x, float* gk, int B, int H, int L, int K, void* stream) {
  const int num_btiles = (B + kRefBtile - 1) / kRefBtile;
  dim3 grid(H, num_btiles, 1);
  dwconv1d_warptile_bwd_weight<<<grid, kRefBlock, 0, static_cast<cudaStream_t>(stream)>>>(gy, x, gk, B, H, L,
                                                                                           K, num_btiles);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
