// pt_tc.cu -- instantiations of the tensor-core FWD / DX kernels.
#include "pathtile_b200.h"
#include "pt_tc.h"
#include "pt_tc_dk.cuh"
#include "pt_tc_kernels.cuh"

namespace pt {
namespace tc {

static_assert(kRowsPerTile == M && kThreads == THREADS, "pt_tc.h and pt_tc_kernels.cuh disagree");

template <int OP>
static const void* func_for(const Layout& lay) {
  if (lay.packed) return lay.lb == 3 ? reinterpret_cast<const void*>(&tc_conv_kernel<OP, 3, true>) : nullptr;
  if (lay.lb == 1) return reinterpret_cast<const void*>(&tc_conv_kernel<OP, 1, false>);
  if (lay.lb == 2) return reinterpret_cast<const void*>(&tc_conv_kernel<OP, 2, false>);
  if (lay.lb == 3) return reinterpret_cast<const void*>(&tc_conv_kernel<OP, 3, false>);
  return nullptr;
}

const void* conv_func(int path, const Layout& lay) {
  if (path == PT_PATH_FWD) return func_for<OP_FWD>(lay);
  if (path == PT_PATH_DX) return func_for<OP_DX>(lay);
  return nullptr;
}

size_t conv_smem(const Layout& lay) {
  if (lay.lb == 1) return Geo<1>::SMEM;
  if (lay.lb == 2) return Geo<2>::SMEM;
  return Geo<3>::SMEM;
}

static_assert(kDkRowsPerTile == DK_ROWS && kDkThreads == DK_THREADS && kDkMaxGroups == DK_MAX_GROUPS,
              "pt_tc.h and pt_tc_dk.cuh disagree");

const void* dk_func(const Layout& lay) {
  if (lay.packed) return lay.lb == 3 ? reinterpret_cast<const void*>(&tc_dk_kernel<3, true>) : nullptr;
  if (lay.lb == 1) return reinterpret_cast<const void*>(&tc_dk_kernel<1, false>);
  if (lay.lb == 2) return reinterpret_cast<const void*>(&tc_dk_kernel<2, false>);
  if (lay.lb == 3) return reinterpret_cast<const void*>(&tc_dk_kernel<3, false>);
  return nullptr;
}

size_t dk_smem(const Layout& lay) {
  if (lay.lb == 1) return DkGeo<1>::SMEM;
  if (lay.lb == 2) return DkGeo<2>::SMEM;
  return DkGeo<3>::SMEM;
}

__global__ void __launch_bounds__(256) tc_dk_reduce_kernel(const float* __restrict__ partial,
                                                           const int* __restrict__ group_of, int n_slots,
                                                           int H, int K, int hc, float* __restrict__ dk,
                                                           int accumulate) {
  const int idx = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (idx >= H * K) return;
  const int h = idx / K;
  const int j = idx - h * K;
  const int grp = h / hc;
  const int c = h - grp * hc;
  float acc = 0.f;
  for (int e = 0; e < n_slots; ++e)
    if (group_of[e] == grp) acc += partial[static_cast<size_t>(e) * hc * K + c * K + j];
  dk[idx] = accumulate ? dk[idx] + acc : acc;
}

const void* bwd_func(int L, int K) {
  // One 48-column tile layout (a 128-B and a 64-B box per row): rows shorter
  // than 48 columns (32 < L < 48, L % 4 == 0) are zero-filled by the loads and
  // clipped by the stores, which leaves dX and dK exact.
  if (L % 4 != 0 || L <= 32 || L > 48 || K < 1 || K > 48) return nullptr;
  return K <= 24 ? bwd_kernel_k1_24(K) : bwd_kernel_k25_48(K);
}

size_t bwd_smem() { return bwd_smem_bytes(); }

void dk_reduce(const float* partial, const int* group_of, int n_slots, int H, int K, int hc, float* dk,
               int accumulate, void* stream) {
  const int n = H * K;
  tc_dk_reduce_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      partial, group_of, n_slots, H, K, hc, dk, accumulate);
}

}  // namespace tc
}  // namespace pt
