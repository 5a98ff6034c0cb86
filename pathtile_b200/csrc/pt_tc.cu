// pt_tc.cu -- instantiations of the tensor-core FWD / DX kernels.
#include "pathtile_b200.h"
#include "pt_tc.h"
#include "pt_tc_kernels.cuh"

namespace pt {
namespace tc {

static_assert(kRowsPerTile == M && kThreads == THREADS, "pt_tc.h and pt_tc_kernels.cuh disagree");

const void* conv_func(int path, int lb) {
  if (path == PT_PATH_FWD) {
    if (lb == 1) return reinterpret_cast<const void*>(&tc_conv_kernel<OP_FWD, 1>);
    if (lb == 2) return reinterpret_cast<const void*>(&tc_conv_kernel<OP_FWD, 2>);
    if (lb == 3) return reinterpret_cast<const void*>(&tc_conv_kernel<OP_FWD, 3>);
  } else if (path == PT_PATH_DX) {
    if (lb == 1) return reinterpret_cast<const void*>(&tc_conv_kernel<OP_DX, 1>);
    if (lb == 2) return reinterpret_cast<const void*>(&tc_conv_kernel<OP_DX, 2>);
    if (lb == 3) return reinterpret_cast<const void*>(&tc_conv_kernel<OP_DX, 3>);
  }
  return nullptr;
}

size_t conv_smem(int lb) {
  if (lb == 1) return Geo<1>::SMEM;
  if (lb == 2) return Geo<2>::SMEM;
  return Geo<3>::SMEM;
}

}  // namespace tc
}  // namespace pt
