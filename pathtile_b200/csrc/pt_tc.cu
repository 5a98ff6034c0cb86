// pt_tc.cu -- instantiations of the tensor-core FWD / DX kernels.
#include "pathtile_b200.h"
#include "pt_tc.h"
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

}  // namespace tc
}  // namespace pt
