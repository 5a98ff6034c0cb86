// pt_tc_bwd_k2.cu -- instantiations of the fused backward kernel for K = 25..48
// (split over two translation units so that they compile in parallel).
#include "pt_tc.h"
#include "pt_tc_bwd.cuh"

namespace pt {
namespace tc {

const void* bwd_kernel_k25_48(int K) {
  switch (K) {
    case 25: return reinterpret_cast<const void*>(&tc_bwd_kernel<25>);
    case 26: return reinterpret_cast<const void*>(&tc_bwd_kernel<26>);
    case 27: return reinterpret_cast<const void*>(&tc_bwd_kernel<27>);
    case 28: return reinterpret_cast<const void*>(&tc_bwd_kernel<28>);
    case 29: return reinterpret_cast<const void*>(&tc_bwd_kernel<29>);
    case 30: return reinterpret_cast<const void*>(&tc_bwd_kernel<30>);
    case 31: return reinterpret_cast<const void*>(&tc_bwd_kernel<31>);
    case 32: return reinterpret_cast<const void*>(&tc_bwd_kernel<32>);
    case 33: return reinterpret_cast<const void*>(&tc_bwd_kernel<33>);
    case 34: return reinterpret_cast<const void*>(&tc_bwd_kernel<34>);
    case 35: return reinterpret_cast<const void*>(&tc_bwd_kernel<35>);
    case 36: return reinterpret_cast<const void*>(&tc_bwd_kernel<36>);
    case 37: return reinterpret_cast<const void*>(&tc_bwd_kernel<37>);
    case 38: return reinterpret_cast<const void*>(&tc_bwd_kernel<38>);
    case 39: return reinterpret_cast<const void*>(&tc_bwd_kernel<39>);
    case 40: return reinterpret_cast<const void*>(&tc_bwd_kernel<40>);
    case 41: return reinterpret_cast<const void*>(&tc_bwd_kernel<41>);
    case 42: return reinterpret_cast<const void*>(&tc_bwd_kernel<42>);
    case 43: return reinterpret_cast<const void*>(&tc_bwd_kernel<43>);
    case 44: return reinterpret_cast<const void*>(&tc_bwd_kernel<44>);
    case 45: return reinterpret_cast<const void*>(&tc_bwd_kernel<45>);
    case 46: return reinterpret_cast<const void*>(&tc_bwd_kernel<46>);
    case 47: return reinterpret_cast<const void*>(&tc_bwd_kernel<47>);
    case 48: return reinterpret_cast<const void*>(&tc_bwd_kernel<48>);
    default: return nullptr;
  }
}

}  // namespace tc
}  // namespace pt
