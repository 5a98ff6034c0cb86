// pt_tc_bwd_k1.cu -- instantiations of the fused backward kernel for K = 1..24
// (split over two translation units so that they compile in parallel).
#include "pt_tc.h"
#include "pt_tc_bwd.cuh"

namespace pt {
namespace tc {

const void* bwd_kernel_k1_24(int K) {
  switch (K) {
    case 1: return reinterpret_cast<const void*>(&tc_bwd_kernel<1>);
    case 2: return reinterpret_cast<const void*>(&tc_bwd_kernel<2>);
    case 3: return reinterpret_cast<const void*>(&tc_bwd_kernel<3>);
    case 4: return reinterpret_cast<const void*>(&tc_bwd_kernel<4>);
    case 5: return reinterpret_cast<const void*>(&tc_bwd_kernel<5>);
    case 6: return reinterpret_cast<const void*>(&tc_bwd_kernel<6>);
    case 7: return reinterpret_cast<const void*>(&tc_bwd_kernel<7>);
    case 8: return reinterpret_cast<const void*>(&tc_bwd_kernel<8>);
    case 9: return reinterpret_cast<const void*>(&tc_bwd_kernel<9>);
    case 10: return reinterpret_cast<const void*>(&tc_bwd_kernel<10>);
    case 11: return reinterpret_cast<const void*>(&tc_bwd_kernel<11>);
    case 12: return reinterpret_cast<const void*>(&tc_bwd_kernel<12>);
    case 13: return reinterpret_cast<const void*>(&tc_bwd_kernel<13>);
    case 14: return reinterpret_cast<const void*>(&tc_bwd_kernel<14>);
    case 15: return reinterpret_cast<const void*>(&tc_bwd_kernel<15>);
    case 16: return reinterpret_cast<const void*>(&tc_bwd_kernel<16>);
    case 17: return reinterpret_cast<const void*>(&tc_bwd_kernel<17>);
    case 18: return reinterpret_cast<const void*>(&tc_bwd_kernel<18>);
    case 19: return reinterpret_cast<const void*>(&tc_bwd_kernel<19>);
    case 20: return reinterpret_cast<const void*>(&tc_bwd_kernel<20>);
    case 21: return reinterpret_cast<const void*>(&tc_bwd_kernel<21>);
    case 22: return reinterpret_cast<const void*>(&tc_bwd_kernel<22>);
    case 23: return reinterpret_cast<const void*>(&tc_bwd_kernel<23>);
    case 24: return reinterpret_cast<const void*>(&tc_bwd_kernel<24>);
    default: return nullptr;
  }
}

size_t bwd_smem_bytes() { return BwdGeo::SMEM; }

int bwd_threads() { return BWD_LAUNCH_THREADS; }

void bwd_dk_reduce(const float* part, float* dk, const BwdSched& sc, int K, int accumulate, void* stream) {
  const int n = sc.H * K;
  bwd_dk_reduce_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(part, dk, sc, K,
                                                                                         accumulate);
}

}  // namespace tc
}  // namespace pt
