// pt_tc.h -- table of the tensor-core FWD / DX kernels (instantiated in pt_tc.cu).
#pragma once

#include <cstddef>

namespace pt {
namespace tc {

constexpr int kRowsPerTile = 128;
constexpr int kThreads = 448;

// Tile layout of a row length L (L % 4 == 0): Hc adjacent channels per
// super-row (48 / L when that divides and L <= 24, else 1), the super-row's
// box class lb (1: 16 columns, 2: 32, 3: 48) and whether the tensor maps are
// 2-D over [B, H*L] (packed) or 3-D over (L, H, B).
struct Layout {
  int hc;
  int lb;
  bool packed;
};

inline Layout layout_for(int L) {
  if (L <= 24 && 48 % L == 0) return Layout{48 / L, 3, true};
  return Layout{1, L <= 16 ? 1 : (L <= 32 ? 2 : 3), false};
}

// Kernel for path PT_PATH_FWD / PT_PATH_DX and a layout, or nullptr.
const void* conv_func(int path, const Layout& lay);

// Dynamic shared memory (bytes) of that kernel.
size_t conv_smem(const Layout& lay);

}  // namespace tc
}  // namespace pt

namespace pt {
namespace tc {

constexpr int kDkRowsPerTile = 64;
constexpr int kDkThreads = 320;
constexpr int kDkMaxGroups = 2;

// tcgen05 dK kernel for a layout, or nullptr.
const void* dk_func(const Layout& lay);
size_t dk_smem(const Layout& lay);

// dk[h][j] (= or +=) the sum, in CTA order, of the partials of every CTA
// accumulator that held h's channel group.
void dk_reduce(const float* partial, const int* group_of, int n_slots, int H, int K, int hc, float* dk,
               int accumulate, void* stream);

}  // namespace tc
}  // namespace pt

namespace pt {
namespace tc {

// Fused backward (dX on the tensor cores + dK on the CUDA cores) for any K <= 48
// and rows of 32 < L <= 48 columns with L % 4 == 0; nullptr otherwise.  The
// host launches it only where the compiled function starts with
// kBwdLaunchRegs registers per thread.
constexpr int kBwdLaunchRegs = 128;
int bwd_threads();

// Work schedule of the fused backward: nblk = ceil(B / 128) batch blocks per
// channel; CTAs g < kp*H are primaries (channel g % H, blocks g / H + i*kp
// below P); the E CTAs after them are helpers (helper e: channels e, e + E, ...,
// each over the tail blocks [P, nblk)); m = ceil(H / E), the most channels a
// helper owns; direct = 1 when each channel has exactly one CTA and no helper
// (the kernel then writes dK itself).  The workspace holds [slots][4][K] floats,
// slots = kp*H + E*m.
struct BwdSched {
  int H, nblk, kp, P, E, m;
  int direct;
};

// dk (=, or += when accumulate) the sum of each channel's partials in a fixed order.
void bwd_dk_reduce(const float* part, float* dk, const BwdSched& sc, int K, int accumulate, void* stream);
const void* bwd_func(int L, int K);
// The fused kernel's instantiations, one per K (pt_tc_bwd_k1.cu, pt_tc_bwd_k2.cu).
const void* bwd_kernel_k1_24(int K);
const void* bwd_kernel_k25_48(int K);
size_t bwd_smem_bytes();
size_t bwd_smem();

}  // namespace tc
}  // namespace pt
