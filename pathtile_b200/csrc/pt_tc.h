// pt_tc.h -- table of the tensor-core FWD / DX kernels (instantiated in pt_tc.cu).
#pragma once

#include <cstddef>

namespace pt {
namespace tc {

// Box layout class of a row length: 1 (L <= 16), 2 (L <= 32), 3 (L <= 48).
inline int layout_class(int L) { return L <= 16 ? 1 : (L <= 32 ? 2 : 3); }

// Kernel for path PT_PATH_FWD / PT_PATH_DX and layout class lb, or nullptr.
const void* conv_func(int path, int lb);

// Dynamic shared memory (bytes) of that kernel.
size_t conv_smem(int lb);

constexpr int kRowsPerTile = 128;
constexpr int kThreads = 448;

}  // namespace tc
}  // namespace pt
