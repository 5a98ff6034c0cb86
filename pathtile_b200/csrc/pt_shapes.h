// pt_shapes.h -- (L, K) pairs that get fully unrolled, in-range-only kernels.
//
// The list is the union of every (L, K) the path is specified and tuned on:
//   * the primary workload (48,48) and the edge shapes (37,13), (16,4), (48,3), (33,33);
//   * the held-out sweep L in {24,32,48} x K in {8,16,32,48}, K <= L;
//   * the 20 PathTile tuning shapes and 10 held-out shapes of the reference
//     (benchmark/benchmark_shape_sweep_ampere.py:79-178);
//   * the reference's correctness cases (kernels/warp_tiled_ampere.py:919-926).
// Any other (L <= 48, K <= 48) runs the generic kernels with runtime bounds.
// X(index, L, K); indices are dense and fix the shard a pair compiles in.
#pragma once

#define PT_EXACT_SHAPES(X) \
  X(0, 48, 48)             \
  X(1, 37, 13)             \
  X(2, 16, 4)              \
  X(3, 48, 3)              \
  X(4, 33, 33)             \
  X(5, 24, 8)              \
  X(6, 24, 16)             \
  X(7, 32, 8)              \
  X(8, 32, 16)             \
  X(9, 32, 32)             \
  X(10, 48, 8)             \
  X(11, 48, 16)            \
  X(12, 48, 32)            \
  X(13, 16, 16)            \
  X(14, 24, 24)            \
  X(15, 48, 24)            \
  X(16, 32, 24)            \
  X(17, 40, 20)            \
  X(18, 40, 32)            \
  X(19, 20, 12)            \
  X(20, 28, 24)            \
  X(21, 40, 40)            \
  X(22, 20, 16)            \
  X(23, 28, 20)            \
  X(24, 40, 12)            \
  X(25, 16, 8)             \
  X(26, 31, 16)

#define PT_NUM_SHARDS 8
