// pt_registry.h -- table of specialised kernels, filled by the shard units.
#pragma once

#include <vector>

#include "pt_kernels.cuh"
#include "pt_shapes.h"

namespace pt {

struct Entry {
  int L, K;
  int loader;          // LOAD_TMA3D or LOAD_BULK1D
  const void* fwd[2];  // conv_rows_kernel<L,K,OP_FWD,loader,TPR>, TPR = 1, 2
  const void* dx[2];   // conv_rows_kernel<L,K,OP_DX,loader,TPR>
  const void* dk[2];   // dk_rows_kernel<L,K,loader,TPR>
  const void* bwd;     // bwd_rows_kernel<L,K,loader>: fused dX + dK on the CUDA cores
};

template <int L, int K>
Entry make_entry() {
  constexpr int LD = (L % 4 == 0) ? LOAD_TMA3D : LOAD_BULK1D;
  return Entry{L,
               K,
               LD,
               {reinterpret_cast<const void*>(&conv_rows_kernel<L, K, OP_FWD, LD, 1>),
                reinterpret_cast<const void*>(&conv_rows_kernel<L, K, OP_FWD, LD, 2>)},
               {reinterpret_cast<const void*>(&conv_rows_kernel<L, K, OP_DX, LD, 1>),
                reinterpret_cast<const void*>(&conv_rows_kernel<L, K, OP_DX, LD, 2>)},
               {reinterpret_cast<const void*>(&dk_rows_kernel<L, K, LD, 1>),
                reinterpret_cast<const void*>(&dk_rows_kernel<L, K, LD, 2>)},
               reinterpret_cast<const void*>(&bwd_rows_kernel<L, K, LD>)};
}

void register_shard_0(std::vector<Entry>& v);
void register_shard_1(std::vector<Entry>& v);
void register_shard_2(std::vector<Entry>& v);
void register_shard_3(std::vector<Entry>& v);
void register_shard_4(std::vector<Entry>& v);
void register_shard_5(std::vector<Entry>& v);
void register_shard_6(std::vector<Entry>& v);
void register_shard_7(std::vector<Entry>& v);

}  // namespace pt

// Body of a shard unit: instantiate the pairs whose index % PT_NUM_SHARDS == SHARD.
#define PT_DEFINE_SHARD(SHARD)                                            \
  namespace pt {                                                          \
  template <int IDX, int L, int K>                                        \
  static void shard_maybe_add(std::vector<Entry>& v) {                    \
    if constexpr (IDX % PT_NUM_SHARDS == (SHARD)) v.push_back(make_entry<L, K>()); \
  }                                                                       \
  void register_shard_##SHARD(std::vector<Entry>& v) {                    \
    _PT_SHARD_BODY                                                        \
  }                                                                       \
  }

#define _PT_SHARD_ADD(I, L, K) shard_maybe_add<I, L, K>(v);
#define _PT_SHARD_BODY PT_EXACT_SHAPES(_PT_SHARD_ADD)
