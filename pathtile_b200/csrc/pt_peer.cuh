// pt_peer.cuh -- sum of the filter gradient over the ranks of one node, through
// the other GPUs' memory (NVLink / NVSwitch), without a separate collective.
//
// Data-parallel training shards the batch: every rank computes its own dK[H, K]
// and the ranks need the sum.  Each rank owns an exchange buffer that every
// other rank has mapped (CUDA IPC):
//   data  [2][W][H][K] floats   slot (p, r, c): rank r's row c of the call with
//                                epoch parity p
//   flags [2][W][H]    u32      the epoch whose slot (p, r, c) is complete
// For one row c (a channel's K taps) the threads that hold it write it into
// slot (p, rank, c) of every rank's buffer (plain stores to peer memory), fence
// at system scope, and one thread per destination publishes the epoch in that
// rank's flag with a release store.  Each rank then waits (bounded) until the
// W flags of row c in its own buffer carry the epoch, and sums the W rows in
// rank order -- the same order on every rank, so all ranks hold the same bits.
// Slots alternate by epoch parity: a rank can only reach call n + 2 after every
// rank has published call n + 1, which each does only after its call-n kernel
// (and its reads of the call-n slots) has finished.  The caller increments the
// epoch by one per call, identically on all ranks, starting at 1 (the buffer
// starts zeroed).  Every wait is bounded; on expiry the kernel sets
// DEVERR_PEER_WAIT in the device error word and leaves the row unwritten.
#pragma once

#include "pt_kernels.cuh"

namespace pt {

constexpr int kMaxPeers = 8;
constexpr unsigned DEVERR_PEER_WAIT = 64u;  // a peer's row never arrived

struct PeerArgs {
  float* data[kMaxPeers];      // rank r's data area as mapped here
  unsigned* flags[kMaxPeers];  // rank r's flags as mapped here
  int rank, world, H, K;
  unsigned epoch;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct PeerSum {
  float sum;  // the rank-ordered sum (threads j < K)
  int ok;     // 0: a peer's row did not arrive in time
};

// Threads [0, nthr) of the CTA (named barrier `bar`; nthr >= max(K, W), a
// multiple of 32) exchange row c: thread j < K brings value v of tap j and gets
// the rank-ordered sum back.  ok is 0 (for every participating thread) when a
// peer's row did not arrive in time.  Not inlined: it runs once per CTA, after
// the kernel's main loop, and inlined its addressing and waits raise the
// register demand of the loop's own role enough to spill.  `pa` refers to a
// __grid_constant__ kernel parameter, so passing its address copies nothing.
static __device__ __noinline__ PeerSum peer_sum_row(const PeerArgs& pa, int c, int tid, int nthr, int bar, float v,
                                                    unsigned* err) {
  const int par = static_cast<int>(pa.epoch & 1u);
  const size_t row = static_cast<size_t>(par * pa.world + pa.rank) * pa.H + c;
  if (tid < pa.K) {
    for (int r = 0; r < pa.world; ++r) pa.data[r][row * pa.K + tid] = v;
  }
  __threadfence_system();
  named_barrier(bar, nthr);
  if (tid < pa.world) st_release_sys(pa.flags[tid] + row, pa.epoch);
  bool ok = true;
  if (tid < pa.world) {
    const unsigned* f = pa.flags[pa.rank] + static_cast<size_t>(par * pa.world + tid) * pa.H + c;
    if (ld_acquire_sys(f) != pa.epoch) {
      const unsigned long long t0 = globaltimer_ns();
      while (ld_acquire_sys(f) != pa.epoch) {
        if (static_cast<long long>(globaltimer_ns() - t0) > static_cast<long long>(WAIT_LIMIT_NS)) {
          atomicOr(err, DEVERR_PEER_WAIT);
          ok = false;
          break;
        }
      }
    }
  }
  PeerSum res{0.f, !named_barrier_or(bar, nthr, !ok)};
  if (res.ok && tid < pa.K) {
    __threadfence_system();
    const float* mine = pa.data[pa.rank];
    for (int r = 0; r < pa.world; ++r)
      res.sum += __ldcg(mine + (static_cast<size_t>(par * pa.world + r) * pa.H + c) * pa.K + tid);
  }
  return res;
}

#ifdef PT_KERNELS_IMPL
// In-place sum over the ranks of dk[H][K]: one CTA per row, one thread per tap
// (blockDim.x = K rounded up to 32, at least W).
__global__ void __launch_bounds__(64) peer_allreduce_kernel(float* __restrict__ dk, const __grid_constant__ PeerArgs pa,
                                                            unsigned* err) {
  const int c = static_cast<int>(blockIdx.x);
  const int tid = static_cast<int>(threadIdx.x);
  const float v = (tid < pa.K) ? dk[static_cast<size_t>(c) * pa.K + tid] : 0.f;
  const PeerSum r = peer_sum_row(pa, c, tid, static_cast<int>(blockDim.x), 1, v, err);
  if (r.ok && tid < pa.K) dk[static_cast<size_t>(c) * pa.K + tid] = r.sum;
}
#endif  // PT_KERNELS_IMPL

}  // namespace pt
