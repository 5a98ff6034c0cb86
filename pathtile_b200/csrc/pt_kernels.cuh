// pt_kernels.cuh -- sm_100a kernels of the short depthwise Conv1D training path.
//
// Math (same-length cross-correlation, left pad K/2, right pad K-1-K/2), the
// contract of the reference path (benchmark/benchmark_shape_sweep_ampere.py:
// 220-239 and kernels/warp_tiled_ampere.py:372-619):
//   FWD  y [b,h,t] = sum_j x [b,h,t+j-K/2]   k[h,j]
//   DX   dx[b,h,t] = sum_j dy[b,h,t-j+K/2]   k[h,j]   (= FWD with reversed taps
//                                                     and left pad K-1-K/2)
//   DK   dk[h,j]   = sum_{b,t} dy[b,h,t] x[b,h,t+j-K/2]
//
// Work decomposition (B200 design, not the reference's): a tile is Tb batches x
// Th channels of whole rows (a row = one (b,h) sequence of L floats).  If H fits
// in the tile (Th = H, "case A") a tile is Tb*H contiguous rows; otherwise the
// channels are split into nhb blocks of Th (Tb = 1, "case B").  A persistent CTA
// keeps one channel block for its whole life, so thread i always owns channel
// hb*Th + i%Th: FWD/DX hold that channel's K taps in registers for the whole
// kernel and DK keeps K per-thread accumulators across all its tiles.
//
// Tiles stream through a ring of `stages` shared-memory buffers filled by TMA:
// a 3-D tensor map (dims L,H,B) when L%4 == 0, whose box is `pitch` floats wide
// so that rows land at a bank-conflict-free pitch for 128-bit LDS, or one 1-D
// bulk copy of the tile's contiguous bytes otherwise.  One thread per row loads
// its row into registers, runs the fully unrolled (L,K) in-range FFMA nest, and
// (FWD/DX) writes the output row back in place; the tile then leaves by a TMA
// store.  Every mbarrier wait is bounded by a %globaltimer limit; on expiry the
// kernel sets a bit in the caller's device error word and returns once its own
// bulk copies have drained.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pt {

enum Op { OP_FWD = 0, OP_DX = 1, OP_DK = 2 };
enum Loader { LOAD_TMA3D = 0, LOAD_BULK1D = 1 };

// Device error bits (written with atomicOr into the error word), one per wait site.
constexpr unsigned DEVERR_TIMEOUT_FULL = 1u;   // consumer: a tile never arrived
constexpr unsigned DEVERR_TIMEOUT_DRAIN = 2u;  // producer: an in-flight copy did not drain
constexpr unsigned DEVERR_TIMEOUT_DONE = 4u;   // producer: a stage's rows were never finished
// Wait limit: far above any legitimate tile latency (microseconds).
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;

struct TileGeom {
  int B, H, L, K;
  int Th, Tb;       // tile = Tb batches x Th channels
  int nhb;          // channel blocks: ceil(H / Th)
  int Q;            // tile positions along the batch: ceil(B / Tb)
  int G;            // persistent CTAs (multiple of nhb)
  int stages;       // ring depth
  int pitch;        // shared-memory row pitch in floats
  unsigned stage_bytes;  // bytes of one stage buffer (one input)
  unsigned tx_bytes;     // TMA transaction bytes of one input per full tile
};

// ---------------------------------------------------------------------------
// PTX helpers (mbarrier, TMA, bulk copies, proxy fences).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for phase `parity` of `bar` for at most `limit_ns`; false (and `errbit`
// set in the error word) on expiry.
__device__ __forceinline__ bool mbar_wait_bounded_for(uint32_t bar, uint32_t parity, unsigned* err,
                                                      unsigned errbit, unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (static_cast<long long>(globaltimer_ns() - t0) > static_cast<long long>(limit_ns)) {
      atomicOr(err, errbit);
      return false;
    }
  }
}

// The wait every kernel uses: bounded by WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, unsigned* err,
                                                  unsigned errbit) {
  return mbar_wait_bounded_for(bar, parity, err, errbit, WAIT_LIMIT_NS);
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Barrier `id` over the first `n` threads (a multiple of 32) of the CTA,
// returning the OR of `pred` over them.
__device__ __forceinline__ bool named_barrier_or(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void named_barrier(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* tm, int c0, int c1,
                                            int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, int c0, int c1,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, uint32_t src, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tm)),
      "r"(src), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* tm, uint32_t src, int c0, int c1,
                                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tm)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void bulk_load_1d(uint32_t dst, const void* src, uint32_t bytes,
                                             uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void bulk_store_1d(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// Dynamic shared memory rounded up to a 1024-byte boundary (the host adds
// 1024 bytes of slack), so every stage buffer is a valid TMA destination.
__device__ __forceinline__ unsigned char* aligned_smem(unsigned char* raw) {
  const uint32_t a = smem_u32(raw);
  return raw + ((1024u - (a & 1023u)) & 1023u);
}

// ---------------------------------------------------------------------------
// Row <-> register movement.  TMA3D rows sit at a pitch that is a multiple of
// 4 floats (128-bit accesses); BULK1D rows are dense at pitch L (64-bit
// accesses when L is even, 32-bit otherwise).
// ---------------------------------------------------------------------------
template <int L, int LOADER>
__device__ __forceinline__ void row_load(const float* __restrict__ p, float (&v)[L]) {
  if constexpr (LOADER == LOAD_TMA3D) {
    static_assert(L % 4 == 0, "TMA3D rows need L % 4 == 0");
#pragma unroll
    for (int c = 0; c < L / 4; ++c) {
      const float4 q = reinterpret_cast<const float4*>(p)[c];
      v[4 * c + 0] = q.x;
      v[4 * c + 1] = q.y;
      v[4 * c + 2] = q.z;
      v[4 * c + 3] = q.w;
    }
  } else if constexpr (L % 2 == 0) {
#pragma unroll
    for (int c = 0; c < L / 2; ++c) {
      const float2 q = reinterpret_cast<const float2*>(p)[c];
      v[2 * c + 0] = q.x;
      v[2 * c + 1] = q.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < L; ++i) v[i] = p[i];
  }
}

template <int L, int LOADER, int T0 = 0, int T1 = L>
__device__ __forceinline__ void row_store(float* __restrict__ p, const float (&v)[L]) {
  if constexpr (LOADER == LOAD_TMA3D) {
#pragma unroll
    for (int c = T0 / 4; c < T1 / 4; ++c)
      reinterpret_cast<float4*>(p)[c] =
          make_float4(v[4 * c + 0], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  } else if constexpr (L % 2 == 0 && T0 % 2 == 0 && T1 % 2 == 0) {
#pragma unroll
    for (int c = T0 / 2; c < T1 / 2; ++c)
      reinterpret_cast<float2*>(p)[c] = make_float2(v[2 * c + 0], v[2 * c + 1]);
  } else {
#pragma unroll
    for (int i = T0; i < T1; ++i) p[i] = v[i];
  }
}

// One output row: y[t] = sum_j in[t + j - PAD] * taps[j], in-range pairs only
// (the out-of-range pairs are dropped at compile time: no predicates).  Four
// outputs advance together so consecutive FFMAs are independent; each output
// still sums its taps in ascending j.
template <int L, int K, int PAD, int T0 = 0, int T1 = L>
__device__ __forceinline__ void conv_row(const float (&in)[L], const float (&taps)[K],
                                         float (&y)[L]) {
  constexpr int G = 4;
#pragma unroll
  for (int t0 = T0; t0 < T1; t0 += G) {
    float acc[G];
#pragma unroll
    for (int u = 0; u < G; ++u) acc[u] = 0.0f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
#pragma unroll
      for (int u = 0; u < G; ++u) {
        const int t = t0 + u;
        const int i = t + j - PAD;
        if (t < T1 && i >= 0 && i < L) acc[u] = fmaf(in[i], taps[j], acc[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < G; ++u)
      if (t0 + u < T1) y[t0 + u] = acc[u];
  }
}

// conv_row with each group of four outputs written to the row at `p` as soon
// as it is complete (the input row is already in registers, so the row may be
// the input's own shared-memory row): four output registers live, not L.
template <int L, int K, int PAD, int LOADER>
__device__ __forceinline__ void conv_row_to_smem(const float (&in)[L], const float (&taps)[K],
                                                 float* __restrict__ p) {
  constexpr int G = 4;
#pragma unroll
  for (int t0 = 0; t0 < L; t0 += G) {
    float acc[G];
#pragma unroll
    for (int u = 0; u < G; ++u) acc[u] = 0.0f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
#pragma unroll
      for (int u = 0; u < G; ++u) {
        const int t = t0 + u;
        const int i = t + j - PAD;
        if (t < L && i >= 0 && i < L) acc[u] = fmaf(in[i], taps[j], acc[u]);
      }
    }
    if constexpr (LOADER == LOAD_TMA3D) {
      *reinterpret_cast<float4*>(p + t0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    } else if constexpr (L % 2 == 0) {
#pragma unroll
      for (int u = 0; u < G; u += 2)
        if (t0 + u < L) *reinterpret_cast<float2*>(p + t0 + u) = make_float2(acc[u], acc[u + 1]);
    } else {
#pragma unroll
      for (int u = 0; u < G; ++u)
        if (t0 + u < L) p[t0 + u] = acc[u];
    }
  }
}

// Output split for two threads per row: the first thread computes outputs
// [0, kSplit), the second [kSplit, L).  A multiple of 4 (128-bit stores) near
// L/2; the in-range FFMA counts of the halves differ by a few percent.
template <int L>
constexpr int row_split() {
  return (L % 4 == 0) ? ((L / 2 + 2) / 4) * 4 : L / 2;
}

// One row's contribution to the filter gradient: acc[j] += sum_t dy[t] x[t+j-PAD].
// t outer / j inner: consecutive FFMAs update different accumulators, so the
// K per-tap chains interleave instead of stalling on FFMA latency.
// With two threads per row (STRIDE = 2) a thread owns the taps j = J0, J0+2, ...
// and acc[m] accumulates tap J0 + STRIDE*m.
template <int L, int K, int PAD, int J0 = 0, int STRIDE = 1>
__device__ __forceinline__ void xcorr_row(const float (&dy)[L], const float (&x)[L],
                                          float (&acc)[(K + STRIDE - 1) / STRIDE]) {
#pragma unroll
  for (int t = 0; t < L; ++t) {
#pragma unroll
    for (int j = J0; j < K; j += STRIDE) {
      const int i = t + j - PAD;
      if (i >= 0 && i < L) acc[(j - J0) / STRIDE] = fmaf(dy[t], x[i], acc[(j - J0) / STRIDE]);
    }
  }
}

// Tile bookkeeping shared by the FWD/DX and DK kernels.
struct TileCursor {
  int hb, q0, qs, n_it;
  __device__ __forceinline__ TileCursor(const TileGeom& g) {
    hb = static_cast<int>(blockIdx.x) % g.nhb;
    q0 = static_cast<int>(blockIdx.x) / g.nhb;
    qs = g.G / g.nhb;
    n_it = (q0 < g.Q) ? (g.Q - q0 + qs - 1) / qs : 0;
  }
  __device__ __forceinline__ int q(int it) const { return q0 + it * qs; }
};

// First row (flattened b*H + h) and row count of tile q in channel block hb.
__device__ __forceinline__ void tile_rows(const TileGeom& g, int hb, int q, long long& row0,
                                          int& nrows) {
  if (g.nhb == 1) {
    const int b0 = q * g.Tb;
    const int nb = min(g.Tb, g.B - b0);
    row0 = static_cast<long long>(b0) * g.H;
    nrows = nb * g.H;
  } else {
    row0 = static_cast<long long>(q) * g.H + static_cast<long long>(hb) * g.Th;
    nrows = min(g.Th, g.H - hb * g.Th);
  }
}

template <int LOADER>
__device__ __forceinline__ void issue_tile_load(const TileGeom& g, const CUtensorMap* tm,
                                                const float* base, int hb, int q, uint32_t dst,
                                                uint32_t bar) {
  if constexpr (LOADER == LOAD_TMA3D) {
    tma_load_3d(dst, tm, 0, hb * g.Th, q * g.Tb, bar);
  } else {
    long long row0;
    int nrows;
    tile_rows(g, hb, q, row0, nrows);
    bulk_load_1d(dst, base + row0 * g.L, static_cast<uint32_t>(nrows) * g.L * 4u, bar);
  }
}

template <int LOADER>
__device__ __forceinline__ uint32_t tile_tx_bytes(const TileGeom& g, int hb, int q) {
  if constexpr (LOADER == LOAD_TMA3D) {
    return g.tx_bytes;  // a TMA box always lands whole (out-of-bounds part zero-filled)
  } else {
    long long row0;
    int nrows;
    tile_rows(g, hb, q, row0, nrows);
    return static_cast<uint32_t>(nrows) * g.L * 4u;
  }
}

// ---------------------------------------------------------------------------
// Warp-specialised persistent kernels.  The CTA is `nc` consumer threads (one
// per tile row, rounded up to whole warps) plus one producer warp whose lane 0
// drives TMA.  Stages are handed over with mbarriers only:
//   full[s]  : producer arrive.expect_tx + TMA bytes -> consumers may read
//   done[s]  : every consumer thread, after its FFMA nest has consumed the row
//              (and, for FWD/DX, written its output row back in place), behind
//              a fence.proxy.async that orders those generic-proxy accesses
//              before the async-proxy store / refill of the stage
// Consumer warps never wait on each other; releasing a stage only after the
// nest means the fence finds nothing outstanding, and shared-memory loads
// overlap the FFMAs.  Every wait is bounded; a thread whose wait expires
// stops, the producer drains the loads it issued, and the error word records it.
// ---------------------------------------------------------------------------
struct PipeBars {
  uint64_t* full;
  uint64_t* done;
};

__device__ __forceinline__ PipeBars carve_bars(unsigned char* base, int stages) {
  uint64_t* b = reinterpret_cast<uint64_t*>(base);
  return PipeBars{b, b + stages};
}

// Producer tail: every stage's most recently issued load has landed (bounded),
// then all bulk stores are complete.
__device__ __forceinline__ void producer_drain(const PipeBars& bars, int stages, int issued,
                                               unsigned* err) {
  for (int t = max(0, issued - stages); t < issued; ++t) {
    const uint32_t parity = static_cast<uint32_t>(t / stages) & 1u;
    if (!mbar_wait_bounded(smem_u32(&bars.full[t % stages]), parity, err, DEVERR_TIMEOUT_DRAIN)) break;
  }
  bulk_wait_all();
}

// ---------------------------------------------------------------------------
// FWD / DX.  Shared memory: tile ring [stages] | mbarriers.  Each consumer
// thread overwrites its input row with its output row; the producer stores the
// tile from the same stage, waits until the store has read it, then refills it.
// ---------------------------------------------------------------------------
template <int L, int K, int OP, int LOADER, int TPR>
__global__ void __launch_bounds__(288, 1)
    conv_rows_kernel(const __grid_constant__ CUtensorMap tm_in,
                     const __grid_constant__ CUtensorMap tm_out, const float* __restrict__ in,
                     const float* __restrict__ taps_hk, float* __restrict__ out, const TileGeom g,
                     unsigned* __restrict__ err) {
  static_assert(OP == OP_FWD || OP == OP_DX, "conv_rows_kernel computes FWD or DX");
  constexpr int PAD = (OP == OP_FWD) ? (K / 2) : (K - 1 - K / 2);
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  const int tid = static_cast<int>(threadIdx.x);
  const int nc = static_cast<int>(blockDim.x) - 32;  // consumer threads
  const TileCursor cur(g);
  const int S = g.stages;
  auto stage_ptr = [&](int s) -> float* {
    return reinterpret_cast<float*>(smem + static_cast<size_t>(s) * g.stage_bytes);
  };
  const PipeBars bars = carve_bars(smem + static_cast<size_t>(S) * g.stage_bytes, S);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.done[s]), static_cast<uint32_t>(nc));
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (tid >= nc) {  // ---------------- producer warp ----------------
    if (tid != nc) return;
    if constexpr (LOADER == LOAD_TMA3D) {
      prefetch_tmap(&tm_in);
      prefetch_tmap(&tm_out);
    }
    auto load = [&](int t) {
      const int s = t % S;
      const int q = cur.q(t);
      const uint32_t bar = smem_u32(&bars.full[s]);
      mbar_arrive_expect_tx(bar, tile_tx_bytes<LOADER>(g, cur.hb, q));
      issue_tile_load<LOADER>(g, &tm_in, in, cur.hb, q, smem_u32(stage_ptr(s)), bar);
    };
    int issued = 0;
    for (; issued < min(S, cur.n_it); ++issued) load(issued);
    for (int it = 0; it < cur.n_it; ++it) {
      const int s = it % S;
      // Every row of tile it has been written back: store it.
      if (!mbar_wait_bounded(smem_u32(&bars.done[s]), static_cast<uint32_t>(it / S) & 1u, err,
                             DEVERR_TIMEOUT_DONE))
        break;
      const int q = cur.q(it);
      if constexpr (LOADER == LOAD_TMA3D) {
        tma_store_3d(&tm_out, smem_u32(stage_ptr(s)), 0, cur.hb * g.Th, q * g.Tb);
      } else {
        long long row0;
        int nrows;
        tile_rows(g, cur.hb, q, row0, nrows);
        bulk_store_1d(out + row0 * g.L, smem_u32(stage_ptr(s)), static_cast<uint32_t>(nrows) * g.L * 4u);
      }
      bulk_commit();
      if (it + S < cur.n_it) {
        bulk_wait_read<0>();  // the store has read stage s: refill it
        load(it + S);
        ++issued;
      }
    }
    producer_drain(bars, S, issued, err);
    return;
  }

  // ---------------- consumer threads: TPR per row ----------------
  // With TPR = 2 the consumer warps form two halves over the same rows; the
  // first computes outputs [0, SPLIT), the second [SPLIT, L).
  constexpr int SPLIT = row_split<L>();
  const int tw = nc / TPR;        // threads per half: whole warps
  const int part = tid / tw;      // warp-uniform
  const int r = tid - part * tw;  // row of the tile
  const int T = g.Th * g.Tb;
  const int h_local = r % g.Th;
  const int b_local = r / g.Th;
  const int h = cur.hb * g.Th + h_local;
  const bool thread_has_row = (r < T) && (h < g.H);
  float taps[K];  // this thread's taps for the whole kernel (reversed for DX)
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const int src = (OP == OP_FWD) ? j : (K - 1 - j);
    taps[j] = thread_has_row ? __ldg(taps_hk + static_cast<long long>(h) * K + src) : 0.0f;
  }
  for (int it = 0; it < cur.n_it; ++it) {
    const int s = it % S;
    if (!mbar_wait_bounded(smem_u32(&bars.full[s]), static_cast<uint32_t>(it / S) & 1u, err,
                           DEVERR_TIMEOUT_FULL))
      return;
    const bool row_valid = thread_has_row && cur.q(it) * g.Tb + b_local < g.B;
    float* rowp = stage_ptr(s) + static_cast<size_t>(r) * g.pitch;
    float yout[L];
    if (row_valid) {
      float xin[L];
      row_load<L, LOADER>(rowp, xin);
      if constexpr (TPR == 1) {
        conv_row<L, K, PAD>(xin, taps, yout);
      } else if (part == 0) {
        conv_row<L, K, PAD, 0, SPLIT>(xin, taps, yout);
      } else {
        conv_row<L, K, PAD, SPLIT, L>(xin, taps, yout);
      }
    }
    if constexpr (TPR == 1) {
      if (row_valid) row_store<L, LOADER>(rowp, yout);
    } else {
      // Both halves have read the rows (in place, one half's outputs would
      // overwrite the other's inputs): meet, then write.
      named_barrier(1 + r / 32, 64);
      if (row_valid) {
        if (part == 0)
          row_store<L, LOADER, 0, SPLIT>(rowp, yout);
        else
          row_store<L, LOADER, SPLIT, L>(rowp, yout);
      }
    }
    fence_proxy_async_smem();
    mbar_arrive(smem_u32(&bars.done[s]));
  }
}

// ---------------------------------------------------------------------------
// DK pass 1.  Shared memory: (dy, x) ring [stages] | mbarriers; a stage is
// released (done[s]) once its rows went through the FFMA nest.  Per-thread
// accumulators run over all tiles; then an in-CTA reduction over the Tb batch
// slots of each channel (fixed order) and either one float atomic per
// (CTA, h, j) or one partial per (CTA, j, h).
// ---------------------------------------------------------------------------
template <int L, int K, int LOADER, int TPR>
__global__ void __launch_bounds__(288, 1)
    dk_rows_kernel(const __grid_constant__ CUtensorMap tm_dy, const __grid_constant__ CUtensorMap tm_x,
                   const float* __restrict__ dy, const float* __restrict__ x,
                   float* __restrict__ dst, const TileGeom g, const int atomic_mode,
                   unsigned* __restrict__ err) {
  constexpr int PAD = K / 2;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  const int tid = static_cast<int>(threadIdx.x);
  const int nc = static_cast<int>(blockDim.x) - 32;
  const TileCursor cur(g);
  const int S = g.stages;
  auto buf = [&](int s, int which) -> float* {
    return reinterpret_cast<float*>(smem + static_cast<size_t>(2 * s + which) * g.stage_bytes);
  };
  const PipeBars bars = carve_bars(smem + static_cast<size_t>(2 * S) * g.stage_bytes, S);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.done[s]), static_cast<uint32_t>(nc));
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (tid >= nc) {  // ---------------- producer warp ----------------
    if (tid != nc) return;
    if constexpr (LOADER == LOAD_TMA3D) {
      prefetch_tmap(&tm_dy);
      prefetch_tmap(&tm_x);
    }
    auto load = [&](int t) {
      const int s = t % S;
      const int q = cur.q(t);
      const uint32_t bar = smem_u32(&bars.full[s]);
      mbar_arrive_expect_tx(bar, 2u * tile_tx_bytes<LOADER>(g, cur.hb, q));
      issue_tile_load<LOADER>(g, &tm_dy, dy, cur.hb, q, smem_u32(buf(s, 0)), bar);
      issue_tile_load<LOADER>(g, &tm_x, x, cur.hb, q, smem_u32(buf(s, 1)), bar);
    };
    int issued = 0;
    for (; issued < min(S, cur.n_it); ++issued) load(issued);
    for (int it = 0; it + S < cur.n_it; ++it) {
      if (!mbar_wait_bounded(smem_u32(&bars.done[it % S]), static_cast<uint32_t>(it / S) & 1u, err,
                             DEVERR_TIMEOUT_DONE))
        break;
      load(it + S);
      ++issued;
    }
    producer_drain(bars, S, issued, err);
    return;
  }

  // ---------------- consumer threads: TPR per row ----------------
  // With TPR = 2 the two halves of the consumer warps read the same rows; the
  // first accumulates the even taps, the second the odd taps.
  constexpr int NACC = (K + TPR - 1) / TPR;
  const int tw = nc / TPR;
  const int part = tid / tw;
  const int r = tid - part * tw;
  const int T = g.Th * g.Tb;
  const int h_local = r % g.Th;
  const int b_local = r / g.Th;
  const int h = cur.hb * g.Th + h_local;
  const bool thread_has_row = (r < T) && (h < g.H);
  float acc[NACC];
#pragma unroll
  for (int m = 0; m < NACC; ++m) acc[m] = 0.0f;
  bool failed = false;
  for (int it = 0; it < cur.n_it; ++it) {
    const int s = it % S;
    if (!mbar_wait_bounded(smem_u32(&bars.full[s]), static_cast<uint32_t>(it / S) & 1u, err,
                           DEVERR_TIMEOUT_FULL)) {
      failed = true;
      break;
    }
    if (thread_has_row && cur.q(it) * g.Tb + b_local < g.B) {
      float gyr[L];
      float xr[L];
      row_load<L, LOADER>(buf(s, 0) + static_cast<size_t>(r) * g.pitch, gyr);
      row_load<L, LOADER>(buf(s, 1) + static_cast<size_t>(r) * g.pitch, xr);
      if constexpr (TPR == 1) {
        xcorr_row<L, K, PAD>(gyr, xr, acc);
      } else if (part == 0) {
        xcorr_row<L, K, PAD, 0, 2>(gyr, xr, acc);
      } else {
        xcorr_row<L, K, PAD, 1, 2>(gyr, xr, acc);
      }
    }
    fence_proxy_async_smem();  // reads of the stage precede its async-proxy refill
    mbar_arrive(smem_u32(&bars.done[s]));
  }
  // All consumers agree before the epilogue reuses the ring (barrier 1 excludes the producer).
  if (named_barrier_or(1, nc, failed)) return;

  float* red = reinterpret_cast<float*>(smem);  // [K][T]; every load was consumed
  if (r < T) {
#pragma unroll
    for (int m = 0; m < NACC; ++m) {
      const int j = part + TPR * m;
      if (j < K) red[j * T + r] = acc[m];
    }
  }
  named_barrier(1, nc);
  const int nh = min(g.Th, g.H - cur.hb * g.Th);
  for (int idx = tid; idx < K * nh; idx += nc) {
    const int j = idx / nh;
    const int hl = idx - j * nh;
    float sum = 0.0f;
    for (int bl = 0; bl < g.Tb; ++bl) sum += red[j * T + bl * g.Th + hl];
    if (atomic_mode) {
      atomicAdd(dst + static_cast<long long>(cur.hb * g.Th + hl) * g.K + j, sum);
    } else {
      dst[(static_cast<long long>(blockIdx.x) * g.K + j) * g.Th + hl] = sum;
    }
  }
}

// ---------------------------------------------------------------------------
// Fused backward on the CUDA cores: dX and dK from one pass over dy and x.
// For the shapes the tensor-core fused kernel does not take (rows of L <= 32
// or L % 4 != 0, or a channel count whose grid cannot keep one channel per
// CTA).  Separately, dX reads dy and writes dx and dK reads dy and x (four
// [B, H, L] streams); here three.  Stages hold the (dy, x) tiles as in DK pass
// 1; each consumer thread takes its dy and x rows into registers, adds the
// row's filter-gradient terms to its K accumulators, computes its dx row from
// the dy row and the channel's reversed taps, and writes it over its dy row.
// The producer stores the dx tile from the dy buffer, waits until the store
// has read it, then refills the stage.  The filter-gradient epilogue is DK
// pass 1's (in-CTA fixed-order sum, then an atomic or a partial per (CTA, j, h));
// it reuses the ring only after the producer reports, on one more mbarrier,
// that its last stores have read shared memory.
// ---------------------------------------------------------------------------
template <int L, int K, int LOADER>
__global__ void __launch_bounds__(288, 1)
    bwd_rows_kernel(const __grid_constant__ CUtensorMap tm_dy, const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_dx, const float* __restrict__ dy,
                    const float* __restrict__ x, const float* __restrict__ taps_hk, float* __restrict__ dx,
                    float* __restrict__ dst, const TileGeom g, const int atomic_mode, unsigned* __restrict__ err) {
  constexpr int PAD_K = K / 2;          // dK: x[t + j - K/2]
  constexpr int PAD_X = K - 1 - K / 2;  // dX: dy[t + j' - (K-1-K/2)] k[K-1-j']
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  const int tid = static_cast<int>(threadIdx.x);
  const int nc = static_cast<int>(blockDim.x) - 32;
  const TileCursor cur(g);
  const int S = g.stages;
  auto buf = [&](int s, int which) -> float* {
    return reinterpret_cast<float*>(smem + static_cast<size_t>(2 * s + which) * g.stage_bytes);
  };
  const PipeBars bars = carve_bars(smem + static_cast<size_t>(2 * S) * g.stage_bytes, S);
  uint64_t* stored = bars.done + S;  // the producer's last stores have read shared memory

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.done[s]), static_cast<uint32_t>(nc));
    }
    mbar_init(smem_u32(stored), 1);
    fence_mbar_init();
  }
  __syncthreads();

  if (tid >= nc) {  // ---------------- producer warp ----------------
    if (tid != nc) return;
    if constexpr (LOADER == LOAD_TMA3D) {
      prefetch_tmap(&tm_dy);
      prefetch_tmap(&tm_x);
      prefetch_tmap(&tm_dx);
    }
    auto load = [&](int t) {
      const int s = t % S;
      const int q = cur.q(t);
      const uint32_t bar = smem_u32(&bars.full[s]);
      mbar_arrive_expect_tx(bar, 2u * tile_tx_bytes<LOADER>(g, cur.hb, q));
      issue_tile_load<LOADER>(g, &tm_dy, dy, cur.hb, q, smem_u32(buf(s, 0)), bar);
      issue_tile_load<LOADER>(g, &tm_x, x, cur.hb, q, smem_u32(buf(s, 1)), bar);
    };
    int issued = 0;
    for (; issued < min(S, cur.n_it); ++issued) load(issued);
    for (int it = 0; it < cur.n_it; ++it) {
      const int s = it % S;
      // Every dx row of tile it is in place over its dy row: store the tile.
      if (!mbar_wait_bounded(smem_u32(&bars.done[s]), static_cast<uint32_t>(it / S) & 1u, err,
                             DEVERR_TIMEOUT_DONE))
        break;
      const int q = cur.q(it);
      if constexpr (LOADER == LOAD_TMA3D) {
        tma_store_3d(&tm_dx, smem_u32(buf(s, 0)), 0, cur.hb * g.Th, q * g.Tb);
      } else {
        long long row0;
        int nrows;
        tile_rows(g, cur.hb, q, row0, nrows);
        bulk_store_1d(dx + row0 * g.L, smem_u32(buf(s, 0)), static_cast<uint32_t>(nrows) * g.L * 4u);
      }
      bulk_commit();
      if (it + S < cur.n_it) {
        bulk_wait_read<0>();  // the store has read stage s: refill it
        load(it + S);
        ++issued;
      }
    }
    producer_drain(bars, S, issued, err);  // loads landed, stores complete
    mbar_arrive(smem_u32(stored));
    return;
  }

  // ---------------- consumer threads: one per row ----------------
  const int r = tid;
  const int T = g.Th * g.Tb;
  const int h_local = r % g.Th;
  const int b_local = r / g.Th;
  const int h = cur.hb * g.Th + h_local;
  const bool thread_has_row = (r < T) && (h < g.H);
  float taps[K];  // reversed: dX is FWD with reversed taps and left pad K-1-K/2
#pragma unroll
  for (int j = 0; j < K; ++j)
    taps[j] = thread_has_row ? __ldg(taps_hk + static_cast<long long>(h) * K + (K - 1 - j)) : 0.0f;
  float acc[K];
#pragma unroll
  for (int j = 0; j < K; ++j) acc[j] = 0.0f;
  bool failed = false;
  for (int it = 0; it < cur.n_it; ++it) {
    const int s = it % S;
    if (!mbar_wait_bounded(smem_u32(&bars.full[s]), static_cast<uint32_t>(it / S) & 1u, err,
                           DEVERR_TIMEOUT_FULL)) {
      failed = true;
      break;
    }
    if (thread_has_row && cur.q(it) * g.Tb + b_local < g.B) {
      float* dyp = buf(s, 0) + static_cast<size_t>(r) * g.pitch;
      float gyr[L];
      row_load<L, LOADER>(dyp, gyr);
      {
        float xr[L];
        row_load<L, LOADER>(buf(s, 1) + static_cast<size_t>(r) * g.pitch, xr);
        xcorr_row<L, K, PAD_K>(gyr, xr, acc);
      }
      conv_row_to_smem<L, K, PAD_X, LOADER>(gyr, taps, dyp);
    }
    fence_proxy_async_smem();  // the dx row write precedes the async-proxy store
    mbar_arrive(smem_u32(&bars.done[s]));
  }
  if (named_barrier_or(1, nc, failed)) return;
  // The ring becomes the reduction buffer once the producer's stores have read it.
  bool ok = mbar_wait_bounded(smem_u32(stored), 0, err, DEVERR_TIMEOUT_DONE);
  if (named_barrier_or(1, nc, !ok)) return;

  float* red = reinterpret_cast<float*>(smem);  // [K][T]
  if (r < T) {
#pragma unroll
    for (int j = 0; j < K; ++j) red[j * T + r] = acc[j];
  }
  named_barrier(1, nc);
  const int nh = min(g.Th, g.H - cur.hb * g.Th);
  for (int idx = tid; idx < K * nh; idx += nc) {
    const int j = idx / nh;
    const int hl = idx - j * nh;
    float sum = 0.0f;
    for (int bl = 0; bl < g.Tb; ++bl) sum += red[j * T + bl * g.Th + hl];
    if (atomic_mode) {
      atomicAdd(dst + static_cast<long long>(cur.hb * g.Th + hl) * g.K + j, sum);
    } else {
      dst[(static_cast<long long>(blockIdx.x) * g.K + j) * g.Th + hl] = sum;
    }
  }
}

// ---------------------------------------------------------------------------
// Generic kernels: shapes outside the specialisation table (any L <= 48,
// K <= 48, any alignment of H*L), with the
// nests compiled for maxima LMAX, KMAX in {16, 32, 48} and the runtime L, K
// taken by zero-padding the row past L and shifting the taps by
// s = PMAX - pad (tap register j' multiplies element t + j' - PMAX; PMAX =
// KMAX/2 for FWD / dK, KMAX/2 - 1 for dX, which keeps s >= 0 and s + K <= KMAX
// for every K <= KMAX).  Rows and taps live in registers, so the FMAs are
// compile-time; the staging is the generic kernels' coalesced one.
// ---------------------------------------------------------------------------
template <int LMAX, int KMAX, int OP>
__global__ void __launch_bounds__(128)
    conv_bucket_kernel(const float* __restrict__ in, const float* __restrict__ taps_hk, float* __restrict__ out,
                       int B, int H, int L, int K, long long n_tiles) {
  static_assert(OP == OP_FWD || OP == OP_DX, "FWD or DX");
  constexpr int ROWS = 128;
  constexpr int PMAX = (OP == OP_FWD) ? KMAX / 2 : KMAX / 2 - 1;
  __shared__ float s_io[ROWS * 48];
  const int tid = static_cast<int>(threadIdx.x);
  const long long S = static_cast<long long>(B) * H;
  const int pad = (OP == OP_FWD) ? (K / 2) : (K - 1 - K / 2);
  const int s = PMAX - pad;
  for (long long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const long long r0 = tile * ROWS;
    const int nrows = static_cast<int>(min(static_cast<long long>(ROWS), S - r0));
    const int nelem = nrows * L;
    const float* src = in + r0 * L;
    for (int e = tid; e < nelem; e += ROWS) s_io[e] = src[e];
    __syncthreads();
    float v[LMAX];
    float w[KMAX];
    if (tid < nrows) {
#pragma unroll
      for (int t = 0; t < LMAX; ++t) v[t] = (t < L) ? s_io[tid * L + t] : 0.f;
      const int hh = static_cast<int>((r0 + tid) % H);
      const float* kp = taps_hk + static_cast<long long>(hh) * K;
#pragma unroll
      for (int jp = 0; jp < KMAX; ++jp) {
        const int j = jp - s;
        w[jp] = (j >= 0 && j < K) ? __ldg(kp + (OP == OP_FWD ? j : K - 1 - j)) : 0.f;
      }
    }
    __syncthreads();  // the rows are in registers: the tile buffer takes the outputs
    if (tid < nrows) {
#pragma unroll
      for (int t0 = 0; t0 < LMAX; t0 += 4) {
        if (t0 < L) {
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int jp = 0; jp < KMAX; ++jp)
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int i = t0 + u + jp - PMAX;
              if (i >= 0 && i < LMAX) acc[u] = fmaf(w[jp], v[i], acc[u]);
            }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (t0 + u < L) s_io[tid * L + t0 + u] = acc[u];
        }
      }
    }
    __syncthreads();
    float* dstp = out + r0 * L;
    for (int e = tid; e < nelem; e += ROWS) dstp[e] = s_io[e];
    __syncthreads();
  }
}

// dK pass 1 for the same shapes: CTA c owns the batches b = c, c + G, ... of
// every channel (partial layout [G][K][H], reduced by dk_reduce_kernel; or
// atomic adds into dk).  Per group of 32 channels, each warp takes a share of the CTA's
// batches: it stages its 32 rows of x and dy (contiguous in [B, H, L]) through
// shared memory, each lane takes its channel's two rows into registers and
// accumulates the KMAX shifted taps; the warps' sums meet in a fixed order.
template <int LMAX, int KMAX>
__global__ void __launch_bounds__(128)
    dk_bucket_kernel(const float* __restrict__ dy, const float* __restrict__ x, float* __restrict__ dst, int B,
                     int H, int L, int K, int G, int atomic_mode) {
  constexpr int PMAX = KMAX / 2;
  // Row staging [warp][x|dy][32 rows x L]; after each channel group the same
  // memory holds the warps' sums [warp][KMAX][33].
  __shared__ float s_buf[4 * 2 * 32 * 48];
  static_assert(4 * KMAX * 33 <= 4 * 2 * 32 * 48, "reduction fits the staging buffer");
  auto s_rows = [&](int ww, int which) { return s_buf + (ww * 2 + which) * (32 * 48); };
  auto s_red = [&](int ww, int jp) { return s_buf + (ww * KMAX + jp) * 33; };
  const int lane = static_cast<int>(threadIdx.x) & 31;
  const int w = static_cast<int>(threadIdx.x) >> 5;
  const int c = static_cast<int>(blockIdx.x);
  const int s = PMAX - K / 2;  // acc[j'] is the gradient of tap j' - s
  for (int h0 = 0; h0 < H; h0 += 32) {
    const int nch = min(32, H - h0);
    float acc[KMAX];
#pragma unroll
    for (int jp = 0; jp < KMAX; ++jp) acc[jp] = 0.f;
    for (int b = c + G * w; b < B; b += 4 * G) {
      const long long row0 = (static_cast<long long>(b) * H + h0) * L;
      const int nelem = nch * L;
      float* sx = s_rows(w, 0);
      float* sd = s_rows(w, 1);
      for (int e = lane; e < nelem; e += 32) {
        sx[e] = __ldg(x + row0 + e);
        sd[e] = __ldg(dy + row0 + e);
      }
      __syncwarp();
      if (lane < nch) {
        float v[LMAX], d[LMAX];
#pragma unroll
        for (int t = 0; t < LMAX; ++t) {
          v[t] = (t < L) ? sx[lane * L + t] : 0.f;
          d[t] = (t < L) ? sd[lane * L + t] : 0.f;
        }
#pragma unroll
        for (int t = 0; t < LMAX; ++t)
#pragma unroll
          for (int jp = 0; jp < KMAX; ++jp) {
            const int i = t + jp - PMAX;
            if (i >= 0 && i < LMAX) acc[jp] = fmaf(d[t], v[i], acc[jp]);
          }
      }
      __syncwarp();  // the staging buffer is refilled for the next batch
    }
    __syncthreads();  // every warp is done with its staging rows
#pragma unroll
    for (int jp = 0; jp < KMAX; ++jp) s_red(w, jp)[lane] = acc[jp];
    __syncthreads();
    for (int idx = static_cast<int>(threadIdx.x); idx < K * 32; idx += 128) {
      const int j = idx >> 5, ch = idx & 31;
      if (ch < nch) {
        const int jp = j + s;
        const float sum = s_red(0, jp)[ch] + s_red(1, jp)[ch] + s_red(2, jp)[ch] + s_red(3, jp)[ch];
        const int hh = h0 + ch;
        if (atomic_mode)
          atomicAdd(dst + static_cast<long long>(hh) * K + j, sum);
        else
          dst[(static_cast<long long>(c) * K + j) * H + hh] = sum;
      }
    }
    __syncthreads();
  }
}

#ifdef PT_KERNELS_IMPL
// Non-template kernels are emitted by exactly one unit (pt_api.cu).

// ---------------------------------------------------------------------------
// DK pass 2 (deterministic): dk[h,j] (+)= sum over the CTAs of h's channel
// block, in ascending CTA order split over 8 warps, then warp-ordered combine.
// partial layout [G][K][Th].  Grid (ceil(H/32), K), block 256.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) dk_reduce_kernel(const float* __restrict__ partial,
                                                        float* __restrict__ dk, const TileGeom g,
                                                        const int accumulate) {
  __shared__ float sums[8][33];
  const int lane = static_cast<int>(threadIdx.x) & 31;
  const int w = static_cast<int>(threadIdx.x) >> 5;
  const int h = static_cast<int>(blockIdx.x) * 32 + lane;
  const int j = static_cast<int>(blockIdx.y);
  float s = 0.0f;
  if (h < g.H) {
    const int hb = h / g.Th;
    const int hl = h - hb * g.Th;
    const int step = g.nhb * 8;
    const long long cstride = static_cast<long long>(g.K) * g.Th;
    const float* base = partial + static_cast<long long>(j) * g.Th + hl;
    // Batches of 8 independent loads, then the adds in ascending CTA order:
    // the same summation order as a plain loop, with 8 L2 requests in flight.
    for (int c0 = hb + g.nhb * w; c0 < g.G; c0 += 8 * step) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * step;
        v[u] = (c < g.G) ? __ldg(base + c * cstride) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) s += v[u];
    }
  }
  sums[w][lane] = s;
  __syncthreads();
  if (w == 0 && h < g.H) {
    float total = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) total += sums[k][lane];
    float* o = dk + static_cast<long long>(h) * g.K + j;
    *o = accumulate ? (*o + total) : total;
  }
}

#endif  // PT_KERNELS_IMPL

}  // namespace pt
