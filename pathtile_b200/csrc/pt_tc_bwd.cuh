// pt_tc_bwd.cuh -- fused backward: dX on the tensor cores and dK on the CUDA
// cores, in one pass over dy and x (rows of up to 48 columns).
//
// Separately, dX reads dy and writes dx, and dK reads dy and x: four [B, H, L]
// streams.  Here one kernel reads dy and x once and writes dx (three streams),
// and the two halves of the work use different pipes: the dX product runs as
// in tc_conv_kernel<DX> (3xTF32 split, Toeplitz operand resident in shared
// memory), while the row threads that split dy for it also accumulate the
// filter gradient of their row with packed FFMAs.
//
// Work: tiles of 128 batch rows of one channel.  A CTA keeps the channel's
// Toeplitz operand and its threads' dK accumulators, so it wants one channel
// for as long as possible; the SMs, not the channels, set the grid.  The host
// chooses a schedule (BwdSched):
//   * primaries: kp CTAs per channel (CTA g < kp*H has channel g % H and
//     takes batch blocks r, r + kp, r + 2 kp, ... below P, r = g / H);
//   * helpers: the E = G - kp*H remaining CTAs take the tail blocks [P, nblk)
//     of every channel: helper e owns channels e, e + E, e + 2E, ... and does
//     their tail blocks one channel after the other, so at any time the
//     helpers read one batch block of E adjacent channels (contiguous in HBM)
//     while the primaries read the blocks below P of all channels.
// P balances the two (the host counts a channel switch as one tile), so every
// SM has work: at B = 16384, H = 128 on 148 SMs the longest CTA does 113
// tiles instead of 128.  Without helpers (E = 0) the schedule is the
// round-robin one-channel-per-CTA grid.
//
// dK: each CTA accumulates per channel "segment" (a primary has one; a helper
// one per channel it owns) and, at the segment's end, reduces its threads'
// sums in a fixed order -- a warp shuffle over the 32 rows of each TMEM lane
// quadrant, one partial per (quadrant, tap) -- and writes them to the
// workspace; bwd_dk_reduce_kernel then sums each channel's partials in a fixed
// order (deterministic).  With one CTA per channel and no helpers ("direct"),
// the CTA sums its four quadrants itself and writes dK.
//
// Roles (512 threads = four warpgroups, one CTA per SM):
//   warp 0       TMA producer: ring of 3 stages, each the dy and x tiles
//   warp 1       allocates 512 TMEM columns; lane 0 issues the dX MMAs
//   warps 2-3    no role after the set-up
//   warps 4-11   row workers, two per tile row: split half of the dy row into
//                TMEM (A of dX), then dK for the even or odd taps over the
//                whole row, streaming dy from shared memory four columns at a
//                time against the x row in registers; release the stage; at a
//                channel switch, flush dK and rebuild the Toeplitz operand
//   warps 12-15  dX epilogue: TMEM -> staging -> TMA store
// After the set-up the CTA's 512 x 128 registers are rebalanced with
// setmaxnreg (warpgroup 0: 72, row workers: 160, epilogue: 120; no region
// spills).  The host launches the kernel only where the compiled function
// starts with 128 registers per thread, the split's budget.  Every wait is
// bounded; on expiry the kernel records a bit in the device error word, drains
// its own copies and MMAs, frees its tensor memory and returns; dK is then
// undefined.
#pragma once

#include "pt_peer.cuh"
#include "pt_tc.h"
#include "pt_tc_kernels.cuh"

namespace pt {
namespace tc {

constexpr int BWD_STAGES = 3;
constexpr int BWD_L = 48;
constexpr int BWD_THREADS = 512;
constexpr int BWD_LAUNCH_THREADS = BWD_THREADS;
constexpr int BWD_LAUNCH_REGS = 128;  // registers per thread at launch (65,536 / 512)
constexpr int BWD_ROW0 = 128;         // first row-worker thread (warp 4)
constexpr int BWD_ROWS = 256;         // row workers
constexpr int BWD_EPI0 = 384;         // first epilogue thread (warp 12)
constexpr int BWD_REG_CTRL = 72;
constexpr int BWD_REG_ROWS = 160;
constexpr int BWD_REG_EPI = 120;
static_assert(128 * BWD_REG_CTRL + BWD_ROWS * BWD_REG_ROWS + 128 * BWD_REG_EPI <= BWD_THREADS * BWD_LAUNCH_REGS,
              "the register split must fit the registers the CTA is launched with");

struct BwdGeo {
  using GG = Geo<3>;                                  // 48-column tiles: 128-B + 64-B boxes
  static constexpr int N = GG::N;                     // 48
  static constexpr int TILE = GG::TILE;               // 24 KB
  static constexpr int STAGE = 2 * TILE;              // dy | x
  static constexpr int OFF_OUT = BWD_STAGES * STAGE;
  static constexpr int OFF_B = OFF_OUT + OUT_SLOTS * TILE;
  static constexpr int OFF_BAR = OFF_B + GG::BMAT;    // one resident Toeplitz operand
  // full, sfree, mfree per stage; aready, adone per A slot; mdone, accfree per
  // accumulator; tready (the Toeplitz operand of a new channel is built).
  static constexpr int N_BARS = 3 * BWD_STAGES + 2 * A_SLOTS + 2 * ACC_SLOTS + 1;
  static constexpr int OFF_RED = OFF_BAR + N_BARS * 8;  // [4 quadrants][48] direct-mode dK sums
  static constexpr int OFF_TMEM = OFF_RED + 4 * BWD_L * 4;
  static constexpr int SMEM = OFF_TMEM + 16 + 1024;
  static_assert(STAGE % 1024 == 0 && OFF_B % 1024 == 0, "swizzled buffers start on 1024-byte boundaries");
};

struct BwdTile {
  int ch, blk, seg;
};

__device__ __forceinline__ int bwd_n_tiles(const BwdSched& sc, int g) {
  if (g < sc.kp * sc.H) {
    const int r = g / sc.H;
    return r < sc.P ? (sc.P - r + sc.kp - 1) / sc.kp : 0;
  }
  const int e = g - sc.kp * sc.H;
  const int nch = (sc.H - e + sc.E - 1) / sc.E;
  return nch * (sc.nblk - sc.P);
}

__device__ __forceinline__ BwdTile bwd_tile(const BwdSched& sc, int g, int i) {
  if (g < sc.kp * sc.H) return BwdTile{g % sc.H, g / sc.H + i * sc.kp, 0};
  const int e = g - sc.kp * sc.H;
  const int tp = sc.nblk - sc.P;
  const int seg = i / tp;
  return BwdTile{e + seg * sc.E, sc.P + (i - seg * tp), seg};
}

// Workspace slot of (CTA g, segment seg): primaries g, helpers kp*H + e*m + seg;
// a slot holds [4 quadrants][K] partial sums.
__device__ __forceinline__ int bwd_slot(const BwdSched& sc, int g, int seg) {
  return g < sc.kp * sc.H ? g : sc.kp * sc.H + (g - sc.kp * sc.H) * sc.m + seg;
}

// D (+)= A B with A read from shared memory through a descriptor (tf32 operands).
__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// dy - (dy with its low 13 mantissa bits cleared): the part of dy a tf32 MMA,
// which ignores those bits, does not see.  Exact in fp32.
__device__ __forceinline__ float bwd_tf32_rest(float v) {
  return v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
}

// Filter-gradient share of one row worker.  The two workers of a tile row take
// the even (half 0) and odd (half 1) taps, j = 2 jj + half, over the whole row:
//   acc[jj] += sum_t dy[t] x[t + 2 jj + half - PAD].
// With X[m + 1] = x[m + half] (X = [0, x0 .. x47] for half 0 and
// [x0 .. x47, 0] for half 1) both halves run one instruction stream,
//   acc[jj] += dy[t] X[t + 2 jj - PAD + 1],   t + 2 jj - PAD in [-1, 48),
// so the two warps that share an SM sub-partition share its instruction cache
// (separate nests per half thrashed it).  dy arrives four columns at a time as
// 16-byte chunks of the swizzled row: one conflict-free LDS.128 per chunk.
template <int K>
struct BwdSplit {
  static constexpr int NJ = (K + 1) / 2;  // taps per row worker
};

// Packed FP32 pairs: fma.rn.f32x2 does two FMAs in one issue slot (same FMA
// pipe throughput as two FFMAs, half the instructions).
__device__ __forceinline__ uint64_t bwd_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float bwd_pair_sum(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo + hi;
}
__device__ __forceinline__ uint64_t bwd_ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// The same sum with even and odd t accumulated apart, two taps-by-column
// products per instruction:
//   (accE, accO)[jj] += (dy[t], dy[t+1]) * (X[k], X[k+1]),  t even,
//   k = t + 2 jj - PAD + 1,
// whose parity is fixed by K, so the X pairs are packed once per tile (XP) and
// the dy pairs are the halves of each 16-byte chunk.  X outside [0, 49) is 0.
template <int K>
struct BwdPairs {
  static constexpr int PAD = K / 2;
  static constexpr int NJ = BwdSplit<K>::NJ;
  static constexpr int KB = ((1 - PAD) % 2 + 2) % 2;  // parity of every k
  // first k >= max(1 - PAD, -1) with parity KB
  static constexpr int K0 = ((1 - PAD) >= -1) ? (1 - PAD) : ((-1 - KB) % 2 == 0 ? -1 : 0);
  static constexpr int KMAX0 = 46 + 2 * (NJ - 1) - PAD + 1;
  static constexpr int K1 = KMAX0 < 48 ? KMAX0 : (48 - ((48 - KB) % 2 != 0));
  static constexpr int NQ = (K1 - K0) / 2 + 1;  // packed X pairs
};

template <int K>
__device__ __forceinline__ void bwd_dk_row2(const unsigned char* dyrow128, const unsigned char* dyrow64,
                                            uint32_t xm128, uint32_t xm64,
                                            const uint64_t (&XP)[BwdPairs<K>::NQ],
                                            uint64_t (&acc)[BwdSplit<K>::NJ]) {
  using P = BwdPairs<K>;
  constexpr int NJ = P::NJ;
#pragma unroll
  for (int c = 0; c < BWD_L / 4; ++c) {
    bool any = false;
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int jj = 0; jj < NJ; ++jj) {
        const int k = 4 * c + 2 * u + 2 * jj - P::PAD + 1;
        any = any || (k >= P::K0 && k <= P::K1);
      }
    if (!any) continue;
    const ulonglong2 q = (c < 8) ? *reinterpret_cast<const ulonglong2*>(dyrow128 + ((16u * c) ^ xm128))
                                 : *reinterpret_cast<const ulonglong2*>(dyrow64 + ((16u * (c - 8)) ^ xm64));
    const uint64_t d[2] = {q.x, q.y};
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int jj = 0; jj < NJ; ++jj) {
        const int k = 4 * c + 2 * u + 2 * jj - P::PAD + 1;
        if (k >= P::K0 && k <= P::K1) acc[jj] = bwd_ffma2(d[u], XP[(k - P::K0) / 2], acc[jj]);
      }
  }
}

template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(N));
}

// The channel's Toeplitz operand for dX, T[s][t] = k[t - s + K/2], into the
// operand buffer, by `nthr` threads (thread index `tid`).
template <int K>
__device__ __forceinline__ void bwd_build_toeplitz(unsigned char* bm, const float* __restrict__ taps, int ch,
                                                   int tid, int nthr) {
  using GG = Geo<3>;
  constexpr int N = GG::N;
  const int pad = K / 2;
  const float* kh = taps + static_cast<size_t>(ch) * K;
  constexpr int CPR = N / 4;
  for (int task = tid; task < N * CPR; task += nthr) {
    const int c4 = task / N;
    const int tp = task - c4 * N;
    const int sp = 4 * c4;
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int j = tp - (sp + q) + pad;
      v[q] = (j >= 0 && j < K) ? __ldg(kh + j) : 0.f;
    }
    float4 hi, lo;
    split4(make_float4(v[0], v[1], v[2], v[3]), hi, lo);
    if (c4 < GG::C128) {
      *reinterpret_cast<float4*>(bm + sw128_off(tp, c4)) = hi;
      *reinterpret_cast<float4*>(bm + GG::BLO128 + sw128_off(tp, c4)) = lo;
    } else {
      unsigned char* b64 = bm + GG::BBOX64;
      *reinterpret_cast<float4*>(b64 + sw64_off(tp, c4 - GG::C128)) = hi;
      *reinterpret_cast<float4*>(b64 + GG::BLO64 + sw64_off(tp, c4 - GG::C128)) = lo;
    }
  }
}

// part: workspace of [slots][4][K] partials (unused when sc.direct); dk: written
// directly (=, or += when accumulate != 0) when sc.direct -- then, with
// pa.world > 1, as the sum over the ranks of their dK rows, exchanged through
// the other GPUs' memory by the same CTA that computed the row (pt_peer.cuh).
template <int K>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    tc_bwd_kernel(const __grid_constant__ CUtensorMap tm_dy128, const __grid_constant__ CUtensorMap tm_dy64,
                  const __grid_constant__ CUtensorMap tm_x128, const __grid_constant__ CUtensorMap tm_x64,
                  const __grid_constant__ CUtensorMap tm_dx128, const __grid_constant__ CUtensorMap tm_dx64,
                  const float* __restrict__ taps, float* __restrict__ part, float* __restrict__ dk,
                  const BwdSched sc, int accumulate, const __grid_constant__ PeerArgs pa, unsigned* err) {
  using GG = Geo<3>;
  using BG = BwdGeo;
  constexpr int N = GG::N;
  constexpr int L = BWD_L;
  constexpr int NJ = BwdSplit<K>::NJ;  // accumulators per row worker
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = aligned_smem(smem_raw);
  const uint32_t base = smem_u32(sm);
  const int warp = static_cast<int>(threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31);
  const uint32_t bar0 = base + BG::OFF_BAR;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto sfree = [&](int s) { return bar0 + 8u * (BWD_STAGES + s); };
  auto aready = [&](int a) { return bar0 + 8u * (2 * BWD_STAGES + a); };
  auto adone = [&](int a) { return bar0 + 8u * (2 * BWD_STAGES + A_SLOTS + a); };
  auto mdone = [&](int d) { return bar0 + 8u * (2 * BWD_STAGES + 2 * A_SLOTS + d); };
  auto accfree = [&](int d) { return bar0 + 8u * (2 * BWD_STAGES + 2 * A_SLOTS + ACC_SLOTS + d); };
  // The dX MMAs of the tile in stage s have completed (they read its dy half).
  auto mfree = [&](int s) { return bar0 + 8u * (2 * BWD_STAGES + 2 * A_SLOTS + 2 * ACC_SLOTS + s); };
  const uint32_t tready = bar0 + 8u * (3 * BWD_STAGES + 2 * A_SLOTS + 2 * ACC_SLOTS);
  const int g = static_cast<int>(blockIdx.x);
  const int n_it = bwd_n_tiles(sc, g);
  const BwdTile first = bwd_tile(sc, g, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < BWD_STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(sfree(s), BWD_ROWS / 32);
      mbar_init(mfree(s), 1);
    }
    for (int a = 0; a < A_SLOTS; ++a) {
      mbar_init(aready(a), BWD_ROWS / 32);
      mbar_init(adone(a), 1);
    }
    for (int d = 0; d < ACC_SLOTS; ++d) {
      mbar_init(mdone(d), 1);
      mbar_init(accfree(d), 4);
    }
    mbar_init(tready, 1);
    fence_mbar_init();
  }
  // The first channel's Toeplitz operand, by the whole CTA.
  bwd_build_toeplitz<K>(sm + BG::OFF_B, taps, first.ch, static_cast<int>(threadIdx.x), BWD_THREADS);
  fence_proxy_async_smem();  // the MMAs read the operand through the async proxy
  if (warp == 1) {
    tmem_alloc(base + BG::OFF_TMEM, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + BG::OFF_TMEM);

  if (warp < 4) {
    setmaxnreg_dec<BWD_REG_CTRL>();
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer ----------------
      int issued = 0;
      for (int i = 0; i < n_it; ++i) {
        const int s = i % BWD_STAGES;
        if (i >= BWD_STAGES &&
            (!mbar_wait_bounded(sfree(s), ((i / BWD_STAGES) - 1) & 1, err, DEVERR_TIMEOUT_DONE) ||
             !mbar_wait_bounded(mfree(s), ((i / BWD_STAGES) - 1) & 1, err, DEVERR_TIMEOUT_DONE)))
          break;
        const BwdTile t = bwd_tile(sc, g, i);
        const int b0 = t.blk * M;
        const uint32_t st = base + static_cast<uint32_t>(s * BG::STAGE);
        mbar_arrive_expect_tx(full(s), BG::STAGE);
        tma_load_3d(st, &tm_dy128, 0, t.ch, b0, full(s));
        tma_load_3d(st + GG::BOX64, &tm_dy64, GG::S64, t.ch, b0, full(s));
        tma_load_3d(st + BG::TILE, &tm_x128, 0, t.ch, b0, full(s));
        tma_load_3d(st + BG::TILE + GG::BOX64, &tm_x64, GG::S64, t.ch, b0, full(s));
        issued = i + 1;
      }
      for (int i = issued > BWD_STAGES ? issued - BWD_STAGES : 0; i < issued; ++i)
        if (!mbar_wait_bounded(full(i % BWD_STAGES), (i / BWD_STAGES) & 1, err, DEVERR_TIMEOUT_DRAIN)) break;
    } else if (warp == 1 && lane == 0) {
      // ---------------- MMA issuer (dX) ----------------
      constexpr uint32_t idesc_n2 = idesc_tf32_m128<2 * N>();
      constexpr uint32_t idesc_n = idesc_tf32_m128<N>();
      int issued = 0;
      int seg = 0;
      for (int i = 0; i < n_it; ++i) {
        const int a = i % A_SLOTS, d = i % ACC_SLOTS, s = i % BWD_STAGES;
        const int tseg = bwd_tile(sc, g, i).seg;
        // A new channel: its Toeplitz operand must be in place.
        if (tseg != seg) {
          if (!mbar_wait_bounded(tready, (tseg - 1) & 1, err, DEVERR_TC_MMA)) break;
          seg = tseg;
        }
        // The stage's dy tile is the A_hi operand: wait for its load as well.
        if (!mbar_wait_bounded(full(s), (i / BWD_STAGES) & 1, err, DEVERR_TC_MMA)) break;
        if (!mbar_wait_bounded(aready(a), (i / A_SLOTS) & 1, err, DEVERR_TC_MMA)) break;
        if (i >= ACC_SLOTS &&
            !mbar_wait_bounded(accfree(d), ((i / ACC_SLOTS) - 1) & 1, err, DEVERR_TC_MMA))
          break;
        tc_fence_after();
        const uint32_t a_lo = tmem + static_cast<uint32_t>(A_COL0 + a * A_SLOT_COLS + LO_COLS);
        const uint32_t dyt = base + static_cast<uint32_t>(s * BG::STAGE);
        const uint32_t bmat = base + static_cast<uint32_t>(BG::OFF_B);
        const uint32_t dacc = tmem + static_cast<uint32_t>(D_COL0 + d * D_SLOT_COLS);
#pragma unroll
        for (int kk = 0; kk < GG::KSTEPS; ++kk) {
          const bool in128 = kk < GG::K128;
          const uint64_t bdesc = kmajor_desc(
              bmat + (in128 ? 32u * kk : GG::BBOX64 + 32u * (kk - GG::K128)), in128);
          const uint64_t adesc = kmajor_desc(
              dyt + (in128 ? 32u * kk : GG::BOX64 + 32u * (kk - GG::K128)), in128);
          mma_tf32_ss(dacc, adesc, bdesc, idesc_n2, kk > 0);    // dy (tf32 part) [T_hi; T_lo]
          mma_tf32_ts(dacc, a_lo + 8u * kk, bdesc, idesc_n, 1);  // dy rest T_hi
        }
        mma_commit(adone(a));
        mma_commit(mfree(s));
        mma_commit(mdone(d));
        issued = i + 1;
      }
      if (issued > 0)
        mbar_wait_bounded(mdone((issued - 1) % ACC_SLOTS), ((issued - 1) / ACC_SLOTS) & 1, err,
                          DEVERR_TC_MMA);
    }
    __syncwarp();
  } else if (warp < BWD_EPI0 / 32) {
    setmaxnreg_inc<BWD_REG_ROWS>();
    // ---------------- row workers ----------------
    const int ct = static_cast<int>(threadIdx.x) - BWD_ROW0;  // 0..255
    const int quad = warp & 3;
    const int row = 32 * quad + lane;                   // tile row (TMEM lane)
    const int half = ct >> 7;                           // dX: half of the row; dK: even or odd taps
    constexpr int CH = (GG::C128 + GG::C64) / 2;        // 6 chunks per half row
    const uint32_t lane_base = static_cast<uint32_t>(32 * quad) << 16;
    // In-row byte offset of 16-byte chunk c of this row: (16 c) ^ xm128 in the
    // 128-B box (chunks 0-7), (16 c) ^ xm64 in the 64-B box (chunks 0-3).
    const uint32_t xm128 = static_cast<uint32_t>(row & 7) << 4;
    const uint32_t xm64 = static_cast<uint32_t>((row >> 1) & 3) << 4;
    uint64_t acc[NJ];  // (even t, odd t) partial sums per tap
#pragma unroll
    for (int jj = 0; jj < NJ; ++jj) acc[jj] = 0ull;
    // The segment's dK: a warp sum over the quadrant's 32 rows per tap, then
    // one partial per (quadrant, tap) -- to the workspace, or (direct) to shared
    // memory for the CTA's own fixed-order sum.
    auto flush = [&](int seg) {
      float* red = reinterpret_cast<float*>(sm + BG::OFF_RED);
      const int slot = bwd_slot(sc, g, seg);
#pragma unroll
      for (int jj = 0; jj < NJ; ++jj) {
        float v = bwd_pair_sum(acc[jj]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        const int j = 2 * jj + half;
        if (lane == 0 && j < K) {
          if (sc.direct)
            red[quad * L + j] = v;
          else
            part[(static_cast<size_t>(slot) * 4 + quad) * K + j] = v;
        }
        acc[jj] = 0ull;
      }
    };
    // Every row worker takes the same path through the named barriers below
    // (the channel switches depend only on the CTA and the tile index), also
    // after a wait has run out: a warp that failed skips the work, not the
    // barriers.
    bool ok = true;
    // Tiles [seg_begin, seg_end) belong to one channel: a primary has one
    // segment, a helper one per channel it owns (tp tiles each).
    const bool helper = g >= sc.kp * sc.H;
    const int tp = sc.nblk - sc.P;
    int seg = 0;
    for (int i = 0;;) {
      const int seg_end = helper ? min(n_it, (seg + 1) * tp) : n_it;
      for (; i < seg_end; ++i) {
        const int s = i % BWD_STAGES, a = i % A_SLOTS;
        if (ok) {
          if (i >= A_SLOTS) ok = mbar_wait_bounded(adone(a), ((i / A_SLOTS) - 1) & 1, err, DEVERR_TC_CONVERT);
          if (ok) ok = mbar_wait_bounded(full(s), (i / BWD_STAGES) & 1, err, DEVERR_TIMEOUT_FULL);
          ok = __all_sync(0xffffffffu, ok);  // each warp arrives as one, so it decides as one
        }
        if (ok) {
          const unsigned char* st = sm + s * BG::STAGE;
          const unsigned char* dy128 = st + 128u * row;
          const unsigned char* dy64 = st + GG::BOX64 + 64u * row;
          const unsigned char* x128 = st + BG::TILE + 128u * row;
          const unsigned char* x64 = st + BG::TILE + GG::BOX64 + 64u * row;
          // dX: the MMA reads dy's tf32 part straight from the stage; this thread
          // writes the rest of its half of the dy row (A_lo) into tensor memory.
          {
            float lo[4 * CH];
  #pragma unroll
            for (int u = 0; u < CH; ++u) {
              const int c = half * CH + u;
              const uint32_t off = (c < GG::C128) ? sw128_off(row, c) : GG::BOX64 + sw64_off(row, c - GG::C128);
              const float4 q = *reinterpret_cast<const float4*>(st + off);
              lo[4 * u] = bwd_tf32_rest(q.x);
              lo[4 * u + 1] = bwd_tf32_rest(q.y);
              lo[4 * u + 2] = bwd_tf32_rest(q.z);
              lo[4 * u + 3] = bwd_tf32_rest(q.w);
            }
            const uint32_t acol =
                tmem + lane_base + static_cast<uint32_t>(A_COL0 + a * A_SLOT_COLS + LO_COLS + half * 4 * CH);
  #pragma unroll
            for (int u = 0; u < CH / 2; ++u) tmem_st8(acol + 8u * u, lo + 8 * u);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(aready(a));
          }
          // dK: the x row in registers, dy[t] streamed from shared memory.
          {
            float x[L];
  #pragma unroll
            for (int c = 0; c < 8; ++c) {
              const float4 q = *reinterpret_cast<const float4*>(x128 + ((16u * c) ^ xm128));
              x[4 * c] = q.x;
              x[4 * c + 1] = q.y;
              x[4 * c + 2] = q.z;
              x[4 * c + 3] = q.w;
            }
  #pragma unroll
            for (int c = 0; c < 4; ++c) {
              const float4 q = *reinterpret_cast<const float4*>(x64 + ((16u * c) ^ xm64));
              x[32 + 4 * c] = q.x;
              x[32 + 4 * c + 1] = q.y;
              x[32 + 4 * c + 2] = q.z;
              x[32 + 4 * c + 3] = q.w;
            }
            // XP[q] = (X[k], X[k + 1]), k = K0 + 2q, with X[n] = x[n - 1 + half] on
            // [0, 49) and 0 elsewhere (half 1's copy of the row is shifted by one).
            using P = BwdPairs<K>;
            auto xz = [&](int n) { return (n >= 0 && n < L) ? x[n] : 0.f; };  // compile-time n
            uint64_t XP[P::NQ];
  #pragma unroll
            for (int q = 0; q < P::NQ; ++q) {
              const int k = P::K0 + 2 * q;
              const float e0 = (k >= 0 && k <= L) ? (half ? xz(k) : xz(k - 1)) : 0.f;
              const float e1 = (k + 1 >= 0 && k + 1 <= L) ? (half ? xz(k + 1) : xz(k)) : 0.f;
              XP[q] = bwd_pack(e0, e1);
            }
            bwd_dk_row2<K>(dy128, dy64, xm128, xm64, XP, acc);
          }
          // The stage is read: order the reads before the next TMA write, release it.
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(sfree(s));
        }
      }
      if (i >= n_it) break;
      // A channel switch (helpers only): flush this channel's dK, then, once the
      // MMAs of the segment's last tile -- and so every earlier one -- are done
      // with the old Toeplitz operand, build the next channel's and signal the
      // MMA issuer.
      const int sl = (i - 1) % BWD_STAGES;
      if (ok) {
        flush(seg);
        ok = mbar_wait_bounded(mfree(sl), ((i - 1) / BWD_STAGES) & 1, err, DEVERR_TC_CONVERT);
      }
      if (named_barrier_or(2, BWD_ROWS, !ok)) ok = false;
      if (ok) {
        bwd_build_toeplitz<K>(sm + BG::OFF_B, taps, bwd_tile(sc, g, i).ch, ct, BWD_ROWS);
        fence_proxy_async_smem();
      }
      if (named_barrier_or(2, BWD_ROWS, !ok)) ok = false;
      if (ok && ct == 0) mbar_arrive(tready);
      ++seg;
    }
    // ---------------- dK of the last (or only) segment ----------------
    if (!named_barrier_or(2, BWD_ROWS, !ok)) {
      flush(seg);
      if (sc.direct) {
        named_barrier(2, BWD_ROWS);
        const float* red = reinterpret_cast<const float*>(sm + BG::OFF_RED);
        const int h = first.ch;
        float sum = 0.f;
        if (ct < K) sum = ((red[ct] + red[L + ct]) + red[2 * L + ct]) + red[3 * L + ct];
        // Data-parallel step: the channel's dK summed over the ranks right here.
        bool write = true;
        if (pa.world > 1) {
          const PeerSum r = peer_sum_row(pa, h, ct, BWD_ROWS, 2, sum, err);
          write = r.ok;
          sum = r.sum;
        }
        if (write && ct < K) {
          float* dst = dk + static_cast<size_t>(h) * K + ct;
          *dst = accumulate ? *dst + sum : sum;
        }
      }
    }
  } else {
    setmaxnreg_dec<BWD_REG_EPI>();
    // ---------------- dX epilogue ----------------
    const int et = static_cast<int>(threadIdx.x) - BWD_EPI0;  // 0..127
    const int quad = warp & 3;
    const int r = 32 * quad + lane;
    for (int j = 0; j < n_it; ++j) {
      const int d = j % ACC_SLOTS, o = j % OUT_SLOTS;
      if (et == 0) bulk_wait_read<OUT_SLOTS - 1>();
      const bool okw = mbar_wait_bounded(mdone(d), (j / ACC_SLOTS) & 1, err, DEVERR_TC_EPILOGUE);
      if (named_barrier_or(1, 128, !okw)) break;
      tc_fence_after();
      // The whole accumulator row in registers, then release the accumulator
      // to the MMAs before the sums and the staging stores.
      float accd[2 * N];
      const uint32_t ta = tmem + (static_cast<uint32_t>(32 * quad) << 16) +
                          static_cast<uint32_t>(D_COL0 + d * D_SLOT_COLS);
#pragma unroll
      for (int u = 0; u < 2 * N / 16; ++u) tmem_ld16(ta + 16u * u, accd + 16 * u);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accfree(d));
      unsigned char* ob = sm + BG::OFF_OUT + o * BG::TILE;
      // D[:, t] + D[:, N + t]
#pragma unroll
      for (int c = 0; c < GG::C128 + GG::C64; ++c) {
        const float4 y = make_float4(accd[4 * c] + accd[N + 4 * c], accd[4 * c + 1] + accd[N + 4 * c + 1],
                                     accd[4 * c + 2] + accd[N + 4 * c + 2],
                                     accd[4 * c + 3] + accd[N + 4 * c + 3]);
        const uint32_t off = (c < GG::C128) ? sw128_off(r, c) : GG::BOX64 + sw64_off(r, c - GG::C128);
        *reinterpret_cast<float4*>(ob + off) = y;
      }
      fence_proxy_async_smem();
      named_barrier(1, 128);
      if (et == 0) {
        const BwdTile t = bwd_tile(sc, g, j);
        const uint32_t os = base + static_cast<uint32_t>(BG::OFF_OUT + o * BG::TILE);
        tma_store_3d(&tm_dx128, os, 0, t.ch, t.blk * M);
        tma_store_3d(&tm_dx64, os + GG::BOX64, GG::S64, t.ch, t.blk * M);
        bulk_commit();
      }
    }
    if (et == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// dk[h][j] (=, or += when accumulate) the channel's partials in a fixed order:
// its kp primaries' four quadrants, then its helper segment's four.
template <int DUMMY = 0>
__global__ void __launch_bounds__(256) bwd_dk_reduce_kernel(const float* __restrict__ part, float* __restrict__ dk,
                                                            const BwdSched sc, int K, int accumulate) {
  const int idx = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (idx >= sc.H * K) return;
  const int h = idx / K;
  const int j = idx - h * K;
  float sum = 0.f;
  for (int r = 0; r < sc.kp; ++r) {
    const float* p = part + static_cast<size_t>(h + r * sc.H) * 4 * K + j;
    sum += ((p[0] + p[K]) + p[2 * K]) + p[3 * K];
  }
  if (sc.E > 0) {
    const int slot = sc.kp * sc.H + (h % sc.E) * sc.m + h / sc.E;
    const float* p = part + static_cast<size_t>(slot) * 4 * K + j;
    sum += ((p[0] + p[K]) + p[2 * K]) + p[3 * K];
  }
  dk[idx] = accumulate ? dk[idx] + sum : sum;
}

}  // namespace tc
}  // namespace pt
