// pt_tc_bwd.cuh -- fused backward: dX on the tensor cores and dK on the CUDA
// cores, in one pass over dy and x (rows of up to 48 columns).
//
// Separately, dX reads dy and writes dx, and dK reads dy and x: four [B, H, L]
// streams.  Here one kernel reads dy and x once and writes dx (three streams),
// and the two halves of the work use different pipes: the dX product runs as
// in tc_conv_kernel<DX> (3xTF32 split, Toeplitz operand resident in shared
// memory), while row threads split dy for it and accumulate the filter
// gradient of their rows with packed FFMAs.
//
// Tiles are 128 batch rows of one channel; CTAs are dealt tiles round-robin
// and the host uses this kernel only where every CTA keeps a single channel
// (a grid that is a multiple of H), so each thread's dK accumulators belong to
// one channel for the whole kernel.  At the end the CTA sums its threads'
// accumulators in a fixed order and writes one partial per (CTA, tap): with
// one CTA per channel that partial is the channel's dK.
//
// Roles (512 threads = four warpgroups, one CTA per SM):
//   warpgroup 0  warp 0: TMA producer (dy ring of 4 tiles, x ring of 3);
//                warp 1: allocates 512 TMEM columns, lane 0 issues the dX MMAs;
//                warps 2-3: no role after the set-up
//   warpgroups 1, 2  row workers, one thread per tile row; warpgroup 1 takes
//                the CTA's even tiles and warpgroup 2 the odd ones, so while
//                one group writes dy's sub-tf32 remainder (A of dX) into
//                tensor memory and loads its x rows, the other runs its FMA
//                nest on the same SM sub-partitions; each thread accumulates
//                every tap of its rows
//   warpgroup 3  dX epilogue: TMEM -> staging -> TMA store
// The row workers need about 170 registers (every tap's accumulator and the
// x row as packed pairs); the others need few, so after the set-up the CTA's
// 512 x 128 registers are rebalanced with setmaxnreg (warpgroup 0: 56, row
// workers: 184, epilogue: 88; none of the three regions spills).  The host
// launches the kernel only where the compiled function starts with 128
// registers per thread, the split's budget.
// Every wait is bounded; on expiry the kernel records a bit in the device
// error word, drains its own copies and MMAs, frees its tensor memory and
// returns without writing dK.
#pragma once

#include "pt_tc_kernels.cuh"

namespace pt {
namespace tc {

constexpr int BWD_L = 48;
constexpr int BWD_DY_SLOTS = 4;   // dy ring: read by the row workers and, as A_hi, by the MMAs
constexpr int BWD_X_SLOTS = 3;    // x ring: read once per tile by the row workers
constexpr int BWD_THREADS = 512;
constexpr int BWD_ROW0 = 128;     // first row-worker thread (warp 4)
constexpr int BWD_ROWS = 256;     // row workers: two groups of 128
constexpr int BWD_EPI0 = 384;     // first epilogue thread (warp 12)
constexpr int BWD_LAUNCH_REGS = 128;  // registers per thread at launch (65,536 / 512)
constexpr int BWD_REG_CTRL = 56;
constexpr int BWD_REG_ROWS = 184;
constexpr int BWD_REG_EPI = 88;
static_assert(128 * BWD_REG_CTRL + BWD_ROWS * BWD_REG_ROWS + 128 * BWD_REG_EPI <= BWD_THREADS * BWD_LAUNCH_REGS,
              "the register split must fit the registers the CTA is launched with");

struct BwdGeo {
  using GG = Geo<3>;                                  // 48-column tiles: 128-B + 64-B boxes
  static constexpr int N = GG::N;                     // 48
  static constexpr int TILE = GG::TILE;               // 24 KB
  static constexpr int OFF_DY = 0;
  static constexpr int OFF_X = OFF_DY + BWD_DY_SLOTS * TILE;
  static constexpr int OFF_OUT = OFF_X + BWD_X_SLOTS * TILE;  // one staging tile for the dx store
  static constexpr int OFF_B = OFF_OUT + TILE;
  static constexpr int OFF_BAR = OFF_B + GG::BMAT;    // one resident Toeplitz operand
  // fullD, dfree, mfree per dy slot; fullX, xfree per x slot; aready, adone per A
  // slot; mdone, accfree per accumulator.
  static constexpr int N_BARS = 3 * BWD_DY_SLOTS + 2 * BWD_X_SLOTS + 2 * A_SLOTS + 2 * ACC_SLOTS;
  static constexpr int OFF_TMEM = OFF_BAR + N_BARS * 8;
  static constexpr int SMEM = OFF_TMEM + 16 + 1024;
  static_assert(TILE % 1024 == 0 && OFF_B % 1024 == 0, "swizzled buffers start on 1024-byte boundaries");
  static_assert(BWD_L * BWD_ROWS * 4 <= BWD_DY_SLOTS * TILE, "dK reduction scratch fits the idle dy ring");
};

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

template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(N));
}

// dy - (dy with its low 13 mantissa bits cleared): the part of dy a tf32 MMA,
// which ignores those bits, does not see.  Exact in fp32.
__device__ __forceinline__ float bwd_tf32_rest(float v) {
  return v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
}

// Packed FP32 pairs: fma.rn.f32x2 does two FMAs in one issue slot (same FMA
// pipe throughput as two FFMAs, half the instructions).
__device__ __forceinline__ uint64_t bwd_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void bwd_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t bwd_ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// Filter gradient of one row, every tap, taps in pairs:
//   (acc[2p], acc[2p+1]) += (dy[t], dy[t]) * (x[i], x[i+1]),  i = t + 2p - K/2,
// with XP[i + 1] = (x[i], x[i + 1]) for i in [-1, 48) (x outside [0, 48) is 0),
// packed once per tile, and dy[t] broadcast into both halves.  For odd K the
// last tap (K - 1) has its own scalar accumulator.  dy arrives four columns at
// a time as 16-byte chunks of the swizzled row (one conflict-free LDS.128).
template <int K>
struct BwdTaps {
  static constexpr int PAD = K / 2;
  static constexpr int NP = K / 2;           // full tap pairs
  static constexpr bool ODD = (K % 2) != 0;  // tap K - 1 on its own
  static constexpr int NACC = NP > 0 ? NP : 1;
};

template <int K>
__device__ __forceinline__ void bwd_dk_row(const unsigned char* dyrow128, const unsigned char* dyrow64,
                                           uint32_t xm128, uint32_t xm64, const uint64_t (&XP)[BWD_L + 1],
                                           uint64_t (&acc)[BwdTaps<K>::NACC], float& acc_odd) {
  using T = BwdTaps<K>;
#pragma unroll
  for (int c = 0; c < BWD_L / 4; ++c) {
    bool any = false;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
#pragma unroll
      for (int p = 0; p < T::NP; ++p) {
        const int i = 4 * c + u + 2 * p - T::PAD;
        any = any || (i >= -1 && i < BWD_L);
      }
      if (T::ODD) {
        const int i1 = 4 * c + u + (K - 1) - T::PAD;
        any = any || (i1 >= 0 && i1 < BWD_L);
      }
    }
    if (!any) continue;
    const float4 q = (c < 8) ? *reinterpret_cast<const float4*>(dyrow128 + ((16u * c) ^ xm128))
                             : *reinterpret_cast<const float4*>(dyrow64 + ((16u * (c - 8)) ^ xm64));
    const float d[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = 4 * c + u;
      const uint64_t d2 = bwd_pack(d[u], d[u]);
#pragma unroll
      for (int p = 0; p < T::NP; ++p) {
        const int i = t + 2 * p - T::PAD;
        if (i >= -1 && i < BWD_L) acc[p] = bwd_ffma2(d2, XP[i + 1], acc[p]);
      }
      if (T::ODD) {
        const int i1 = t + (K - 1) - T::PAD;
        if (i1 >= 0 && i1 < BWD_L) {
          float lo, hi;
          bwd_unpack(XP[i1 + 1], lo, hi);
          acc_odd = fmaf(d[u], lo, acc_odd);
        }
      }
    }
  }
}

// n_tiles = ceil(B / 128) * H; tile tau: channel tau % H, rows [128 * (tau / H), +128).
// Requires gridDim.x % H == 0 (each CTA keeps channel blockIdx.x % H).
// dk_out: partial[(g * 2) * K + j] with group_of[2g] = channel, group_of[2g + 1] = -1
// (the tensor-core dK reduce layout), or, if direct != 0, dk[h * K + j] (=, or += when
// accumulate != 0) -- valid when each channel has exactly one CTA.
template <int K>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    tc_bwd_kernel(const __grid_constant__ CUtensorMap tm_dy128, const __grid_constant__ CUtensorMap tm_dy64,
                  const __grid_constant__ CUtensorMap tm_x128, const __grid_constant__ CUtensorMap tm_x64,
                  const __grid_constant__ CUtensorMap tm_dx128, const __grid_constant__ CUtensorMap tm_dx64,
                  const float* __restrict__ taps, float* __restrict__ dk_out, int* __restrict__ group_of,
                  int H, int n_tiles, int direct, int accumulate, unsigned* err) {
  using GG = Geo<3>;
  using BG = BwdGeo;
  using TP = BwdTaps<K>;
  constexpr int N = GG::N;
  constexpr int L = BWD_L;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = aligned_smem(smem_raw);
  const uint32_t base = smem_u32(sm);
  const int warp = static_cast<int>(threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31);
  const uint32_t bar0 = base + BG::OFF_BAR;
  constexpr int DS = BWD_DY_SLOTS, XS = BWD_X_SLOTS;
  auto fullD = [&](int s) { return bar0 + 8u * s; };                       // dy tile landed
  auto dfree = [&](int s) { return bar0 + 8u * (DS + s); };                // row workers done with dy
  auto mfree = [&](int s) { return bar0 + 8u * (2 * DS + s); };            // dX MMAs done with dy
  auto fullX = [&](int s) { return bar0 + 8u * (3 * DS + s); };            // x tile landed
  auto xfree = [&](int s) { return bar0 + 8u * (3 * DS + XS + s); };       // x rows taken
  constexpr int B2 = 3 * DS + 2 * XS;
  auto aready = [&](int a) { return bar0 + 8u * (B2 + a); };
  auto adone = [&](int a) { return bar0 + 8u * (B2 + A_SLOTS + a); };
  auto mdone = [&](int d) { return bar0 + 8u * (B2 + 2 * A_SLOTS + d); };
  auto accfree = [&](int d) { return bar0 + 8u * (B2 + 2 * A_SLOTS + ACC_SLOTS + d); };
  const int G = static_cast<int>(gridDim.x);
  const int g = static_cast<int>(blockIdx.x);
  const int h = g % H;  // the CTA's channel (G % H == 0)
  const int n_it = (g < n_tiles) ? (n_tiles - 1 - g) / G + 1 : 0;

  // Partials mode: mark this CTA's slots unused before any bounded wait, so a
  // CTA that gives up after a timed-out wait adds nothing to the reduce (and no
  // slot id left in the workspace by an earlier launch is read).
  if (!direct && threadIdx.x == 0) {
    group_of[2 * g] = -1;
    group_of[2 * g + 1] = -1;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < DS; ++s) {
      mbar_init(fullD(s), 1);
      mbar_init(dfree(s), 4);  // the four warps of the group that took the tile
      mbar_init(mfree(s), 1);
    }
    for (int s = 0; s < XS; ++s) {
      mbar_init(fullX(s), 1);
      mbar_init(xfree(s), 4);
    }
    for (int a = 0; a < A_SLOTS; ++a) {
      mbar_init(aready(a), 4);
      mbar_init(adone(a), 1);
    }
    for (int d = 0; d < ACC_SLOTS; ++d) {
      mbar_init(mdone(d), 1);
      mbar_init(accfree(d), 4);
    }
    fence_mbar_init();
  }
  // The channel's Toeplitz operand for dX, T[s][t] = k[t - s + K/2], built once
  // by the whole CTA (every tile of this CTA has channel h).
  {
    const int pad = K / 2;
    unsigned char* bm = sm + BG::OFF_B;
    const float* kh = taps + static_cast<size_t>(h) * K;
    constexpr int CPR = N / 4;
    for (int task = static_cast<int>(threadIdx.x); task < N * CPR; task += BWD_THREADS) {
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
    fence_proxy_async_smem();  // the MMAs read the operand through the async proxy
  }
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
        const int sd = i % DS, sx = i % XS;
        if (i >= DS && (!mbar_wait_bounded(dfree(sd), ((i / DS) - 1) & 1, err, DEVERR_TIMEOUT_DONE) ||
                        !mbar_wait_bounded(mfree(sd), ((i / DS) - 1) & 1, err, DEVERR_TIMEOUT_DONE)))
          break;
        if (i >= XS && !mbar_wait_bounded(xfree(sx), ((i / XS) - 1) & 1, err, DEVERR_TIMEOUT_DONE)) break;
        const int b0 = ((g + i * G) / H) * M;
        const uint32_t dst = base + static_cast<uint32_t>(BG::OFF_DY + sd * BG::TILE);
        const uint32_t xst = base + static_cast<uint32_t>(BG::OFF_X + sx * BG::TILE);
        mbar_arrive_expect_tx(fullD(sd), BG::TILE);
        tma_load_3d(dst, &tm_dy128, 0, h, b0, fullD(sd));
        tma_load_3d(dst + GG::BOX64, &tm_dy64, GG::S64, h, b0, fullD(sd));
        mbar_arrive_expect_tx(fullX(sx), BG::TILE);
        tma_load_3d(xst, &tm_x128, 0, h, b0, fullX(sx));
        tma_load_3d(xst + GG::BOX64, &tm_x64, GG::S64, h, b0, fullX(sx));
        issued = i + 1;
      }
      for (int i = issued > DS ? issued - DS : 0; i < issued; ++i)
        if (!mbar_wait_bounded(fullD(i % DS), (i / DS) & 1, err, DEVERR_TIMEOUT_DRAIN)) break;
      for (int i = issued > XS ? issued - XS : 0; i < issued; ++i)
        if (!mbar_wait_bounded(fullX(i % XS), (i / XS) & 1, err, DEVERR_TIMEOUT_DRAIN)) break;
    } else if (warp == 1 && lane == 0) {
      // ---------------- MMA issuer (dX) ----------------
      constexpr uint32_t idesc_n2 = idesc_tf32_m128<2 * N>();
      constexpr uint32_t idesc_n = idesc_tf32_m128<N>();
      int issued = 0;
      for (int i = 0; i < n_it; ++i) {
        const int a = i % A_SLOTS, d = i % ACC_SLOTS, sd = i % DS;
        // The dy tile is the A_hi operand: wait for its load as well.
        if (!mbar_wait_bounded(fullD(sd), (i / DS) & 1, err, DEVERR_TC_MMA)) break;
        if (!mbar_wait_bounded(aready(a), (i / A_SLOTS) & 1, err, DEVERR_TC_MMA)) break;
        if (i >= ACC_SLOTS &&
            !mbar_wait_bounded(accfree(d), ((i / ACC_SLOTS) - 1) & 1, err, DEVERR_TC_MMA))
          break;
        tc_fence_after();
        const uint32_t a_lo = tmem + static_cast<uint32_t>(A_COL0 + a * A_SLOT_COLS + LO_COLS);
        const uint32_t dyt = base + static_cast<uint32_t>(BG::OFF_DY + sd * BG::TILE);
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
        mma_commit(mfree(sd));
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
    bool ok = true;
    const int ct = static_cast<int>(threadIdx.x) - BWD_ROW0;  // 0..255
    const int grp = ct >> 7;                                   // 0: even tiles, 1: odd tiles
    const int quad = warp & 3;
    const int row = 32 * quad + lane;                          // tile row (TMEM lane)
    const uint32_t lane_base = static_cast<uint32_t>(32 * quad) << 16;
    // In-row byte offset of 16-byte chunk c of this row: (16 c) ^ xm128 in the
    // 128-B box (chunks 0-7), (16 c) ^ xm64 in the 64-B box (chunks 0-3).
    const uint32_t xm128 = static_cast<uint32_t>(row & 7) << 4;
    const uint32_t xm64 = static_cast<uint32_t>((row >> 1) & 3) << 4;
    uint64_t acc[TP::NACC];
#pragma unroll
    for (int p = 0; p < TP::NACC; ++p) acc[p] = 0ull;
    float acc_odd = 0.f;
    for (int i = grp; i < n_it; i += 2) {
      const int sd = i % DS, sx = i % XS, a = i % A_SLOTS;  // a == grp
      if (i >= A_SLOTS) ok = mbar_wait_bounded(adone(a), ((i / A_SLOTS) - 1) & 1, err, DEVERR_TC_CONVERT);
      if (ok) ok = mbar_wait_bounded(fullD(sd), (i / DS) & 1, err, DEVERR_TIMEOUT_FULL);
      if (!__all_sync(0xffffffffu, ok)) {  // each warp arrives as one, so it decides as one
        ok = false;
        break;
      }
      const unsigned char* dy128 = sm + BG::OFF_DY + sd * BG::TILE + 128u * row;
      const unsigned char* dy64 = sm + BG::OFF_DY + sd * BG::TILE + GG::BOX64 + 64u * row;
      // dX: the MMA reads dy's tf32 part straight from the stage; this thread
      // writes the rest of its dy row (A_lo) into tensor memory.
      {
        const uint32_t acol = tmem + lane_base + static_cast<uint32_t>(A_COL0 + a * A_SLOT_COLS + LO_COLS);
#pragma unroll
        for (int u = 0; u < L / 8; ++u) {
          float lo[8];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int c = 2 * u + hh;
            const float4 q = (c < 8) ? *reinterpret_cast<const float4*>(dy128 + ((16u * c) ^ xm128))
                                     : *reinterpret_cast<const float4*>(dy64 + ((16u * (c - 8)) ^ xm64));
            lo[4 * hh] = bwd_tf32_rest(q.x);
            lo[4 * hh + 1] = bwd_tf32_rest(q.y);
            lo[4 * hh + 2] = bwd_tf32_rest(q.z);
            lo[4 * hh + 3] = bwd_tf32_rest(q.w);
          }
          tmem_st8(acol + 8u * u, lo);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(aready(a));
      }
      // dK: the x row as packed pairs in registers, dy streamed from shared memory.
      ok = mbar_wait_bounded(fullX(sx), (i / XS) & 1, err, DEVERR_TIMEOUT_FULL);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      uint64_t XP[L + 1];
      {
        const unsigned char* x128 = sm + BG::OFF_X + sx * BG::TILE + 128u * row;
        const unsigned char* x64 = sm + BG::OFF_X + sx * BG::TILE + GG::BOX64 + 64u * row;
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
        // The x rows are in registers: the x slot can be refilled.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(xfree(sx));
        auto xz = [&](int n) { return (n >= 0 && n < L) ? x[n] : 0.f; };  // compile-time n
#pragma unroll
        for (int q = 0; q <= L; ++q) XP[q] = bwd_pack(xz(q - 1), xz(q));
      }
      bwd_dk_row<K>(dy128, dy64, xm128, xm64, XP, acc, acc_odd);
      // The dy tile is read: order the reads before the next TMA write, release it.
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(dfree(sd));
    }
    // ---------------- dK: sum the CTA's rows in a fixed order ----------------
    // The scratch below overwrites the dy ring, which the last tiles' MMAs may
    // still read: wait for the last MMA group (groups complete in issue order).
    if (ok && n_it > 0)
      ok = mbar_wait_bounded(mfree((n_it - 1) % DS), ((n_it - 1) / DS) & 1, err, DEVERR_TC_CONVERT);
    if (!named_barrier_or(2, BWD_ROWS, !ok)) {
      // Both groups are done with every tile and every load has been consumed:
      // reuse the dy ring as [K][256] scratch.
      float* red = reinterpret_cast<float*>(sm + BG::OFF_DY);
#pragma unroll
      for (int p = 0; p < TP::NP; ++p) {
        float lo, hi;
        bwd_unpack(acc[p], lo, hi);
        red[(2 * p) * BWD_ROWS + ct] = lo;
        red[(2 * p + 1) * BWD_ROWS + ct] = hi;
      }
      if (TP::ODD) red[(K - 1) * BWD_ROWS + ct] = acc_odd;
      named_barrier(2, BWD_ROWS);
      for (int j = ct; j < K; j += BWD_ROWS) {
        float sum = 0.f;
        for (int r = 0; r < BWD_ROWS; ++r) sum += red[j * BWD_ROWS + r];
        if (direct) {
          float* dst = dk_out + static_cast<size_t>(h) * K + j;
          *dst = accumulate ? *dst + sum : sum;
        } else {
          dk_out[static_cast<size_t>(g) * 2 * K + j] = sum;
        }
      }
      if (!direct && ct == 0) {
        group_of[2 * g] = h;
        group_of[2 * g + 1] = -1;
      }
    }
  } else {
    setmaxnreg_dec<BWD_REG_EPI>();
    // ---------------- dX epilogue ----------------
    const int et = static_cast<int>(threadIdx.x) - BWD_EPI0;  // 0..127
    const int quad = warp & 3;
    const int r = 32 * quad + lane;
    unsigned char* ob = sm + BG::OFF_OUT;
    const uint32_t os = base + static_cast<uint32_t>(BG::OFF_OUT);
    for (int j = 0; j < n_it; ++j) {
      const int d = j % ACC_SLOTS;
      if (et == 0) bulk_wait_read<0>();  // the previous store has read the staging tile
      const bool okw = mbar_wait_bounded(mdone(d), (j / ACC_SLOTS) & 1, err, DEVERR_TC_EPILOGUE);
      if (named_barrier_or(1, 128, !okw)) break;
      tc_fence_after();
      const uint32_t ta = tmem + (static_cast<uint32_t>(32 * quad) << 16) +
                          static_cast<uint32_t>(D_COL0 + d * D_SLOT_COLS);
#pragma unroll
      for (int cc = 0; cc < N / 16; ++cc) {
        float v0[16], v1[16];
        tmem_ld16(ta + 16u * cc, v0);
        tmem_ld16(ta + static_cast<uint32_t>(N) + 16u * cc, v1);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = 4 * cc + q;  // 16-byte chunk of the row
          const float4 y = make_float4(v0[4 * q] + v1[4 * q], v0[4 * q + 1] + v1[4 * q + 1],
                                       v0[4 * q + 2] + v1[4 * q + 2], v0[4 * q + 3] + v1[4 * q + 3]);
          const uint32_t off = (c < GG::C128) ? sw128_off(r, c) : GG::BOX64 + sw64_off(r, c - GG::C128);
          *reinterpret_cast<float4*>(ob + off) = y;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accfree(d));
      fence_proxy_async_smem();
      named_barrier(1, 128);
      if (et == 0) {
        const int b0 = ((g + j * G) / H) * M;
        tma_store_3d(&tm_dx128, os, 0, h, b0);
        tma_store_3d(&tm_dx64, os + GG::BOX64, GG::S64, h, b0);
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

}  // namespace tc
}  // namespace pt
