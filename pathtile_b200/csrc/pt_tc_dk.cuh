// pt_tc_dk.cuh -- filter gradient dK on the 5th-generation tensor cores (tcgen05).
//
// For one channel, dK is a diagonal sum of a small correlation matrix:
//   C[t][s] = sum_b dy[b][t] x[b][s]            (an L x L GEMM over the batch)
//   dk[j]   = sum_t C[t][t + j - K/2]           (0 <= t, t + j - K/2 < L)
// A tile is 64 batch rows (the MMA's K extent) of a super-row of W columns
// (one channel, or 48 / L packed channels as in the FWD/DX kernels; the
// correlation of a packed super-row is W x W and channel c uses its diagonal
// block).  Accumulators stay in tensor memory across all tiles a CTA visits
// of a channel group, so the per-tile work is: TMA the dy and x tiles, split,
// MMA; the diagonal sums run once per CTA at the end.
//
// FP32 accuracy with TF32 MMAs: the MMA reads a TF32 operand from an FP32
// word by ignoring its low 13 mantissa bits, so v = hi + lo with hi = v as
// stored (read as trunc(v)) and lo = v - trunc(v) (exact in FP32, read as
// trunc(lo)); the split costs two instructions per value and no store for
// hi.  A (in tensor memory, lane = row) holds the dy columns: lanes 0..63 =
// dy_hi column t = lane, lanes 64..127 = dy_lo column t = lane - 64; B
// (shared memory, MN-major) holds [x_hi | x_lo] along N.  One M = 128 MMA per
// 8 batch rows then yields all four products, and C[t][s] = D[t][hi(s)] +
// D[t][lo(s)] + D[64+t][hi(s)] + D[64+t][lo(s)] (the lo*lo term is kept).
// Per product the error is below about 2^-19 of |dy x| (the truncation of lo),
// far inside the 1e-4 relative bar of dK.
//
// B comes straight from TMA: MN-major tf32 operands need the 128-byte
// swizzle with 32-byte atoms (4 batch rows of 128 bytes per atom), which the
// TMA writes with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B; x is loaded as one or
// two boxes of 32 columns (x_hi), and x_lo goes to the same offsets one block
// row further, so the four (or two) 32-column blocks sit at a uniform stride
// (the descriptor's leading offset).  The dy tile is
// only read by the converters (128-B and 64-B swizzled boxes as in FWD/DX).
//
// Roles (320 threads, one CTA per SM):
//   warp 0      TMA producer (dy and x tiles, ring of 5 stages)
//   warp 1      allocates 512 TMEM columns (3 A slots of 64 columns, 2 accumulators
//               of 128); lane 0 issues the MMAs and commits them
//   warps 2-5   A converters, one per TMEM lane quadrant: each lane reads one dy
//               column of the tile and writes it (hi rows) or its lo part (lo rows)
//               as 64 TMEM columns
//   warps 6-9   B converters: write x_lo beside the x tile (x_hi is the tile itself)
//   then warps 2-9 run the epilogue: accumulators -> shared memory -> diagonal
//   sums -> one partial per (CTA, group, channel, tap), or float atomics.
// The channel groups a CTA visits must be resident (period 1 or 2); the host
// runs other shapes on the FFMA kernels.  Waits are bounded as in every kernel
// of this library.
#pragma once

#include "pt_tc_kernels.cuh"

namespace pt {
namespace tc {

constexpr int DK_ROWS = 64;        // batch rows per tile (MMA K per tile)
constexpr int DK_STAGES = 5;
constexpr int DK_A_SLOTS = 3;
constexpr int DK_A_COLS = 64;      // one A slot: 64 TMEM columns (one per batch row)
constexpr int DK_D_COL0 = 256;     // accumulators at columns 256 and 384
constexpr int DK_D_COLS = 128;
constexpr int DK_THREADS = 64 + 256;
constexpr int DK_MAX_GROUPS = 2;   // resident accumulators per CTA

template <int LB>
struct DkGeo {
  static constexpr int RB128 = (LB >= 2) ? 128 : 0;  // dy tile: 128-B swizzled box (columns 0..31)
  static constexpr int RB64 = (LB & 1) ? 64 : 0;     //          64-B swizzled box (32..47 or 0..15)
  static constexpr int S64 = (LB >= 2) ? 32 : 0;     // first column of the 64-B box
  static constexpr int W = 16 * LB;                  // super-row width
  static constexpr int NB = (W > 32) ? 2 : 1;        // 32-column x boxes
  static constexpr int N = 64 * NB;                  // MMA N: x_hi blocks then x_lo blocks
  static constexpr int DY_TILE = DK_ROWS * (RB128 + RB64);
  static constexpr int DY_BOX64 = DK_ROWS * RB128;
  static constexpr int XBLOCK = DK_ROWS * 128;       // one 32-column x block (8 KB)
  static constexpr int OFF_X = DY_TILE;              // x_hi blocks, then x_lo blocks
  static constexpr int XLO = NB * XBLOCK;            // x_hi -> x_lo offset
  static constexpr int STAGE = DY_TILE + 2 * NB * XBLOCK;
  static constexpr int OFF_BAR = DK_STAGES * STAGE;
  static constexpr int N_BARS = 3 * DK_STAGES + DK_A_SLOTS + 1;  // full, conv, sfree | afree | dfin
  static constexpr int OFF_TMEM = OFF_BAR + N_BARS * 8;
  static constexpr int SMEM = OFF_TMEM + 16 + 1024;
  static_assert(DY_TILE % 1024 == 0 && DY_BOX64 % 1024 == 0 && STAGE % 1024 == 0,
                "swizzled tiles start on 1024-byte boundaries");
  static_assert(2 * 64 * W * 4 <= DK_STAGES * STAGE, "epilogue scratch fits the idle ring");
};

// Shared-memory descriptor of an MN-major tf32 operand in the 128-byte swizzle
// with 32-byte atoms (layout type 1): start >> 4, stride between 32-column N
// blocks >> 4 (leading-offset field), stride between 4-row K groups (512 B)
// >> 4, version 1.
__device__ __forceinline__ uint64_t mn32b_desc(uint32_t addr, uint32_t nblock_stride) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((nblock_stride >> 4) & 0x3FFFu) << 16) | (static_cast<uint64_t>(512 >> 4) << 32) |
         (1ull << 46) | (1ull << 61);
}

// Instruction descriptor: D f32, A and B tf32, A K-major (tensor memory), B
// MN-major (bit 16), N >> 3, M = 128.
template <int N>
constexpr uint32_t idesc_tf32_m128_bmn() {
  return (1u << 4) | (2u << 7) | (2u << 10) | (1u << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(128 >> 4) << 24);
}

// lo part of v in the truncation split: v - (v with its low 13 mantissa bits cleared).
__device__ __forceinline__ float tf32_trunc_lo(float v) {
  return v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
}

// n_tiles = ceil(B / 64) * Hg; tile tau: group tau % Hg, batch rows [64 * (tau / Hg), +64).
// CTA g takes tiles g, g + G, ...; bperiod (1 or 2) = groups it visits.
// tm_dy128 / tm_dy64: the dy boxes of the FWD/DX layout (32 and 16 columns,
// 64 rows); tm_x32b: 32-column x boxes, 64 rows, 128-B swizzle with 32-B atoms.
// Output: atomic != 0: dk[(grp*Hc + c)*K + j] += partial; else partial[(g*2 + slot)*Hc*K + c*K + j]
// and group_of[g*2 + slot] (-1 for an unused slot).
template <int LB, bool PACKED>
__global__ void __launch_bounds__(DK_THREADS, 1)
    tc_dk_kernel(const __grid_constant__ CUtensorMap tm_dy128, const __grid_constant__ CUtensorMap tm_dy64,
                 const __grid_constant__ CUtensorMap tm_x32b, float* __restrict__ out,
                 int* __restrict__ group_of, int H, int L, int K, int Hc, int Hg, int n_tiles, int bperiod,
                 int atomic, unsigned* err) {
  using GG = DkGeo<LB>;
  constexpr int W = GG::W;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = aligned_smem(smem_raw);
  const uint32_t base = smem_u32(sm);
  const int warp = static_cast<int>(threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31);
  const uint32_t bar0 = base + GG::OFF_BAR;
  // full (TMA landed), conv (tile converted: A slot written, x split), sfree
  // (MMAs of the stage done), afree (MMAs reading the A slot done), dfin (all MMAs done).
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto conv = [&](int s) { return bar0 + 8u * (DK_STAGES + s); };
  auto sfree = [&](int s) { return bar0 + 8u * (2 * DK_STAGES + s); };
  auto afree = [&](int a) { return bar0 + 8u * (3 * DK_STAGES + a); };
  const uint32_t dfin = bar0 + 8u * (3 * DK_STAGES + DK_A_SLOTS);
  const int G = static_cast<int>(gridDim.x);
  const int g = static_cast<int>(blockIdx.x);
  const int n_it = (g < n_tiles) ? (n_tiles - 1 - g) / G + 1 : 0;
  const int Wp = Hc * L;  // packed super-row width (PACKED only)

  // Mark this CTA's partial slots unused before any bounded wait: a CTA that
  // gives up after a timed-out wait then contributes nothing to the reduce,
  // never a slot id left behind by an earlier launch in the same workspace.
  if (!atomic && threadIdx.x == 0)
    for (int slot = 0; slot < DK_MAX_GROUPS; ++slot) group_of[g * DK_MAX_GROUPS + slot] = -1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < DK_STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(conv(s), 8);  // one arrival per converter warp
      mbar_init(sfree(s), 1);
    }
    for (int a = 0; a < DK_A_SLOTS; ++a) mbar_init(afree(a), 1);
    mbar_init(dfin, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(base + GG::OFF_TMEM, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + GG::OFF_TMEM);
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < n_it; ++i) {
        const int s = i % DK_STAGES;
        if (i >= DK_STAGES &&
            !mbar_wait_bounded(sfree(s), ((i / DK_STAGES) - 1) & 1, err, DEVERR_TIMEOUT_DONE))
          break;
        const int tau = g + i * G;
        const int grp = tau % Hg;
        const int b0 = (tau / Hg) * DK_ROWS;
        const uint32_t st = base + static_cast<uint32_t>(s * GG::STAGE);
        mbar_arrive_expect_tx(full(s), GG::DY_TILE + GG::NB * GG::XBLOCK);
        if constexpr (PACKED) {
          if constexpr (LB >= 2) tma_load_2d(st, &tm_dy128, grp * Wp, b0, full(s));
          if constexpr (LB & 1) tma_load_2d(st + GG::DY_BOX64, &tm_dy64, grp * Wp + GG::S64, b0, full(s));
#pragma unroll
          for (int q = 0; q < GG::NB; ++q)
            tma_load_2d(st + GG::OFF_X + q * GG::XBLOCK, &tm_x32b, grp * Wp + 32 * q, b0, full(s));
        } else {
          if constexpr (LB >= 2) tma_load_3d(st, &tm_dy128, 0, grp, b0, full(s));
          if constexpr (LB & 1) tma_load_3d(st + GG::DY_BOX64, &tm_dy64, GG::S64, grp, b0, full(s));
#pragma unroll
          for (int q = 0; q < GG::NB; ++q)
            tma_load_3d(st + GG::OFF_X + q * GG::XBLOCK, &tm_x32b, 32 * q, grp, b0, full(s));
        }
        issued = i + 1;
      }
      for (int i = issued > DK_STAGES ? issued - DK_STAGES : 0; i < issued; ++i)
        if (!mbar_wait_bounded(full(i % DK_STAGES), (i / DK_STAGES) & 1, err, DEVERR_TIMEOUT_DRAIN))
          break;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32_m128_bmn<GG::N>();
      for (int i = 0; i < n_it; ++i) {
        const int s = i % DK_STAGES, a = i % DK_A_SLOTS, d = i % bperiod;
        if (!mbar_wait_bounded(conv(s), (i / DK_STAGES) & 1, err, DEVERR_TC_MMA)) break;
        tc_fence_after();
        const bool first = i < bperiod;  // first tile of this accumulator
        const uint32_t a_t = tmem + static_cast<uint32_t>(a * DK_A_COLS);
        const uint32_t d_t = tmem + static_cast<uint32_t>(DK_D_COL0 + d * DK_D_COLS);
        const uint32_t xh = base + static_cast<uint32_t>(s * GG::STAGE + GG::OFF_X);
#pragma unroll
        for (int kk = 0; kk < DK_ROWS / 8; ++kk)  // 8 batch rows = 1024 B of every x block
          mma_tf32_ts(d_t, a_t + 8u * kk, mn32b_desc(xh + 1024u * kk, GG::XBLOCK), idesc,
                      (first && kk == 0) ? 0u : 1u);
        mma_commit(sfree(s));
        mma_commit(afree(a));
      }
      mma_commit(dfin);
      if (!mbar_wait_bounded(dfin, 0, err, DEVERR_TC_MMA)) ok = false;
    }
    __syncwarp();
  } else {
    const int ct = static_cast<int>(threadIdx.x) - 64;  // 0..255
    if (warp < 6) {
      // ---------------- A converters: dy column t -> TMEM row t (hi) or 64 + t (lo) ----------------
      const int quad = warp & 3;
      const int t = 32 * (quad & 1) + lane;  // dy column of this lane
      const bool lo_rows = quad >= 2;        // warp-uniform
      const uint32_t lane_base = static_cast<uint32_t>(32 * quad) << 16;
      for (int i = 0; i < n_it; ++i) {
        const int s = i % DK_STAGES, a = i % DK_A_SLOTS;
        if (i >= DK_A_SLOTS) ok = mbar_wait_bounded(afree(a), ((i / DK_A_SLOTS) - 1) & 1, err, DEVERR_TC_CONVERT);
        if (ok) ok = mbar_wait_bounded(full(s), (i / DK_STAGES) & 1, err, DEVERR_TIMEOUT_FULL);
        if (!__all_sync(0xffffffffu, ok)) {  // the warp leaves together (it arrives as one)
          ok = false;
          break;
        }
        // Every lane executes the (warp-collective) TMEM stores; columns past the
        // super-row width hold zeros and their accumulator rows are never read.
        // Row r of column t sits at r * pitch + base[r % 8] in its box: the
        // few bases are hoisted, so the 64 loads take immediate offsets.
        const unsigned char* dyt = sm + s * GG::STAGE;
        float v[DK_ROWS];
        if (LB >= 2 && (quad & 1) == 0) {  // columns 0..31: 128-B box
          uint32_t bse[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) bse[k] = sw128_off(k, t >> 2) - 128u * k + 4u * (t & 3);
#pragma unroll
          for (int r = 0; r < DK_ROWS; ++r)
            v[r] = *reinterpret_cast<const float*>(dyt + 128u * r + bse[r & 7]);
        } else {  // the 64-B box (columns 32..47, or 0..15 when W = 16)
          const int c = t - GG::S64;
          uint32_t bse[8];
#pragma unroll
          for (int k = 0; k < 8; ++k)
            bse[k] = GG::DY_BOX64 + sw64_off(k, (c >> 2) & 3) - 64u * k + 4u * (c & 3);
          const bool in = (t < W) && (LB & 1);
#pragma unroll
          for (int r = 0; r < DK_ROWS; ++r)
            v[r] = in ? *reinterpret_cast<const float*>(dyt + 64u * r + bse[r & 7]) : 0.f;
        }
        if (lo_rows) {
#pragma unroll
          for (int r = 0; r < DK_ROWS; ++r) v[r] = tf32_trunc_lo(v[r]);
        }
        const uint32_t acol = tmem + lane_base + static_cast<uint32_t>(a * DK_A_COLS);
#pragma unroll
        for (int u = 0; u < DK_ROWS / 8; ++u) tmem_st8(acol + 8u * u, v + 8 * u);
        tmem_wait_st();
        tc_fence_before();
        fence_proxy_async_smem();  // dy reads ordered before the stage's next TMA write
        __syncwarp();
        if (lane == 0) mbar_arrive(conv(s));
      }
    } else {
      // ---------------- B converters: x blocks (x_hi as loaded) -> x_lo ----------------
      // Element-wise, so the swizzled layout needs no decoding: consecutive
      // threads take consecutive 16-byte chunks (conflict-free).
      const int bt = ct - 128;  // 0..127
      for (int i = 0; i < n_it; ++i) {
        const int s = i % DK_STAGES;
        ok = mbar_wait_bounded(full(s), (i / DK_STAGES) & 1, err, DEVERR_TIMEOUT_FULL);
        if (!__all_sync(0xffffffffu, ok)) {  // the warp leaves together (it arrives as one)
          ok = false;
          break;
        }
        unsigned char* xt = sm + s * GG::STAGE + GG::OFF_X;
#pragma unroll 4
        for (int o = 16 * bt; o < GG::NB * GG::XBLOCK; o += 16 * 128) {
          const float4 v = *reinterpret_cast<const float4*>(xt + o);
          *reinterpret_cast<float4*>(xt + GG::XLO + o) =
              make_float4(tf32_trunc_lo(v.x), tf32_trunc_lo(v.y), tf32_trunc_lo(v.z), tf32_trunc_lo(v.w));
        }
        fence_proxy_async_smem();  // the MMAs read x_lo through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(conv(s));
      }
    }
    // ---------------- epilogue (warps 2-9) ----------------
    const bool fin = ok && mbar_wait_bounded(dfin, 0, err, DEVERR_TC_EPILOGUE);
    if (!named_barrier_or(2, 256, !fin)) {
      // The ring is idle: stage memory becomes [hi rows 0..63 | lo rows 64..127] x W.
      float* scratch = reinterpret_cast<float*>(sm);
      const int n_slots = n_it < bperiod ? n_it : bperiod;
      for (int slot = 0; slot < n_slots; ++slot) {
        if (warp < 6) {
          const int quad = warp & 3;
          const int lrow = 32 * quad + lane;  // accumulator row
          tc_fence_after();
          float dv[GG::N];
          const uint32_t ta = tmem + (static_cast<uint32_t>(32 * quad) << 16) +
                              static_cast<uint32_t>(DK_D_COL0 + slot * DK_D_COLS);
#pragma unroll
          for (int u = 0; u < GG::N / 16; ++u) tmem_ld16(ta + 16u * u, dv + 16 * u);
          tmem_wait_ld();
          // Row lrow times (x_hi part + x_lo part); hi and lo rows meet in the sums below.
          if ((lrow & 63) < W) {
#pragma unroll
            for (int s2 = 0; s2 < W; ++s2) scratch[lrow * W + s2] = dv[s2] + dv[GG::N / 2 + s2];
          }
        }
        named_barrier(2, 256);
        // Diagonal sums per (channel of the group, tap).
        const int grp = (g + slot * G) % Hg;
        for (int task = ct; task < Hc * K; task += 256) {
          const int c = task / K;
          const int j = task - c * K;
          const int ch = grp * Hc + c;
          const int off = c * L;  // block of channel c in the super-row
          float acc = 0.f;
          for (int tt = 0; tt < L; ++tt) {
            const int ss = tt + j - K / 2;
            if (ss >= 0 && ss < L) acc += scratch[(off + tt) * W + off + ss] + scratch[(64 + off + tt) * W + off + ss];
          }
          if (atomic) {
            if (ch < H) atomicAdd(out + static_cast<size_t>(ch) * K + j, acc);
          } else {
            out[static_cast<size_t>(g * DK_MAX_GROUPS + slot) * Hc * K + task] = acc;
          }
        }
        if (!atomic && ct == 0) group_of[g * DK_MAX_GROUPS + slot] = grp;
        named_barrier(2, 256);
      }
      if (!atomic && ct == 0)
        for (int slot = n_slots; slot < DK_MAX_GROUPS; ++slot) group_of[g * DK_MAX_GROUPS + slot] = -1;
    }
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
