// pt_tc_kernels.cuh -- FWD / DX on the 5th-generation tensor cores (tcgen05).
//
// For one channel h the same-length convolution is a matrix product: a row of
// L inputs times an L x L Toeplitz matrix whose entries are the channel's taps,
//   FWD  y[t]  = sum_s x[s]  T[s][t],  T[s][t] = k[s - t + K/2]   (0 <= . < K)
//   DX   dx[t] = sum_s dy[s] T[s][t],  T[s][t] = k[t - s + K/2]
// A tile is 128 batch rows (the MMA M) of a "super-row" of W columns: one
// channel (W = L rounded up to 16, padding columns read as zero), or, when
// 48 % L == 0 and L <= 24, Hc = 48 / L adjacent channels (W = 48; the
// channels of one batch row are contiguous in HBM).  The GEMM is then
// 128 x W x W with a block-diagonal Toeplitz operand, one L x L block per
// channel, so every tile moves the same bytes whatever L is.
//
// FP32 accuracy from TF32 tensor cores (the "3xTF32" split): every operand
// value v is written as hi + lo with hi = v rounded to TF32 (10 mantissa bits,
// round to nearest, ties away from zero) and lo = (v - hi) rounded the same
// way; y = x_hi (T_hi + T_lo) + x_lo T_hi, accumulated in FP32 in tensor
// memory.  The dropped x_lo T_lo term and the rounding of lo bound the error
// of one product by about 2^-21 of |x T|, below the FP32 rounding of the FFMA
// path's sum of up to 48 products.
//
// Shared-memory bandwidth is what bounds a 128 x 48 x 8 MMA whose operands
// both sit in shared memory, so A lives in tensor memory: converter threads
// read their tile row from the TMA stage, split it, and write hi and lo to
// TMEM (lane = row, column = k); the stage is free again as soon as it has
// been read.  Only the Toeplitz operand is read from shared memory: one
// 2N-row operand [T_hi; T_lo], so each 8-wide k step is two MMAs,
//   D[:, 0:2N] (+)= A_hi [T_hi; T_lo]^T     D[:, 0:N] += A_lo T_hi^T
// and the epilogue adds D[:, t] + D[:, N + t] (fewer, wider MMAs measured
// faster than three N-wide ones).
//
// Data movement: tile rows are TMA-loaded as one box of 32 floats with the
// 128-byte swizzle (columns 0..31) and/or one box of 16 floats with the 64-byte
// swizzle (columns 32..47, or 0..15 when W = 16); a 3-D map (L, H, B) per
// channel, or a 2-D map over [B, H*L] for packed super-rows.  Columns past
// the channel (or past H*L) and rows past B read as zeros and are clipped on
// store.  The Toeplitz operand is written in the K-major canonical layouts
// of the MMA shared-memory descriptors (same swizzles).  Tiles are ordered
// batch-major (channel group fastest) and dealt round-robin to persistent
// CTAs, so the CTAs in flight together stream contiguous slabs of HBM.  CTA g
// then visits groups (g + i*G) mod Hg, a sequence of period P = Hg / gcd(G,
// Hg); the host picks G with P <= 2 where it can, and the CTA builds its one
// or two Toeplitz operands once and keeps them.  Otherwise (P = 0 passed) the
// operand is rebuilt for every tile into a ring of two slots.
//
// Roles (448 threads, one CTA per SM):
//   warp 0       TMA producer: ring of 5 raw stages
//   warp 1       allocates 512 TMEM columns (2 A slots of hi + lo, 2
//                accumulators of 2N columns); lane 0 issues the MMAs and
//                commits them to mbarriers
//   warps 2-9    converters: two threads per tile row (warp quadrant = TMEM lane
//                group), half a row each; they also build the Toeplitz operand
//   warps 10-13  epilogue: TMEM -> registers -> one of 2 swizzled staging
//                buffers -> TMA store
// Every wait is bounded (%globaltimer); on expiry the kernel records a bit in
// the device error word, stops issuing, drains its own copies and MMAs, frees
// its tensor memory and returns.
#pragma once

#include "pt_kernels.cuh"

namespace pt {
namespace tc {

constexpr int M = 128;           // batch rows per tile (MMA M)
constexpr int STAGES = 5;        // TMA ring of raw tiles
constexpr int OUT_SLOTS = 2;     // output staging for the TMA store
constexpr int B_SLOTS = 2;       // Toeplitz operand [T_hi; T_lo]
constexpr int A_SLOTS = 2;       // A hi/lo in tensor memory
constexpr int ACC_SLOTS = 2;     // accumulators in tensor memory
constexpr int TMEM_COLS = 512;   // A slots @0, 128 (lo @+64); D @256, 384
constexpr int A_COL0 = 0;
constexpr int A_SLOT_COLS = 128;
constexpr int LO_COLS = 64;      // A_lo sits 64 columns after A_hi
constexpr int D_COL0 = A_SLOTS * A_SLOT_COLS;
constexpr int D_SLOT_COLS = 128;
constexpr int CONVERTERS = 256;  // warps 2-9
constexpr int EPI0 = 64 + CONVERTERS;  // first epilogue thread (warps 10-13)
constexpr int THREADS = EPI0 + 128;
static_assert(D_COL0 + ACC_SLOTS * D_SLOT_COLS <= TMEM_COLS, "tensor memory budget");

constexpr unsigned DEVERR_TC_CONVERT = 8u;   // converters: a tile, A slot or operand never freed
constexpr unsigned DEVERR_TC_MMA = 16u;      // MMA issuer: converted A or a free accumulator never came
constexpr unsigned DEVERR_TC_EPILOGUE = 32u; // epilogue: an accumulator was never completed

// Shared-memory geometry for LB = 1 (W = 16: one 64-B box), 2 (W = 32: one
// 128-B box), 3 (W = 48: a 128-B box and a 64-B box).
template <int LB>
struct Geo {
  static constexpr int RB128 = (LB >= 2) ? 128 : 0;  // bytes per row, 128-B swizzled box
  static constexpr int RB64 = (LB & 1) ? 64 : 0;     // bytes per row, 64-B swizzled box
  static constexpr int C128 = RB128 / 16;            // 16-B chunks per row in each box
  static constexpr int C64 = RB64 / 16;
  static constexpr int S64 = (LB >= 2) ? 32 : 0;     // first column held by the 64-B box
  static constexpr int N = 16 * LB;                  // MMA N = W = padded reduction extent
  static constexpr int KSTEPS = N / 8;               // tf32 MMAs reduce over 8 columns
  static constexpr int K128 = C128 / 2;              // k steps inside the 128-B box
  static constexpr int TILE = M * (RB128 + RB64);    // one raw or staged tile
  static constexpr int BOX64 = M * RB128;            // offset of the 64-B box in a tile
  static constexpr int BMAT = 2 * N * (RB128 + RB64);  // [T_hi; T_lo]: 2N rows
  static constexpr int BLO128 = N * RB128;           // T_lo rows in the 128-B box
  static constexpr int BBOX64 = 2 * N * RB128;       // offset of the 64-B box
  static constexpr int BLO64 = N * RB64;             // T_lo rows in the 64-B box
  static constexpr int OFF_OUT = STAGES * TILE;
  static constexpr int OFF_B = OFF_OUT + OUT_SLOTS * TILE;
  static constexpr int OFF_BAR = OFF_B + B_SLOTS * BMAT;
  static constexpr int N_BARS = 2 * STAGES + 2 * A_SLOTS + 2 * ACC_SLOTS;
  static constexpr int OFF_TMEM = OFF_BAR + N_BARS * 8;
  static constexpr int SMEM = OFF_TMEM + 16 + 1024;  // + slack for 1024-B alignment
  static_assert(TILE % 1024 == 0 && BMAT % 1024 == 0 && BBOX64 % 1024 == 0 && BOX64 % 1024 == 0 &&
                    BLO128 % 1024 == 0 && BLO64 % 1024 == 0,
                "swizzled operands must start on 1024-byte boundaries");
  static_assert(N <= LO_COLS && 2 * N <= D_SLOT_COLS, "A and accumulator slots must fit their columns");
};

// ---------------------------------------------------------------------------
// tcgen05 / TMEM helpers (PTX ISA 8.6+, sm_100a).
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor of a K-major operand with the 128-B or 64-B
// swizzle: start address >> 4 (bits 0-13), leading offset unused for swizzled
// K-major (1), stride between 8-row groups >> 4 (bits 32-45), descriptor
// version 1 (bits 46-47), swizzle mode (bits 61-63: 2 = 128 B, 4 = 64 B).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t addr, bool sw128) {
  const uint64_t sbo = sw128 ? 1024u : 512u;
  const uint64_t mode = sw128 ? 2u : 4u;
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((sbo >> 4) << 32) |
         (1ull << 46) | (mode << 61);
}

// Instruction descriptor: D f32 (bits 4-5 = 1), A and B tf32 (bits 7-9 and
// 10-12 = 2), both K-major, N >> 3 (bits 17-22), M >> 4 (bits 24-28).
template <int N>
constexpr uint32_t idesc_tf32_m128() {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// D[M x N] (+)= A[M x 8] B[N x 8]^T with A in tensor memory (lane m, column k)
// and B a K-major shared-memory operand.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes (one lane per thread).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 8 consecutive 32-bit columns of this warp's 32 TMEM lanes (one lane per thread).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// v rounded to TF32 (sign, 8 exponent bits, 10 mantissa bits): adding half a
// TF32 unit to the magnitude bits and truncating rounds to nearest with ties
// away from zero; a mantissa carry correctly bumps the exponent.
__device__ __forceinline__ float tf32_round(float v) {
  return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u);
}

__device__ __forceinline__ void split4(const float4 v, float4& hi, float4& lo) {
  hi.x = tf32_round(v.x);
  hi.y = tf32_round(v.y);
  hi.z = tf32_round(v.z);
  hi.w = tf32_round(v.w);
  lo.x = tf32_round(v.x - hi.x);
  lo.y = tf32_round(v.y - hi.y);
  lo.z = tf32_round(v.z - hi.z);
  lo.w = tf32_round(v.w - hi.w);
}

// Byte offset of 16-byte chunk c of row r in a swizzled box (TMA and the MMA
// descriptors agree on this address-based XOR pattern on 1024-B-aligned buffers).
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint32_t sw64_off(int r, int c) {
  return static_cast<uint32_t>(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// ---------------------------------------------------------------------------
// The kernel.  Hc channels per super-row (1 unless PACKED), Hg = ceil(H / Hc)
// channel groups, n_tiles = ceil(B / 128) * Hg; tile tau covers group tau % Hg
// and batch rows [128 * (tau / Hg), +128).  CTA g takes tiles g, g + G, ...
// bperiod = number of distinct groups CTA g visits (1 or 2), or 0.
// PACKED: 2-D tensor maps over [B, H*L] (coordinates: column, batch);
// otherwise 3-D maps (L, H, B) (coordinates: column, channel, batch).
// ---------------------------------------------------------------------------
template <int OP, int LB, bool PACKED>
__global__ void __launch_bounds__(THREADS, 1)
    tc_conv_kernel(const __grid_constant__ CUtensorMap tm_in128,
                   const __grid_constant__ CUtensorMap tm_in64,
                   const __grid_constant__ CUtensorMap tm_out128,
                   const __grid_constant__ CUtensorMap tm_out64, const float* __restrict__ taps,
                   int H, int L, int K, int Hc, int Hg, int n_tiles, int bperiod, unsigned* err) {
  using GG = Geo<LB>;
  constexpr int N = GG::N;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = aligned_smem(smem_raw);
  const uint32_t base = smem_u32(sm);
  const int warp = static_cast<int>(threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31);
  const uint32_t bar0 = base + GG::OFF_BAR;
  const uint32_t tmem_slot = base + GG::OFF_TMEM;
  // Barriers: full (TMA landed), sfree (stage read by the converters), aready
  // (A slot written), adone (MMAs reading the A slot / Toeplitz slot done),
  // mdone (accumulator complete), accfree (accumulator read by the epilogue).
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto sfree = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto aready = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto adone = [&](int a) { return bar0 + 8u * (2 * STAGES + A_SLOTS + a); };
  auto mdone = [&](int d) { return bar0 + 8u * (2 * STAGES + 2 * A_SLOTS + d); };
  auto accfree = [&](int d) { return bar0 + 8u * (2 * STAGES + 2 * A_SLOTS + ACC_SLOTS + d); };
  const int G = static_cast<int>(gridDim.x);
  const int g = static_cast<int>(blockIdx.x);
  const int n_it = (g < n_tiles) ? (n_tiles - 1 - g) / G + 1 : 0;
  const int W = Hc * L;  // packed super-row width (PACKED only)

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(sfree(s), CONVERTERS / 32);  // one arrival per converter warp
    }
    for (int a = 0; a < A_SLOTS; ++a) {
      mbar_init(aready(a), CONVERTERS / 32);
      mbar_init(adone(a), 1);
    }
    for (int d = 0; d < ACC_SLOTS; ++d) {
      mbar_init(mdone(d), 1);
      mbar_init(accfree(d), 4);  // one arrival per epilogue warp
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + GG::OFF_TMEM);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      if (LB >= 2) prefetch_tmap(&tm_in128);
      if (LB & 1) prefetch_tmap(&tm_in64);
      int issued = 0;
      for (int i = 0; i < n_it; ++i) {
        const int s = i % STAGES;
        if (i >= STAGES &&
            !mbar_wait_bounded(sfree(s), ((i / STAGES) - 1) & 1, err, DEVERR_TIMEOUT_DONE))
          break;
        const int tau = g + i * G;
        const int grp = tau % Hg;
        const int b0 = (tau / Hg) * M;
        const uint32_t dst = base + static_cast<uint32_t>(s * GG::TILE);
        mbar_arrive_expect_tx(full(s), GG::TILE);
        if constexpr (PACKED) {
          if constexpr (LB >= 2) tma_load_2d(dst, &tm_in128, grp * W, b0, full(s));
          if constexpr (LB & 1) tma_load_2d(dst + GG::BOX64, &tm_in64, grp * W + GG::S64, b0, full(s));
        } else {
          if constexpr (LB >= 2) tma_load_3d(dst, &tm_in128, 0, grp, b0, full(s));
          if constexpr (LB & 1) tma_load_3d(dst + GG::BOX64, &tm_in64, GG::S64, grp, b0, full(s));
        }
        issued = i + 1;
      }
      // Every issued load must land before the CTA may exit.
      for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i)
        if (!mbar_wait_bounded(full(i % STAGES), (i / STAGES) & 1, err, DEVERR_TIMEOUT_DRAIN)) break;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_n2 = idesc_tf32_m128<2 * N>();
      constexpr uint32_t idesc_n = idesc_tf32_m128<N>();
      int issued = 0;
      for (int i = 0; i < n_it; ++i) {
        const int a = i % A_SLOTS, d = i % ACC_SLOTS;
        const int bs = bperiod ? i % bperiod : i % B_SLOTS;
        if (!mbar_wait_bounded(aready(a), (i / A_SLOTS) & 1, err, DEVERR_TC_MMA)) break;
        if (i >= ACC_SLOTS &&
            !mbar_wait_bounded(accfree(d), ((i / ACC_SLOTS) - 1) & 1, err, DEVERR_TC_MMA))
          break;
        tc_fence_after();
        const uint32_t a_hi = tmem + static_cast<uint32_t>(A_COL0 + a * A_SLOT_COLS);
        const uint32_t a_lo = a_hi + LO_COLS;
        const uint32_t bmat = base + static_cast<uint32_t>(GG::OFF_B + bs * GG::BMAT);
        const uint32_t dacc = tmem + static_cast<uint32_t>(D_COL0 + d * D_SLOT_COLS);
#pragma unroll
        for (int kk = 0; kk < GG::KSTEPS; ++kk) {
          const bool in128 = kk < GG::K128;
          // [T_hi; T_lo] rows 0..2N-1 (the 2N-wide MMA), T_hi alone = rows 0..N-1.
          const uint64_t bdesc = kmajor_desc(
              bmat + (in128 ? 32u * kk : GG::BBOX64 + 32u * (kk - GG::K128)), in128);
          mma_tf32_ts(dacc, a_hi + 8u * kk, bdesc, idesc_n2, kk > 0);  // A_hi [T_hi; T_lo]
          mma_tf32_ts(dacc, a_lo + 8u * kk, bdesc, idesc_n, 1);        // A_lo T_hi
        }
        mma_commit(adone(a));
        mma_commit(mdone(d));
        issued = i + 1;
      }
      // No MMA may still be running when tensor memory is released.
      if (issued > 0)
        mbar_wait_bounded(mdone((issued - 1) % ACC_SLOTS), ((issued - 1) / ACC_SLOTS) & 1, err,
                          DEVERR_TC_MMA);
    }
    __syncwarp();
  } else if (warp < EPI0 / 32) {
    // ---------------- converters ----------------
    const int ct = static_cast<int>(threadIdx.x) - 64;  // 0..255
    const int quad = warp & 3;                          // TMEM lanes 32*quad .. +31
    const int row = 32 * quad + lane;                   // tile row of this thread
    const int half = (warp - 2) >> 2;                   // which half of the row
    constexpr int CH = (GG::C128 + GG::C64) / 2;        // 16-byte chunks per half row
    const uint32_t lane_base = static_cast<uint32_t>(32 * quad) << 16;
    const int pad = K / 2;
    for (int i = 0; i < n_it; ++i) {
      const int s = i % STAGES, a = i % A_SLOTS;
      const bool rebuild = (bperiod == 0) || (i < bperiod);
      const int bs = bperiod ? i % bperiod : i % B_SLOTS;
      // The A slot was last read by the MMAs of tile i - A_SLOTS, a rebuilt
      // Toeplitz slot by those of tile i - B_SLOTS; the tile must have landed.
      bool ok = true;
      if (i >= A_SLOTS)
        ok = mbar_wait_bounded(adone(a), ((i / A_SLOTS) - 1) & 1, err, DEVERR_TC_CONVERT);
      if (ok && rebuild && bperiod == 0 && i >= B_SLOTS) {
        const int ip = i - B_SLOTS;
        ok = mbar_wait_bounded(adone(ip % A_SLOTS), (ip / A_SLOTS) & 1, err, DEVERR_TC_CONVERT);
      }
      if (ok) ok = mbar_wait_bounded(full(s), (i / STAGES) & 1, err, DEVERR_TIMEOUT_FULL);
      ok = __all_sync(0xffffffffu, ok);  // each warp arrives as one, so it decides as one
      if (rebuild) {
        if (named_barrier_or(2, CONVERTERS, !ok)) break;  // all converters leave together
        // Block-diagonal [T_hi; T_lo] of group grp: row t' (hi) and N + t' (lo);
        // block c of channel grp*Hc + c covers rows and columns [c*L, c*L + L).
        const int grp = (g + i * G) % Hg;
        unsigned char* bm = sm + GG::OFF_B + bs * GG::BMAT;
        constexpr int CPR = N / 4;  // 16-byte chunks per Toeplitz row
        for (int task = ct; task < N * CPR; task += CONVERTERS) {
          const int c4 = task / N;  // row-fastest: 8 consecutive rows share a chunk column
          const int tp = task - c4 * N;
          const int sp = 4 * c4;
          const int cb = tp / L;  // L % 4 == 0: a 4-column chunk never straddles blocks
          const int ch = grp * Hc + cb;
          float v[4] = {0.f, 0.f, 0.f, 0.f};
          if (cb == sp / L && cb < Hc && ch < H) {
            const int t = tp - cb * L;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int sx = sp + q - cb * L;
              const int j = (OP == OP_FWD) ? sx - t + pad : t - sx + pad;
              if (sx < L && t < L && j >= 0 && j < K) v[q] = __ldg(taps + static_cast<size_t>(ch) * K + j);
            }
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
      } else if (!ok) {
        break;  // no converter barrier remains after the resident operands are built
      }
      // This thread's half row: 16-byte chunks [half*CH, +CH), columns k = 4*chunk.
      const unsigned char* st = sm + s * GG::TILE;
      float v[4 * CH];
#pragma unroll
      for (int u = 0; u < CH; ++u) {
        const int c = half * CH + u;
        const uint32_t off = (c < GG::C128) ? sw128_off(row, c) : GG::BOX64 + sw64_off(row, c - GG::C128);
        const float4 q = *reinterpret_cast<const float4*>(st + off);
        v[4 * u] = q.x;
        v[4 * u + 1] = q.y;
        v[4 * u + 2] = q.z;
        v[4 * u + 3] = q.w;
      }
      // The stage is read: order the reads before the next TMA write, release it.
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(sfree(s));
      float lo[4 * CH];
#pragma unroll
      for (int e = 0; e < 4 * CH; ++e) {
        const float hi = tf32_round(v[e]);
        lo[e] = tf32_round(v[e] - hi);
        v[e] = hi;
      }
      const uint32_t acol =
          tmem + lane_base + static_cast<uint32_t>(A_COL0 + a * A_SLOT_COLS + half * 4 * CH);
#pragma unroll
      for (int u = 0; u < CH / 2; ++u) {
        tmem_st8(acol + 8u * u, v + 8 * u);
        tmem_st8(acol + LO_COLS + 8u * u, lo + 8 * u);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(aready(a));
    }
  } else {
    // ---------------- epilogue ----------------
    const int et = static_cast<int>(threadIdx.x) - EPI0;  // 0..127
    const int quad = warp & 3;                            // TMEM lanes 32*quad .. +31
    const int r = 32 * quad + lane;                       // tile row = accumulator lane
    for (int j = 0; j < n_it; ++j) {
      const int d = j % ACC_SLOTS, o = j % OUT_SLOTS;
      const int tau = g + j * G;
      // The staging slot was last stored from by tile j - OUT_SLOTS.
      if (et == 0) bulk_wait_read<OUT_SLOTS - 1>();
      const bool ok = mbar_wait_bounded(mdone(d), (j / ACC_SLOTS) & 1, err, DEVERR_TC_EPILOGUE);
      if (named_barrier_or(1, 128, !ok)) break;  // all epilogue threads leave together
      tc_fence_after();
      float acc[2 * N];
      const uint32_t ta = tmem + (static_cast<uint32_t>(32 * quad) << 16) +
                          static_cast<uint32_t>(D_COL0 + d * D_SLOT_COLS);
#pragma unroll
      for (int u = 0; u < 2 * N / 16; ++u) tmem_ld16(ta + 16u * u, acc + 16 * u);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accfree(d));
      unsigned char* ob = sm + GG::OFF_OUT + o * GG::TILE;
#pragma unroll
      for (int c = 0; c < GG::C128 + GG::C64; ++c) {
        const float4 y = make_float4(acc[4 * c] + acc[N + 4 * c], acc[4 * c + 1] + acc[N + 4 * c + 1],
                                     acc[4 * c + 2] + acc[N + 4 * c + 2],
                                     acc[4 * c + 3] + acc[N + 4 * c + 3]);
        const uint32_t off = (c < GG::C128) ? sw128_off(r, c) : GG::BOX64 + sw64_off(r, c - GG::C128);
        *reinterpret_cast<float4*>(ob + off) = y;
      }
      fence_proxy_async_smem();
      named_barrier(1, 128);
      if (et == 0) {
        const int grp = tau % Hg;
        const int b0 = (tau / Hg) * M;
        const uint32_t os = base + static_cast<uint32_t>(GG::OFF_OUT + o * GG::TILE);
        if constexpr (PACKED) {
          if constexpr (LB >= 2) tma_store_2d(&tm_out128, os, grp * W, b0);
          if constexpr (LB & 1) tma_store_2d(&tm_out64, os + GG::BOX64, grp * W + GG::S64, b0);
        } else {
          if constexpr (LB >= 2) tma_store_3d(&tm_out128, os, 0, grp, b0);
          if constexpr (LB & 1) tma_store_3d(&tm_out64, os + GG::BOX64, GG::S64, grp, b0);
        }
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
