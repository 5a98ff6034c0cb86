// pt_cl.cu -- channels-last ([B, L, H]) depthwise Conv1D: FWD, dX and dK.
//
// The S4 block of the reference holds its activations as [B, L, H] and
// transposes them to [B, H, L] around the convolution and back
// (kernels/warp_tiled_ampere.py:1186, :1190).  These kernels convolve the
// [B, L, H] tensors in place of those two copies.
//
// One thread owns one (b, h) sequence; a warp covers 32 consecutive channels
// of one batch row, so every per-t load or store of the warp is one coalesced
// 128-byte row segment.  The sequence (L values) and the channel's taps (K)
// live in registers, so the FMA nests are compile-time: kernels are
// instantiated for maxima LMAX, KMAX in {16, 32, 48} and take the runtime L, K
// by zero-padding the sequence past L and shifting the taps by s = PMAX - pad
// (tap register j' holds k[j' - s], so register j' always multiplies element
// t + j' - PMAX -- a compile-time index).
//
// dK: each thread accumulates its channel's K taps over a slice of batch rows;
// the CTA (32 channels x 4 warps of rows) sums its warps in a fixed order into
// one partial per (slice, h), and a second kernel sums the slices in order.
// Bit-reproducible for a fixed device (the slice count follows the SM count).
#include "pt_cl.h"

#include <cstdint>

namespace pt {
namespace cl {

constexpr int CH = 32;    // channels per CTA (one warp-wide row segment)
constexpr int ROWS = 4;   // batch rows per CTA (one per warp)

template <int LMAX, int KMAX, bool REV>
__global__ void __launch_bounds__(CH * ROWS)
    cl_conv_kernel(const float* __restrict__ in, const float* __restrict__ k, float* __restrict__ out, int B,
                   int L, int H, int K) {
  const int h = static_cast<int>(blockIdx.x) * CH + static_cast<int>(threadIdx.x);
  const int b = static_cast<int>(blockIdx.y) * ROWS + static_cast<int>(threadIdx.y);
  if (h >= H || b >= B) return;
  // Compile-time centre: tap register j' multiplies element t + j' - PMAX.  It
  // must satisfy pad <= PMAX <= KMAX - K + pad for every K <= KMAX: KMAX/2 for
  // FWD (pad = K/2), KMAX/2 - 1 for dX (pad = K - 1 - K/2).
  constexpr int PMAX = REV ? KMAX / 2 - 1 : KMAX / 2;
  const int pad = REV ? (K - 1 - K / 2) : K / 2;
  const int s = PMAX - pad;  // >= 0, and s + K - 1 < KMAX
  const float* kh = k + static_cast<size_t>(h) * K;
  float w[KMAX];
#pragma unroll
  for (int jp = 0; jp < KMAX; ++jp) {
    const int j = jp - s;
    w[jp] = (j >= 0 && j < K) ? __ldg(kh + (REV ? K - 1 - j : j)) : 0.f;
  }
  const size_t base = static_cast<size_t>(b) * L * H + h;
  float v[LMAX];
#pragma unroll
  for (int t = 0; t < LMAX; ++t) v[t] = (t < L) ? __ldg(in + base + static_cast<size_t>(t) * H) : 0.f;
  // Four outputs at a time: four independent FMA chains per tap loop.
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
        if (t0 + u < L) out[base + static_cast<size_t>(t0 + u) * H] = acc[u];
    }
  }
}

// The same convolution with the input rows staged through shared memory: each
// warp walks `rows` batch rows (b = b0 + warp, + ROWS, ...) and prefetches the
// next row with 16-byte cp.async while it computes the current one, so its
// loads overlap its FMAs (the direct kernel above waits for every row it
// loads).  Needs H % 4 == 0 (16-byte aligned row segments).
__device__ __forceinline__ void cl_cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}

template <int LMAX, int KMAX, bool REV>
__global__ void __launch_bounds__(CH * ROWS)
    cl_conv_pipe_kernel(const float* __restrict__ in, const float* __restrict__ k, float* __restrict__ out, int B,
                        int L, int H, int K, int rows) {
  __shared__ __align__(16) float buf[2][ROWS][LMAX][CH];
  const int tx = static_cast<int>(threadIdx.x), ty = static_cast<int>(threadIdx.y);
  const int h0 = static_cast<int>(blockIdx.x) * CH;
  const int h = h0 + tx;
  constexpr int PMAX = REV ? KMAX / 2 - 1 : KMAX / 2;
  const int pad = REV ? (K - 1 - K / 2) : K / 2;
  const int s = PMAX - pad;
  float w[KMAX];
#pragma unroll
  for (int jp = 0; jp < KMAX; ++jp) {
    const int j = jp - s;
    w[jp] = (h < H && j >= 0 && j < K) ? __ldg(k + static_cast<size_t>(h) * K + (REV ? K - 1 - j : j)) : 0.f;
  }
  const int bfirst = static_cast<int>(blockIdx.y) * ROWS * rows + ty;
  // Lane tx copies 16-byte chunks id = tx + 32 m of the row: t = id / 8, part id % 8.
  auto prefetch = [&](int b, int st) {
    if (b < B) {
#pragma unroll
      for (int m = 0; m < LMAX * CH / 4 / 32; ++m) {
        const int id = tx + 32 * m;
        const int t = id >> 3, part = id & 7;
        if (t < L && h0 + 4 * part < H)
          cl_cp_async16(&buf[st][ty][t][4 * part], in + (static_cast<size_t>(b) * L + t) * H + h0 + 4 * part);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  prefetch(bfirst, 0);
  for (int i = 0; i < rows; ++i) {
    const int b = bfirst + i * ROWS;
    if (b >= B) break;
    prefetch(b + ROWS, (i + 1) & 1);
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncwarp();
    const int st = i & 1;
    float v[LMAX];
#pragma unroll
    for (int t = 0; t < LMAX; ++t) v[t] = (t < L) ? buf[st][ty][t][tx] : 0.f;
    __syncwarp();  // the buffer is refilled by the next iteration's prefetch
    if (h < H) {
      const size_t base = static_cast<size_t>(b) * L * H + h;
#pragma unroll
      for (int t0 = 0; t0 < LMAX; t0 += 4) {
        if (t0 < L) {
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int jp = 0; jp < KMAX; ++jp)
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int ii = t0 + u + jp - PMAX;
              if (ii >= 0 && ii < LMAX) acc[u] = fmaf(w[jp], v[ii], acc[u]);
            }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (t0 + u < L) out[base + static_cast<size_t>(t0 + u) * H] = acc[u];
        }
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

template <int LMAX, int KMAX>
__global__ void __launch_bounds__(CH * ROWS)
    cl_dk_kernel(const float* __restrict__ dy, const float* __restrict__ x, float* __restrict__ partial, int B,
                 int L, int H, int K, int rows_per_slice) {
  __shared__ float red[ROWS][KMAX][CH];
  const int tx = static_cast<int>(threadIdx.x), ty = static_cast<int>(threadIdx.y);
  const int h = static_cast<int>(blockIdx.x) * CH + tx;
  const int slice = static_cast<int>(blockIdx.y);
  constexpr int PMAX = KMAX / 2;
  const int s = PMAX - K / 2;  // acc[j'] is the gradient of tap j' - s
  float acc[KMAX];
#pragma unroll
  for (int jp = 0; jp < KMAX; ++jp) acc[jp] = 0.f;
  if (h < H) {
    const int b0 = slice * rows_per_slice;
    const int b1 = min(B, b0 + rows_per_slice);
    for (int b = b0 + ty; b < b1; b += ROWS) {
      // Both rows into registers first: 2 L loads in flight per thread.
      const size_t base = static_cast<size_t>(b) * L * H + h;
      float v[LMAX], d[LMAX];
#pragma unroll
      for (int t = 0; t < LMAX; ++t) {
        v[t] = (t < L) ? __ldg(x + base + static_cast<size_t>(t) * H) : 0.f;
        d[t] = (t < L) ? __ldg(dy + base + static_cast<size_t>(t) * H) : 0.f;
      }
#pragma unroll
      for (int t = 0; t < LMAX; ++t) {
#pragma unroll
        for (int jp = 0; jp < KMAX; ++jp) {
          const int i = t + jp - PMAX;
          if (i >= 0 && i < LMAX) acc[jp] = fmaf(d[t], v[i], acc[jp]);
        }
      }
    }
  }
#pragma unroll
  for (int jp = 0; jp < KMAX; ++jp) red[ty][jp][tx] = acc[jp];
  __syncthreads();
  if (h >= H) return;
  for (int jp = ty; jp < KMAX; jp += ROWS) {
    const int j = jp - s;
    if (j < 0 || j >= K) continue;
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) sum += red[r][jp][tx];
    partial[(static_cast<size_t>(slice) * H + h) * K + j] = sum;
  }
}

__global__ void cl_dk_reduce_kernel(const float* __restrict__ partial, float* __restrict__ dk, int slices, int HK,
                                    int accumulate) {
  const int idx = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (idx >= HK) return;
  float sum = 0.f;
  for (int e = 0; e < slices; ++e) sum += partial[static_cast<size_t>(e) * HK + idx];
  dk[idx] = accumulate ? dk[idx] + sum : sum;
}

namespace {

int bucket(int n) { return n <= 16 ? 16 : (n <= 32 ? 32 : 48); }

template <bool REV>
const void* conv_pipe_func(int lmax, int kmax) {
#define PT_CL_CONV(LM, KM) \
  if (lmax == LM && kmax == KM) return reinterpret_cast<const void*>(&cl_conv_pipe_kernel<LM, KM, REV>);
  PT_CL_CONV(16, 16) PT_CL_CONV(16, 32) PT_CL_CONV(16, 48)
  PT_CL_CONV(32, 16) PT_CL_CONV(32, 32) PT_CL_CONV(32, 48)
  PT_CL_CONV(48, 16) PT_CL_CONV(48, 32) PT_CL_CONV(48, 48)
#undef PT_CL_CONV
  return nullptr;
}

template <bool REV>
const void* conv_func(int lmax, int kmax) {
#define PT_CL_CONV(LM, KM) \
  if (lmax == LM && kmax == KM) return reinterpret_cast<const void*>(&cl_conv_kernel<LM, KM, REV>);
  PT_CL_CONV(16, 16) PT_CL_CONV(16, 32) PT_CL_CONV(16, 48)
  PT_CL_CONV(32, 16) PT_CL_CONV(32, 32) PT_CL_CONV(32, 48)
  PT_CL_CONV(48, 16) PT_CL_CONV(48, 32) PT_CL_CONV(48, 48)
#undef PT_CL_CONV
  return nullptr;
}

const void* dk_func(int lmax, int kmax) {
#define PT_CL_DK(LM, KM) \
  if (lmax == LM && kmax == KM) return reinterpret_cast<const void*>(&cl_dk_kernel<LM, KM>);
  PT_CL_DK(16, 16) PT_CL_DK(16, 32) PT_CL_DK(16, 48)
  PT_CL_DK(32, 16) PT_CL_DK(32, 32) PT_CL_DK(32, 48)
  PT_CL_DK(48, 16) PT_CL_DK(48, 32) PT_CL_DK(48, 48)
#undef PT_CL_DK
  return nullptr;
}

// Batch-row slices of the dK kernel: one full wave of CTAs (resident CTAs per
// SM from the occupancy of the bucket's instantiation, times the SMs).
int dk_slices(int B, int L, int H, int K, int sm_count) {
  const int hb = (H + CH - 1) / CH;
  int per_sm = 0;
  const void* f = dk_func(bucket(L), bucket(K));
  if (!f || cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, f, CH * ROWS, 0) != cudaSuccess || per_sm < 1)
    per_sm = 2;
  int slices = (per_sm * (sm_count > 0 ? sm_count : 148)) / hb;
  const int max_slices = (B + ROWS - 1) / ROWS;
  if (slices > max_slices) slices = max_slices;
  return slices < 1 ? 1 : slices;
}

}  // namespace

cudaError_t launch_conv(const float* in, const float* k, float* out, int B, int L, int H, int K, bool rev,
                        cudaStream_t stream) {
  if (H % 4 == 0) {
    // Pipelined form: each warp streams kRowsPerWarp batch rows.
    constexpr int kRowsPerWarp = 8;
    const void* fp =
        rev ? conv_pipe_func<true>(bucket(L), bucket(K)) : conv_pipe_func<false>(bucket(L), bucket(K));
    if (!fp) return cudaErrorInvalidValue;
    const long long groups = (static_cast<long long>(B) + ROWS * kRowsPerWarp - 1) / (ROWS * kRowsPerWarp);
    if (groups <= 65535) {
      int rows = kRowsPerWarp;
      dim3 grid((H + CH - 1) / CH, static_cast<unsigned>(groups)), block(CH, ROWS);
      void* args[] = {const_cast<float**>(&in), const_cast<float**>(&k), &out, &B, &L, &H, &K, &rows};
      return cudaLaunchKernel(fp, grid, block, args, 0, stream);
    }
  }
  const void* f = rev ? conv_func<true>(bucket(L), bucket(K)) : conv_func<false>(bucket(L), bucket(K));
  if (!f) return cudaErrorInvalidValue;
  // gridDim.y holds batch rows / ROWS and is limited to 65535: launch in chunks.
  constexpr int kMaxRows = 65535 * ROWS;
  for (int b0 = 0; b0 < B; b0 += kMaxRows) {
    int nb = B - b0 < kMaxRows ? B - b0 : kMaxRows;
    const size_t off = static_cast<size_t>(b0) * L * H;
    const float* inp = in + off;
    float* outp = out + off;
    dim3 grid((H + CH - 1) / CH, (nb + ROWS - 1) / ROWS), block(CH, ROWS);
    void* args[] = {const_cast<float**>(&inp), const_cast<float**>(&k), &outp, &nb, &L, &H, &K};
    cudaError_t e = cudaLaunchKernel(f, grid, block, args, 0, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

size_t dk_workspace_bytes(int B, int L, int H, int K, int sm_count) {
  (void)L;
  return static_cast<size_t>(dk_slices(B, L, H, K, sm_count)) * H * K * sizeof(float);
}

cudaError_t launch_dk(const float* dy, const float* x, float* dk, int B, int L, int H, int K, int accumulate,
                      void* ws, int sm_count, cudaStream_t stream) {
  const void* f = dk_func(bucket(L), bucket(K));
  if (!f) return cudaErrorInvalidValue;
  int slices = dk_slices(B, L, H, K, sm_count);
  int rows = (B + slices - 1) / slices;
  float* partial = static_cast<float*>(ws);
  dim3 grid((H + CH - 1) / CH, slices), block(CH, ROWS);
  void* args[] = {const_cast<float**>(&dy), const_cast<float**>(&x), &partial, &B, &L, &H, &K, &rows};
  cudaError_t e = cudaLaunchKernel(f, grid, block, args, 0, stream);
  if (e != cudaSuccess) return e;
  const int hk = H * K;
  cl_dk_reduce_kernel<<<(hk + 255) / 256, 256, 0, stream>>>(partial, dk, slices, hk, accumulate);
  return cudaGetLastError();
}

}  // namespace cl
}  // namespace pt
