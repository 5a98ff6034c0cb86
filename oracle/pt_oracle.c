/*
 * pt_oracle.c -- TEST INFRASTRUCTURE ONLY.  CPU restatement of the reference's
 * depthwise Conv1D training path, used by tests/, __graft_entry__.smoke() and
 * bench.py's CPU baseline as the checker.  Never linked into the product.
 *
 * Algorithm (restated, not copied):
 *   FWD  y[b,h,t]  = sum_{j<K, 0<=t+j-K/2<L} x[b,h,t+j-K/2] * k[h,j]
 *        the reference PyTorch path F.pad(x,(K//2, K-1-K//2)) + grouped conv1d,
 *        benchmark/benchmark_shape_sweep_ampere.py:220-239, and the CUDA forward
 *        kernels/warp_tiled_ampere.py:403-433;
 *   DX   gx[b,h,t] = sum_{j<K, 0<=t-j+K/2<L} dy[b,h,t-j+K/2] * k[h,j]
 *        kernels/warp_tiled_ampere.py:471-498 (the adjoint of FWD);
 *   DK   gk[h,j]   = sum_b sum_{t, 0<=t+j-K/2<L} dy[b,h,t] * x[b,h,t+j-K/2]
 *        the direct FP64 reference of benchmark/check_dk_fp64_seeds.py:33-43 and
 *        benchmark/diagnose_dk_correctness.py:21-60.
 * All sums are accumulated in double precision, so the results are an FP64
 * reference for FP32 inputs.  Parity of this file is pinned against golden
 * vectors produced by the reference's own Python functions
 * (tests/golden/make_golden.py).
 */
#include <stddef.h>
#include <stdint.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline long long row_index(int b, int h, int H) { return (long long)b * H + h; }

void pto_fwd_f64(const float* x, const float* k, double* y, int B, int H, int L, int K) {
  const int pad = K / 2;
#pragma omp parallel for schedule(static)
  for (long long s = 0; s < (long long)B * H; ++s) {
    const int h = (int)(s % H);
    const float* xr = x + s * L;
    const float* kr = k + (long long)h * K;
    double* yr = y + s * L;
    for (int t = 0; t < L; ++t) {
      double acc = 0.0;
      for (int j = 0; j < K; ++j) {
        const int i = t + j - pad;
        if (i >= 0 && i < L) acc += (double)xr[i] * (double)kr[j];
      }
      yr[t] = acc;
    }
  }
}

void pto_dx_f64(const float* dy, const float* k, double* gx, int B, int H, int L, int K) {
  const int pad = K / 2;
#pragma omp parallel for schedule(static)
  for (long long s = 0; s < (long long)B * H; ++s) {
    const int h = (int)(s % H);
    const float* gr = dy + s * L;
    const float* kr = k + (long long)h * K;
    double* outr = gx + s * L;
    for (int t = 0; t < L; ++t) {
      double acc = 0.0;
      for (int j = 0; j < K; ++j) {
        const int i = t - j + pad;
        if (i >= 0 && i < L) acc += (double)gr[i] * (double)kr[j];
      }
      outr[t] = acc;
    }
  }
}

void pto_dk_f64(const float* dy, const float* x, double* gk, int B, int H, int L, int K) {
  const int pad = K / 2;
#pragma omp parallel for schedule(static)
  for (int hj = 0; hj < H * K; ++hj) {
    const int h = hj / K;
    const int j = hj % K;
    /* valid t: 0 <= t+j-pad < L */
    int t_lo = pad - j;
    if (t_lo < 0) t_lo = 0;
    int t_hi = L + pad - j;
    if (t_hi > L) t_hi = L;
    double acc = 0.0;
    for (int b = 0; b < B; ++b) {
      const long long s = row_index(b, h, H);
      const float* gr = dy + s * L;
      const float* xr = x + s * L;
      for (int t = t_lo; t < t_hi; ++t) acc += (double)gr[t] * (double)xr[t + j - pad];
    }
    gk[(long long)h * K + j] = acc;
  }
}

/* FWD for a subset of rows (flattened b*H+h indices), for spot checks at full size. */
void pto_fwd_rows_f64(const float* x, const float* k, double* y, int H, int L, int K,
                      const long long* rows, long long n_rows) {
  const int pad = K / 2;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < n_rows; ++r) {
    const long long s = rows[r];
    const int h = (int)(s % H);
    const float* xr = x + s * L;
    const float* kr = k + (long long)h * K;
    double* yr = y + r * L;
    for (int t = 0; t < L; ++t) {
      double acc = 0.0;
      for (int j = 0; j < K; ++j) {
        const int i = t + j - pad;
        if (i >= 0 && i < L) acc += (double)xr[i] * (double)kr[j];
      }
      yr[t] = acc;
    }
  }
}

void pto_dx_rows_f64(const float* dy, const float* k, double* gx, int H, int L, int K,
                     const long long* rows, long long n_rows) {
  const int pad = K / 2;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < n_rows; ++r) {
    const long long s = rows[r];
    const int h = (int)(s % H);
    const float* gr = dy + s * L;
    const float* kr = k + (long long)h * K;
    double* outr = gx + r * L;
    for (int t = 0; t < L; ++t) {
      double acc = 0.0;
      for (int j = 0; j < K; ++j) {
        const int i = t - j + pad;
        if (i >= 0 && i < L) acc += (double)gr[i] * (double)kr[j];
      }
      outr[t] = acc;
    }
  }
}

int pto_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
