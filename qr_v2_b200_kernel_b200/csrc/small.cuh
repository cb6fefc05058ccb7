// Fully fused QR of small matrices: one CTA factors one whole n x n matrix (n <= NMAX) in a
// single launch -- the one-CTA-per-matrix path of the reference's fused kernel
// (submission.py:72-175), restructured for shared memory and 32 warps:
//
//   the matrix lives in shared memory for the whole factorisation (read once from A,
//   written once to H); for each 32-column panel warp c pulls panel column c into registers
//   and factor_panel_owner produces the reflectors, tau and T; then the trailing columns are
//   updated in shared memory with the compact-WY product C <- C - V T^T (V^T C)
//   (milestones/01_eager_official123203us.py:102-107), all 1024 threads sharing
//     W  = V^T C   (warp = reflector c, lanes = trailing columns),
//     W2 = T^T W   (same mapping),
//     C -= V W2    (warp = rows, lanes = trailing columns).
#pragma once

#include "panel.cuh"

namespace qrb200 {

template <int NMAX>
struct SmallShared {
  static constexpr int LD = NMAX + 1;  // odd row stride: column-parallel reads hit distinct banks
  float M[NMAX * LD];
  float W[32][NMAX];   // V^T C, then T^T V^T C
  float W2[32][NMAX];
  OwnerShared<NMAX / 32, 1> ps;
};

template <int NMAX>
__global__ void __launch_bounds__(kPanelThreads) small_qr_kernel(const float* __restrict__ A, long long a_bstride,
                                                                  float* __restrict__ H, float* __restrict__ tau,
                                                                  int n) {
  constexpr int NT = kPanelThreads;
  constexpr int RPL = NMAX / 32;
  constexpr int LD = SmallShared<NMAX>::LD;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  SmallShared<NMAX>& sh = *reinterpret_cast<SmallShared<NMAX>*>(smem_raw);
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* __restrict__ Ab = A + (long long)b * a_bstride;
  float* __restrict__ Hb = H + (long long)b * n * n;
  float* __restrict__ taub = tau + (long long)b * n;

  for (int e = tid; e < n * n; e += NT) sh.M[(e / n) * LD + (e % n)] = Ab[e];
  __syncthreads();

  for (int k = 0; k < n; k += 32) {
    const int m = n - k;
    const int w = min(32, m);
    const int nc = n - k - w;
    float* Mk = sh.M + k * LD + k;  // panel origin
    float a[1][RPL];
#pragma unroll
    for (int i = 0; i < RPL; ++i) {
      const int lr = lane + 32 * i;
      a[0][i] = (lr < m && warp < w) ? Mk[lr * LD + warp] : 0.f;
    }
    for (int e = tid; e < 32 * 33; e += NT) (&sh.ps.T[0][0])[e] = 0.f;
    __syncthreads();
    factor_panel_owner<RPL, 1, true>(a, w, w, sh.ps, taub + k);
    __syncthreads();
    if (warp == 0) larft_inverse_warp(sh.ps.T, sh.ps.G, sh.ps.tau, w);
    if (warp < w) {
#pragma unroll
      for (int i = 0; i < RPL; ++i) {
        const int lr = lane + 32 * i;
        if (lr < m) Mk[lr * LD + warp] = a[0][i];
      }
    }
    __syncthreads();
    if (nc <= 0) break;
    // W[c][j] = sum_r V[r][c] C[r][j]; warp = c, lanes stride the trailing columns.
    for (int j = lane; j < nc; j += 32) {
      float s = 0.f;
      const int c = warp;
      if (c < w) {
        s = Mk[c * LD + 32 + j];  // V[c][c] = 1
        for (int r = c + 1; r < m; ++r) s = fmaf(Mk[r * LD + c], Mk[r * LD + 32 + j], s);
      }
      sh.W[c][j] = s;
    }
    __syncthreads();
    // W2[i][j] = sum_{c <= i} T[c][i] W[c][j]
    for (int j = lane; j < nc; j += 32) {
      const int i = warp;
      float s = 0.f;
      for (int c = 0; c <= i; ++c) s = fmaf(sh.ps.T[c][i], sh.W[c][j], s);
      sh.W2[i][j] = s;
    }
    __syncthreads();
    // C[r][j] -= sum_c V[r][c] W2[c][j]; warp strides rows, lanes stride columns.
    for (int r = warp; r < m; r += 32) {
      float v[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) v[c] = (c < w) ? ((r > c) ? Mk[r * LD + c] : (r == c ? 1.f : 0.f)) : 0.f;
      for (int j = lane; j < nc; j += 32) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          s0 = fmaf(v[c], sh.W2[c][j], s0);
          s1 = fmaf(v[c + 1], sh.W2[c + 1][j], s1);
        }
        Mk[r * LD + 32 + j] -= s0 + s1;
      }
    }
    __syncthreads();
  }
  for (int e = tid; e < n * n; e += NT) Hb[e] = sh.M[(e / n) * LD + (e % n)];
}

}  // namespace qrb200
