// Applying Q (or Q^T) of a factorisation held as (H, tau) to another matrix: the blocked
// compact-WY application of LAPACK sormqr / sorgqr, on the tensor-core kernels of the QR's
// 128-wide trailing update. Per 128-column block of reflectors (V = unit lower trapezoid of
// H[k0:, k0:k0+128]):
//   G = V^T V (tc_gram), the four 32 x 32 panel factors from G's diagonal blocks and tau
//   (larft_blocks_kernel), the 128 x 128 block factor T (tbuild_kernel, stored transposed when
//   applying Q), Y = V T^T or V T (tc_ygemm), then C <- C - Y (V^T C) (tc_vtc128, tc_upd128).
// Q^T C = H_{n-1} ... H_0 C takes the blocks first to last with Y = V T^T; Q C = H_0 ... H_{n-1} C
// takes them last to first with Y = V T. The reference checks its factorisations through
// torch.linalg.householder_product (harness/reference.py:206), the LAPACK sorgqr that this
// replaces on the GPU.
#pragma once

#include "panel.cuh"
#include "wy_tc128.cuh"

namespace qrb200 {

// The four 32 x 32 panel factors of the block at column k0 (width ow) from the Gram partials:
// warp b sums the diagonal block G[32b:32b+32, 32b:32b+32] over the row splits and runs the
// one-warp LARFT of the panels (T^-1 = diag(1/tau) + striu(V^T V), zero row and column for
// tau = 0). Output in the batch x 4 x 32 x 32 layout tbuild_kernel reads. One CTA per matrix.
__global__ void __launch_bounds__(128) larft_blocks_kernel(const float* __restrict__ Gp, int nsplit,
                                                            const float* __restrict__ tau, long long tau_bstride,
                                                            int k0, int ow, float* __restrict__ Tpanels) {
  __shared__ float G[4][32][33];
  __shared__ float T[4][32][33];
  __shared__ float taus[4][32];
  const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int jmax = min(32, ow - 32 * warp);
  float* out = Tpanels + (long long)b * 4096 + warp * 1024;
  if (jmax <= 0) {
    for (int i = lane; i < 1024; i += 32) out[i] = 0.f;
    return;
  }
  const float* g0 = Gp + (long long)b * nsplit * kOB * kOB;
  for (int i = 0; i < 32; ++i) {
    float acc = 0.f;
    for (int q = 0; q < nsplit; ++q) acc += g0[(long long)q * kOB * kOB + (32 * warp + i) * kOB + 32 * warp + lane];
    G[warp][i][lane] = acc;
  }
  taus[warp][lane] = lane < jmax ? tau[(long long)b * tau_bstride + k0 + 32 * warp + lane] : 0.f;
  __syncwarp();
  larft_inverse_warp(T[warp], G[warp], taus[warp], jmax);
  __syncwarp();
  for (int i = 0; i < 32; ++i) out[i * 32 + lane] = T[warp][i][lane];
}

// C = I for each matrix of a batch x n x n array (n % 4 == 0, 16-byte aligned rows).
__global__ void set_identity_kernel(float* __restrict__ C, long long batch, int n) {
  const long long quads = batch * (long long)n * n / 4;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < quads;
       q += (long long)gridDim.x * blockDim.x) {
    const long long e = 4 * q;
    const long long within = e % ((long long)n * n);
    const int r = (int)(within / n), c = (int)(within % n);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r >= c && r < c + 4) (&v.x)[r - c] = 1.f;
    reinterpret_cast<float4*>(C)[q] = v;
  }
}

}  // namespace qrb200
