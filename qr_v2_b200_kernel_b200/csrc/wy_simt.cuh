// Compact-WY trailing update on CUDA cores (FP32 FFMA), three launches:
//
//   wy_vtc_kernel : Wp[s] = V_s^T C_s      row-split partial products (NB x nc per split)
//   wy_tw_kernel  : W2    = T^T sum_s Wp[s] (NB x nc)
//   wy_upd_kernel : C    <- C - V W2       (m x nc)
//
// so that C <- (I - V T^T V^T) C = Q_panel^T C, the application of
// milestones/01_eager_official123203us.py:102-107 and submission.py:453-480.
// V is read implicitly from the factored panel in H (unit diagonal, zeros above it);
// C is read from `src` (A for the first panel, H afterwards) and always written to H.
// This is the exact-FP32 path; the tensor-core path replaces the first and last GEMM.
#pragma once

#include "common.cuh"

namespace qrb200 {

struct WyParams {
  const float* src;       // trailing-matrix source (A for the first panel, else H)
  long long src_bstride;  // elements between matrices of src
  float* H;               // output batch (n x n row-major, contiguous)
  const float* T;         // T factors, t_bstride elements apart (w x w, row stride w)
  long long t_bstride;
  float* Wp;              // partial products V^T C of the row splits
  float* W2;              // T^T V^T C
  int n, k, w;            // block reflector: rows/columns start at k, width w
  int cend;               // trailing columns updated: [k + w, cend)
  int nsplit;             // row splits of the V^T C product
  int rows_per_split;     // multiple of 32
  int ncmax;              // leading dimension of Wp / W2 (>= cend - k - w)
  int coff;               // first trailing column (relative to k + w) of this launch (tile-aligned
                          // for the 128-wide kernels)
  // C outside H (tc_vtcw_pipe_kernel only): row stride of src and the column of src that holds
  // trailing column 0. ldc == 0: C is in the matrix itself (row stride n, column k + w).
  int ldc, ccol;
};

// V[r][c] of the panel starting at (k, k): unit lower trapezoid stored in H.
__device__ __forceinline__ float load_v(const float* __restrict__ Hb, int n, int k, int w, int r, int c) {
  if (c >= w) return 0.f;
  if (r > c) return Hb[(long long)(k + r) * n + k + c];
  return (r == c) ? 1.f : 0.f;
}

// Tile: 64 trailing columns x NB rows of W; 256 threads, each 8 W-rows of one column.
template <int NB>
__global__ void __launch_bounds__(256) wy_vtc_kernel(WyParams P) {
  static_assert(NB == 32, "tile assumes NB == 32");
  __shared__ float Vs[32][NB + 1];
  __shared__ float Cs[32][64 + 1];
  const int bidx = blockIdx.z, split = blockIdx.y;
  const int n = P.n, k = P.k, w = P.w, m = n - k, nc = P.cend - k - w;
  const int col0 = P.coff + blockIdx.x * 64;
  const float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  const int tid = threadIdx.x;
  const int tc = tid & 63, tr = (tid >> 6) * 8;
  const int r_begin = split * P.rows_per_split;
  const int r_end = min(m, r_begin + P.rows_per_split);
  float acc[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) acc[q] = 0.f;
  for (int r0 = r_begin; r0 < r_end; r0 += 32) {
    for (int e = tid; e < 32 * NB; e += 256) {
      const int rr = e / NB, cc = e % NB, r = r0 + rr;
      Vs[rr][cc] = (r < r_end) ? load_v(Hb, n, k, w, r, cc) : 0.f;
    }
    for (int e = tid; e < 32 * 64; e += 256) {
      const int rr = e / 64, cc = e % 64, r = r0 + rr, col = col0 + cc;
      Cs[rr][cc] = (r < r_end && col < nc) ? Sb[(long long)(k + r) * n + k + w + col] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int rr = 0; rr < 32; ++rr) {
      const float cv = Cs[rr][tc];
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = fmaf(Vs[rr][tr + q], cv, acc[q]);
    }
    __syncthreads();
  }
  const int col = col0 + tc;
  if (col < nc) {
    float* out = P.Wp + ((long long)bidx * P.nsplit + split) * NB * P.ncmax;
#pragma unroll
    for (int q = 0; q < 8; ++q) out[(long long)(tr + q) * P.ncmax + col] = acc[q];
  }
}

// W2[i][col] = sum_{c <= i} T[c][i] * W[c][col], W = sum over splits. One column per thread.
template <int NB>
__global__ void __launch_bounds__(128) wy_tw_kernel(WyParams P) {
  __shared__ float Ts[NB][NB + 1];
  const int bidx = blockIdx.y;
  const int nc = P.cend - P.k - P.w;
  const float* Tb = P.T + (long long)bidx * P.t_bstride;
  for (int e = threadIdx.x; e < NB * NB; e += blockDim.x) Ts[e / NB][e % NB] = Tb[e];
  __syncthreads();
  const int col = P.coff + blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= nc) return;
  float wv[NB];
#pragma unroll
  for (int c = 0; c < NB; ++c) wv[c] = 0.f;
  for (int s = 0; s < P.nsplit; ++s) {
    const float* Wb = P.Wp + ((long long)bidx * P.nsplit + s) * NB * P.ncmax;
#pragma unroll
    for (int c = 0; c < NB; ++c) wv[c] += Wb[(long long)c * P.ncmax + col];
  }
  float* out = P.W2 + (long long)bidx * NB * P.ncmax;
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c <= i; ++c) acc = fmaf(Ts[c][i], wv[c], acc);
    out[(long long)i * P.ncmax + col] = acc;
  }
}

// C[r][col] -= sum_c V[r][c] W2[c][col]; 64 x 64 tile, 256 threads, 4 x 4 per thread.
template <int NB>
__global__ void __launch_bounds__(256) wy_upd_kernel(WyParams P) {
  __shared__ float Vt[NB][64 + 4];  // V transposed: Vt[c][r]
  __shared__ float Ws[NB][64 + 4];
  const int bidx = blockIdx.z;
  const int n = P.n, k = P.k, w = P.w, m = n - k, nc = P.cend - k - w;
  const int row0 = blockIdx.y * 64, col0 = P.coff + blockIdx.x * 64;
  const float* __restrict__ Hb_in = P.H + (long long)bidx * n * n;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  const float* __restrict__ W2b = P.W2 + (long long)bidx * NB * P.ncmax;
  const int tid = threadIdx.x;
  for (int e = tid; e < 64 * NB; e += 256) {
    const int rr = e / NB, cc = e % NB, r = row0 + rr;
    Vt[cc][rr] = (r < m) ? load_v(Hb_in, n, k, w, r, cc) : 0.f;
  }
  for (int e = tid; e < NB * 64; e += 256) {
    const int cc = e / 64, jj = e % 64, col = col0 + jj;
    Ws[cc][jj] = (col < nc) ? W2b[(long long)cc * P.ncmax + col] : 0.f;
  }
  __syncthreads();
  const int tx = (tid & 15) * 4, ty = (tid >> 4) * 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int jx = 0; jx < 4; ++jx) acc[i][jx] = 0.f;
#pragma unroll 8
  for (int c = 0; c < NB; ++c) {
    const float4 v = *reinterpret_cast<const float4*>(&Vt[c][ty]);
    const float4 x = *reinterpret_cast<const float4*>(&Ws[c][tx]);
    const float vv[4] = {v.x, v.y, v.z, v.w};
    const float xx[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int jx = 0; jx < 4; ++jx) acc[i][jx] = fmaf(vv[i], xx[jx], acc[i][jx]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = row0 + ty + i;
    if (r >= m) continue;
#pragma unroll
    for (int jx = 0; jx < 4; ++jx) {
      const int col = col0 + tx + jx;
      if (col < nc) {
        const long long off = (long long)(k + r) * n + k + w + col;
        Hb[off] = Sb[off] - acc[i][jx];
      }
    }
  }
}

}  // namespace qrb200
