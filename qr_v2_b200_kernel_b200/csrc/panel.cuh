// Householder panel factorisation (larfg + larf over the panel) with the LARFT T factor
// built in the same pass.
//
// One thread-block cluster of CP CTAs factors the m x w panel H[k:n, k:k+w] of one matrix.
// CTA p of the cluster holds panel rows [p*R, (p+1)*R) in registers (R = NT*RPT rows, one
// row per thread per RPT slot, all NBT columns of a row in one thread). For every column j:
//
//   1. each thread accumulates d_c = sum_{rows r > j} a[r][j] * a[r][c] for all c < NBT:
//      c > j are the dot products of the unscaled tail x_j with the trailing panel columns,
//      c == j is ||x_j||^2 and c < j are x_j . v_c, the LARFT column (V^T v_j);
//   2. d is reduced over the CTA (warp transposed butterfly + one shared-memory pass) and,
//      for CP > 1, over the cluster through distributed shared memory (one cluster barrier
//      per column, partial slots double-buffered by column parity);
//   3. every thread derives beta, tau and the scale 1/(alpha - beta) from alpha = a[j][j]
//      and ||x||^2 (reference arithmetic, submission.py:91-107), then applies
//      a[r][c] -= tau * v_r * (a[j][c] + scale * d_c) to its rows (v_r = scale * a[r][j],
//      v_j = 1), which is the rank-1 update of submission.py:100-103 with v^T a_c
//      assembled from the reduced dots;
//   4. one warp of CTA 0 appends column j of T:
//      T[:j, j] = -tau_j T[:j, :j] z, z_c = a[j][c] + scale * d_c = v_c . v_j
//      (the LARFT recurrence of submission.py:129-137 fed by the same reduction).
//
// The panel therefore costs one block reduction (plus one cluster barrier when CP > 1) per
// reflector, reads and writes the panel once, and needs no separate Gram (V^T V) pass.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace qrb200 {

namespace cg = cooperative_groups;

struct PanelParams {
  const float* src;      // panel source matrix batch (A for the first panel, else H)
  long long src_bstride; // elements between matrices of src
  float* H;              // output batch, n x n row-major, contiguous
  float* tau;            // batch x n
  float* T;              // batch x NBT x NBT upper-triangular T factors (may be null)
  int n;                 // matrix order
  int k;                 // first panel column (== first panel row)
  int w;                 // panel width, <= NBT
};

template <int NBT, int NT, int RPT, bool HAS_T>
__global__ void __launch_bounds__(NT, 1) panel_factor_kernel(PanelParams P) {
  constexpr int NW = NT / 32;
  constexpr int Q = NBT / 32;
  constexpr int R = NT * RPT;
  static_assert(NBT % 32 == 0 && NT % 32 == 0, "shape");
  static_assert(NBT <= R, "the diagonal block must sit in the first CTA");

  __shared__ float wsum[NW][NBT];
  __shared__ float slot[2][2 * NBT];  // cluster-visible partials: [dots | row j]
  __shared__ float tot_s[2][NBT];
  __shared__ float rowj_s[2][NBT];
  constexpr int TD = HAS_T ? NBT : 1;
  __shared__ float T_s[TD][TD + 1];

  cg::cluster_group cluster = cg::this_cluster();
  const int CP = (int)cluster.num_blocks();
  const int p = (int)cluster.block_rank();
  const int bidx = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = P.n, k = P.k, w = P.w;
  const int m = n - k;
  const bool want_T = HAS_T && P.T != nullptr;
  const float* __restrict__ S = P.src + (long long)bidx * P.src_bstride;
  float* __restrict__ Hb = P.H + (long long)bidx * n * n;

  for (int i = tid; i < TD * (TD + 1); i += NT) (&T_s[0][0])[i] = 0.f;

  float a[RPT][NBT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int lr = p * R + i * NT + tid;
    if (lr < m) {
      const float* row = S + (long long)(k + lr) * n + k;
#pragma unroll
      for (int c = 0; c < NBT; ++c) a[i][c] = (c < w) ? row[c] : 0.f;
    } else {
#pragma unroll
      for (int c = 0; c < NBT; ++c) a[i][c] = 0.f;
    }
  }
  if (CP > 1) cluster.sync();  // every CTA of the cluster is running before any DSMEM access
  __syncthreads();

  const int jmax = min(w, m);
  for (int j = 0; j < jmax; ++j) {
    const int ph = j & 1;
    float d[NBT];
#pragma unroll
    for (int c = 0; c < NBT; ++c) d[c] = 0.f;
    float xj[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int lr = p * R + i * NT + tid;
      float x = 0.f;
#pragma unroll
      for (int c = 0; c < NBT; ++c) x = (c == j) ? a[i][c] : x;
      xj[i] = x;
      const float f = (lr > j) ? x : 0.f;
#pragma unroll
      for (int c = 0; c < NBT; ++c) d[c] = fmaf(f, a[i][c], d[c]);
      if (lr == j) {
#pragma unroll
        for (int c = 0; c < NBT; ++c) rowj_s[ph][c] = a[i][c];
      }
    }
    warp_transpose_reduce<NBT>(d, lane);
#pragma unroll
    for (int q = 0; q < Q; ++q) wsum[warp][lane * Q + q] = d[q];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        const int c = lane * Q + q;
        float s = 0.f;
#pragma unroll
        for (int v = 0; v < NW; ++v) s += wsum[v][c];
        if (CP == 1) {
          tot_s[ph][c] = s;
        } else {
          slot[ph][c] = s;
          slot[ph][NBT + c] = (p == 0) ? rowj_s[ph][c] : 0.f;
        }
      }
    }
    if (CP > 1) {
      cluster.sync();
      if (warp == 0) {
        const float* r0 = cluster.map_shared_rank(&slot[ph][0], 0);
#pragma unroll
        for (int q = 0; q < Q; ++q) {
          const int c = lane * Q + q;
          float s = 0.f;
          for (int qq = 0; qq < CP; ++qq) s += cluster.map_shared_rank(&slot[ph][0], qq)[c];
          tot_s[ph][c] = s;
          if (p != 0) rowj_s[ph][c] = r0[NBT + c];
        }
      }
    }
    __syncthreads();

    const float alpha = rowj_s[ph][j];
    const Reflector rf = make_reflector(alpha, tot_s[ph][j]);
    // wv[c] = v_j^T a_c for the trailing panel columns (v_j = e_j + scale * x_j).
    float wv[NBT];
#pragma unroll
    for (int c = 0; c < NBT; ++c) wv[c] = fmaf(rf.scale, tot_s[ph][c], rowj_s[ph][c]);
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int lr = p * R + i * NT + tid;
      if (lr >= j) {
        const bool diag_row = (lr == j);
        const float coef = diag_row ? rf.tau : rf.tau * rf.scale * xj[i];
        const float newj = diag_row ? rf.diag : rf.scale * xj[i];
#pragma unroll
        for (int c = 0; c < NBT; ++c) {
          if (c > j) a[i][c] = fmaf(-coef, wv[c], a[i][c]);
          if (c == j) a[i][c] = newj;
        }
      }
    }
    if (p == 0) {
      if (tid == 0) P.tau[(long long)bidx * n + k + j] = rf.tau;
      if (HAS_T && want_T && warp == NW - 1) {
        // T[i][j] = -tau_j * sum_{i <= c < j} T[i][c] * z_c ; T[j][j] = tau_j.
        // z_c = v_c . v_j = a[j][c] + scale * d_c for c < j, which is wv[c].
        for (int i = lane; i <= j; i += 32) {
          float acc = 0.f;
#pragma unroll
          for (int c = 0; c < NBT; ++c)
            if (c >= i && c < j) acc = fmaf(T_s[i % TD][c % TD], wv[c], acc);
          T_s[i % TD][j % TD] = (i == j) ? rf.tau : -rf.tau * acc;
        }
      }
    }
  }

#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int lr = p * R + i * NT + tid;
    if (lr < m) {
      float* row = Hb + (long long)(k + lr) * n + k;
#pragma unroll
      for (int c = 0; c < NBT; ++c)
        if (c < w) row[c] = a[i][c];
    }
  }
  // Columns of a row that lies above the panel but inside the matrix are written by the
  // previous panels' trailing updates; nothing else to store here.
  if (HAS_T && want_T && p == 0) {
    __syncthreads();
    float* Tb = P.T + (long long)bidx * NBT * NBT;
    for (int i = tid; i < NBT * NBT; i += NT) Tb[i] = T_s[(i / NBT) % TD][(i % NBT) % TD];
  }
  if (CP > 1) cluster.sync();  // keep this CTA's shared memory alive for remote readers
}

}  // namespace qrb200
