// Single-CTA Householder panel with in-panel look-ahead (panels of up to 32 * RPL rows).
//
// Layout as in the owner-computes panel: NW = 32 / CPW warps, warp g owns columns g + NW q
// (q < CPW) and holds rows lane + 32 i (i < RPL) of each in registers. Reflector j:
//   * the raw column x_j (every earlier reflector applied) sits in a shared slot; each warp
//     reads it and forms, over the rows below j, ||x||^2 and x . a_c for its columns c, one
//     warp-wide reduction for all of them;
//   * every warp derives beta, tau and scale = 1 / (alpha - beta) from alpha = x_j[j] and
//     ||x||^2 itself (bitwise the same in every warp), so no reflector has to be broadcast;
//   * with v_j = (1, scale x) the trailing dot is v_j . a_c = a[j][c] + scale (x . a_c) and the
//     column update a_c -= tau (v_j . a_c) v_j (submission.py:100-103); for c < j the same
//     expression is the Gram entry v_c . v_j of the LARFT recurrence (submission.py:129-137);
//   * the owner of column j + 1 updates that column first and publishes it as x_{j+1} before it
//     updates its other columns, so the next reflector's reduction starts while the other
//     warps still apply reflector j.
// Hand-off through two shared slots and named barriers: FULL[s] (the publisher arrives, the
// other warps wait) and EMPTY[s] (the readers of a slot arrive, the next writer of the slot
// waits), so a reflector costs one producer-to-consumer hop instead of a CTA-wide barrier.
#pragma once

#include "panel.cuh"

namespace qrb200 {

template <int RPL>
struct LaShared {
  float x[2][32 * RPL];
  float tau[32];
  float G[32][33];
  float T[32][33];
};

constexpr int kBarFull0 = 1, kBarEmpty0 = 3;  // named barriers 1-2 (FULL), 3-4 (EMPTY)

template <int RPL, int CPW>
__device__ __forceinline__ void factor_panel_la(float (&a)[CPW][RPL], const int w, const int jmax,
                                                LaShared<RPL>& sh, float* __restrict__ tau_out) {
  constexpr int NW = 32 / CPW, NT = 32 * NW;
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  if (g == 0 && jmax > 0) {  // column 0 is final from the start
#pragma unroll
    for (int i = 0; i < RPL; ++i) sh.x[0][lane + 32 * i] = a[0][i];
    __syncwarp();
    named_arrive(kBarFull0, NT);
  }
  for (int j = 0; j < jmax; ++j) {
    const int s = j & 1;
    if (g != j % NW) named_sync(kBarFull0 + s, NT);
    float xm[RPL];
#pragma unroll
    for (int i = 0; i < RPL; ++i) xm[i] = sh.x[s][lane + 32 * i];
    const float alpha = sh.x[s][j];
    // Readers release slot s, except the warp that will write x_{j+2} into it (it waits there).
    if (!(j + 2 < jmax && g == (j + 2) % NW)) named_arrive(kBarEmpty0 + s, NT);
    if (lane <= j) xm[0] = 0.f;  // rows <= j (j < 32: all of them in register 0)
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < RPL; ++i) s2 = fmaf(xm[i], xm[i], s2);
    const bool pub = (j + 1 < jmax) && (g == (j + 1) % NW);
    const int q1 = (j + 1) / NW;
    Reflector rf;
    if (pub) {
      float d1 = 0.f;
#pragma unroll
      for (int q = 0; q < CPW; ++q)
        if (q == q1)
#pragma unroll
          for (int i = 0; i < RPL; ++i) d1 = fmaf(xm[i], a[q][i], d1);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        s2 += __shfl_xor_sync(kFullMask, s2, o);
        d1 += __shfl_xor_sync(kFullMask, d1, o);
      }
      rf = make_reflector(alpha, s2);
#pragma unroll
      for (int q = 0; q < CPW; ++q) {
        if (q != q1) continue;
        const float e = __shfl_sync(kFullMask, a[q][0], j);
        const float f = rf.tau * fmaf(rf.scale, d1, e);
        const float fs = f * rf.scale;
#pragma unroll
        for (int i = 0; i < RPL; ++i) a[q][i] = fmaf(-fs, xm[i], a[q][i]);
        if (lane == j) a[q][0] -= f;
        const int s1 = (j + 1) & 1;
        if (j + 1 >= 2) named_sync(kBarEmpty0 + s1, NT);  // readers of x_{j-1} are done
#pragma unroll
        for (int i = 0; i < RPL; ++i) sh.x[s1][lane + 32 * i] = a[q][i];
        __syncwarp();
        named_arrive(kBarFull0 + s1, NT);
      }
    } else {
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) s2 += __shfl_xor_sync(kFullMask, s2, o);
      rf = make_reflector(alpha, s2);
    }
    float d[CPW];
#pragma unroll
    for (int q = 0; q < CPW; ++q) {
      d[q] = 0.f;
      const int c = g + NW * q;
      if (c < w && c != j && !(pub && q == q1))
#pragma unroll
        for (int i = 0; i < RPL; ++i) d[q] = fmaf(xm[i], a[q][i], d[q]);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
      for (int q = 0; q < CPW; ++q) d[q] += __shfl_xor_sync(kFullMask, d[q], o);
#pragma unroll
    for (int q = 0; q < CPW; ++q) {
      const int c = g + NW * q;
      if (c >= w || (pub && q == q1)) continue;
      if (c == j) {  // the reflector itself: v tail, beta on the diagonal, tau
#pragma unroll
        for (int i = 0; i < RPL; ++i) a[q][i] = (lane + 32 * i > j) ? xm[i] * rf.scale : a[q][i];
        if (lane == j) a[q][0] = rf.diag;
        if (lane == 0) {
          sh.tau[j] = rf.tau;
          tau_out[j] = rf.tau;
        }
      } else {
        const float e = __shfl_sync(kFullMask, a[q][0], j);
        const float z = fmaf(rf.scale, d[q], e);  // v_j . a_c, or v_c . v_j for c < j
        if (c > j) {
          const float f = rf.tau * z;
          const float fs = f * rf.scale;
#pragma unroll
          for (int i = 0; i < RPL; ++i) a[q][i] = fmaf(-fs, xm[i], a[q][i]);
          if (lane == j) a[q][0] -= f;
        } else if (lane == 0) {
          sh.G[c][j] = z;
        }
      }
    }
  }
  __syncthreads();
  if (g == 0) larft_inverse_warp(sh.T, sh.G, sh.tau, jmax);
}

// One CTA per panel (m <= 32 * RPL rows), coalesced staged load and store as in
// panel_owner_kernel; always produces T (t_bstride apart) when P.T is set.
template <int RPL, int CPW>
__global__ void __launch_bounds__(32 * (32 / CPW), (CPW >= 4 ? 2 : 1)) panel_la_kernel(PanelParams P) {
  constexpr int NW = 32 / CPW, NT = 32 * NW;
  constexpr int R = 32 * RPL;
  __shared__ LaShared<RPL> sh;
  const int bidx = blockIdx.y;
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int n = P.n, k = P.k, w = P.w;
  const int m = n - k;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  float* stage = reinterpret_cast<float*>(smem_raw);  // 32 x (R + 1) floats
  const float* __restrict__ S = P.src + (long long)bidx * P.src_bstride;
  float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  for (int i = threadIdx.x; i < 32 * 33; i += NT) {
    (&sh.T[0][0])[i] = 0.f;
    (&sh.G[0][0])[i] = 0.f;
  }
  panel_stage_in<R, NT>(S, n, k, 0, min(R, m), w, stage);
  __syncthreads();
  float a[CPW][RPL];
#pragma unroll
  for (int q = 0; q < CPW; ++q) {
    const int c = g + NW * q;
#pragma unroll
    for (int i = 0; i < RPL; ++i) a[q][i] = stage[c * (R + 1) + lane + 32 * i];
  }
  factor_panel_la<RPL, CPW>(a, w, min(w, m), sh, P.tau + (long long)bidx * n + k);
#pragma unroll
  for (int q = 0; q < CPW; ++q) {
    const int c = g + NW * q;
#pragma unroll
    for (int i = 0; i < RPL; ++i) stage[c * (R + 1) + lane + 32 * i] = a[q][i];
  }
  __syncthreads();
  panel_stage_out(Hb, n, k, 0, R, min(R, m), w, stage, NT);
  if (P.T != nullptr) {
    float* Tb = P.T + (long long)bidx * P.t_bstride;
    for (int i = threadIdx.x; i < 32 * 32; i += NT) Tb[i] = sh.T[i / 32][i % 32];
  }
}

}  // namespace qrb200
