// Householder panel factorisation (larfg + larf over the panel) with the LARFT T factor
// built in the same pass.
//
// Layout: one warp per panel column. A CTA has 32 warps; warp c owns panel column c, and
// its lanes hold the CTA's rows of that column, lane l holding local rows l + 32 i
// (i < RPL). A thread-block cluster of CP CTAs covers a panel taller than 32 * RPL rows,
// CTA p holding rows [p*R, (p+1)*R), R = 32 * RPL.
//
// Reflector j (the loop over columns is a runtime loop: the body is a few hundred bytes):
//   (a) warp j, whose column already carries every earlier reflector, publishes the
//       unscaled tail x_j (rows below j, zero elsewhere) in shared memory; lane j of every
//       warp publishes its row-j value a[j][c];
//   (b) __syncthreads;
//   (c) every warp c forms d_c = x_j . a_c over its rows and reduces it across the warp:
//       c > j gives the trailing dots, c == j gives ||x_j||^2 and c < j gives x_j . v_c,
//       the LARFT column; for CP > 1 the per-CTA sums are added across the cluster through
//       distributed shared memory after ONE cluster barrier;
//   (d) every warp derives beta, tau and scale = 1/(alpha - beta) from alpha = a[j][j] and
//       ||x_j||^2 (the reference arithmetic, submission.py:91-107); warps c > j apply
//       a_c -= tau * v_j (v_j^T a_c) with v_j^T a_c = a[j][c] + scale * d_c (the rank-1
//       update of submission.py:100-103); warp j scales its tail into v_j, stores tau and
//       appends column j of T: T[i][j] = -tau_j sum_{i<=c<j} T[i][c] z_c,
//       z_c = v_c^T v_j = a[j][c] + scale * d_c (LARFT, submission.py:129-137).
// Shared slots are double-buffered by the parity of j, so each reflector costs two CTA
// barriers (one of them the cluster barrier when CP > 1) and no extra Gram pass.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace qrb200 {

namespace cg = cooperative_groups;

constexpr int kPanelW = 32;        // panel width (columns) == warps per panel CTA
constexpr int kPanelThreads = 1024;

struct PanelParams {
  const float* src;       // panel source matrix batch (A for the first panel, else H)
  long long src_bstride;  // elements between matrices of src
  float* H;               // output batch, n x n row-major, contiguous
  float* tau;             // batch x n
  float* T;               // 32 x 32 upper-triangular T factors, t_bstride apart (may be null)
  int n;                  // matrix order
  int k;                  // first panel column (== first panel row)
  int w;                  // panel width, <= 32
  long long t_bstride;    // elements between the T factors of consecutive matrices
};

// Coalesced panel transfer through shared memory. The panel rows [r0, r0 + rows) x columns
// [k, k + w) of a row-major matrix are moved with 16-byte row segments and kept transposed in
// `stage` (stage[c * ld + r], ld = rows + 1, so both the transposing writes and the per-column
// reads are bank-conflict free); each warp then takes its columns from shared memory instead
// of issuing one 4-byte load per row.
// ROWS and NT (the threads sharing the copy, == blockDim.x) are compile-time, so every thread
// issues up to eight 16-byte loads before its first shared-memory store: a panel load costs
// one memory latency per eight pieces instead of one per piece.
template <int ROWS, int NT>
__device__ __forceinline__ void panel_stage_in(const float* __restrict__ S, int n, int k, int r0, int rows_valid,
                                               int w, float* stage) {
  constexpr int LD = ROWS + 1, TOTAL = ROWS * 8;
  constexpr int ITERS = (TOTAL + NT - 1) / NT;
  constexpr int B = ITERS < 8 ? ITERS : 8;
  const bool vec = ((n & 3) == 0) && ((k & 3) == 0) && ((reinterpret_cast<uintptr_t>(S) & 15u) == 0);
#pragma unroll
  for (int b0 = 0; b0 < ITERS; b0 += B) {
    float4 x[B];
#pragma unroll
    for (int u = 0; u < B; ++u) {
      const int idx = (b0 + u) * NT + (int)threadIdx.x;
      const int r = idx >> 3, c = 4 * (idx & 7);
      x[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (b0 + u < ITERS && idx < TOTAL && r < rows_valid && c < w) {
        const float* src = S + (long long)(k + r0 + r) * n + k + c;
        if (vec && c + 3 < w) {
          x[u] = *reinterpret_cast<const float4*>(src);
        } else {
          x[u].x = src[0];
          x[u].y = (c + 1 < w) ? src[1] : 0.f;
          x[u].z = (c + 2 < w) ? src[2] : 0.f;
          x[u].w = (c + 3 < w) ? src[3] : 0.f;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < B; ++u) {
      const int idx = (b0 + u) * NT + (int)threadIdx.x;
      if (b0 + u < ITERS && idx < TOTAL) {
        const int r = idx >> 3, c = 4 * (idx & 7);
        stage[(c + 0) * LD + r] = x[u].x;
        stage[(c + 1) * LD + r] = x[u].y;
        stage[(c + 2) * LD + r] = x[u].z;
        stage[(c + 3) * LD + r] = x[u].w;
      }
    }
  }
}
// t0 / nthreads: this thread's index among the nthreads threads that share the copy.
__device__ __forceinline__ void panel_stage_out(float* __restrict__ Hb, int n, int k, int r0, int rows,
                                                int rows_valid, int w, const float* stage, int nthreads,
                                                int t0 = -1) {
  const int ld = rows + 1;
  const bool vec = ((n & 3) == 0) && ((k & 3) == 0) && ((reinterpret_cast<uintptr_t>(Hb) & 15u) == 0);
  for (int idx = (t0 < 0 ? (int)threadIdx.x : t0); idx < rows * 8; idx += nthreads) {
    const int r = idx >> 3, q = idx & 7, c = 4 * q;
    if (r >= rows_valid || c >= w) continue;
    const float4 x = make_float4(stage[(c + 0) * ld + r], stage[(c + 1) * ld + r], stage[(c + 2) * ld + r],
                                 stage[(c + 3) * ld + r]);
    float* dst = Hb + (long long)(k + r0 + r) * n + k + c;
    if (vec && c + 3 < w) {
      *reinterpret_cast<float4*>(dst) = x;
    } else {
      dst[0] = x.x;
      if (c + 1 < w) dst[1] = x.y;
      if (c + 2 < w) dst[2] = x.z;
      if (c + 3 < w) dst[3] = x.w;
    }
  }
}

template <int RPL>
struct PanelShared {
  float xs[2][32 * RPL];                // broadcast tail x_j of the pivot column
  __align__(16) float rowj[2][32];      // row j of the panel
  __align__(16) float dsum[2][32];      // per-column dot totals
  __align__(16) float slot[2][64];      // cluster-visible partials: [column dots | pivot row]
  float tau[32];           // reflector coefficients (CTA 0)
  float G[32][33];         // G[c][j] = v_c . v_j, c < j (CTA 0)
  float T[32][33];         // T factor (CTA 0)
};

// T of a 32-column panel by one warp from the Gram entries G[c][i] = v_c . v_i (c < i) and
// tau: T^-1 = diag(1/tau) + striu(V^T V) (the compact-WY factor of H_0 .. H_{k-1}, cf. the LARFT
// recurrence of submission.py:129-137, which builds the same T column by column). Lane j solves
// U t = e_j by column-oriented back substitution, t_i = tau_i (e_j - sum_{c>i} U_ic t_c)_i, so
// no reciprocal is formed and tau_i = 0 (an identity reflector) gives a zero row and column.
__device__ __forceinline__ void larft_inverse_warp(float (&T)[32][33], const float (&G)[32][33], const float* tau,
                                                   int jmax) {
  const int j = threadIdx.x & 31;
  float r[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) r[i] = (i == j) ? 1.f : 0.f;
#pragma unroll
  for (int i = 31; i >= 0; --i) {
    float ti = 0.f;
    if (i < jmax) {
      ti = (i <= j) ? r[i] * tau[i] : 0.f;
#pragma unroll
      for (int c = 0; c < i; ++c) r[c] = fmaf(-G[c][i], ti, r[c]);
    }
    T[i][j] = ti;
  }
}

// Factor the panel whose column `warp` this warp holds in a[] (rows lane + 32 i of the
// CTA's row block, p = cluster rank). All threads of the CTA -- and of the cluster when
// cluster_size > 1 -- must call this with the same (w, jmax).
template <int RPL, bool HAS_T>
__device__ __forceinline__ void factor_panel_cols(float (&a)[RPL], const int w, const int jmax,
                                                  PanelShared<RPL>& sh, float* __restrict__ tau_out,
                                                  const int cluster_size, const int p) {
  const int lane = threadIdx.x & 31, c = threadIdx.x >> 5;
  const int lr0 = p * 32 * RPL + lane;  // local panel row of a[0]
  cg::cluster_group cluster = cg::this_cluster();

  for (int j = 0; j < jmax; ++j) {
    const int ph = j & 1;
    // (a) publish x_j and row j.
    if (c == j) {
#pragma unroll
      for (int i = 0; i < RPL; ++i) sh.xs[ph][lane + 32 * i] = (lr0 + 32 * i > j) ? a[i] : 0.f;
    }
    if (p == 0 && lane == j) sh.rowj[ph][c] = a[0];
    __syncthreads();
    // (c) d_c = x_j . a_c
    float x[RPL];
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < RPL; ++i) {
      x[i] = sh.xs[ph][lane + 32 * i];
      d = fmaf(x[i], a[i], d);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) d += __shfl_xor_sync(kFullMask, d, o);
    float xn2, alpha, ajc;
    if (cluster_size == 1) {
      if (lane == 0) sh.dsum[ph][c] = d;
      __syncthreads();
      xn2 = sh.dsum[ph][j];
      alpha = sh.rowj[ph][j];
      ajc = sh.rowj[ph][c];
    } else {
      if (lane == 0) {
        sh.slot[ph][c] = d;
        sh.slot[ph][32 + c] = (p == 0) ? sh.rowj[ph][c] : 0.f;
      }
      cluster.sync();
      // One warp gathers the cluster in a single DSMEM round trip: lane l reads columns
      // 16 (l % 2) .. +15 of CTA l / 2's partial dots (four 16-byte loads; clusters of up to 16
      // CTAs), the sums over CTAs are formed with four xor shuffles, and lanes 0..1 also fetch
      // the pivot row from CTA 0. Totals are published in this CTA's shared memory.
      if (c == 0) {
        const int q = lane >> 1, cg = lane & 1;
        float4 v[4], pr[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) v[t] = pr[t] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q < cluster_size) {
          const float* rq = cluster.map_shared_rank(&sh.slot[ph][0], q) + 16 * cg;
#pragma unroll
          for (int t = 0; t < 4; ++t) v[t] = *reinterpret_cast<const float4*>(rq + 4 * t);
        }
        if (q == 0) {
          const float* r0 = cluster.map_shared_rank(&sh.slot[ph][0], 0) + 32 + 16 * cg;
#pragma unroll
          for (int t = 0; t < 4; ++t) pr[t] = *reinterpret_cast<const float4*>(r0 + 4 * t);
        }
#pragma unroll
        for (int o = 2; o <= 16; o <<= 1) {
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            v[t].x += __shfl_xor_sync(kFullMask, v[t].x, o);
            v[t].y += __shfl_xor_sync(kFullMask, v[t].y, o);
            v[t].z += __shfl_xor_sync(kFullMask, v[t].z, o);
            v[t].w += __shfl_xor_sync(kFullMask, v[t].w, o);
          }
        }
        if (q == 0) {
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            *reinterpret_cast<float4*>(&sh.dsum[ph][16 * cg + 4 * t]) = v[t];
            *reinterpret_cast<float4*>(&sh.rowj[ph][16 * cg + 4 * t]) = pr[t];
          }
        }
      }
      __syncthreads();
      d = sh.dsum[ph][c];
      xn2 = sh.dsum[ph][j];
      alpha = sh.rowj[ph][j];
      ajc = sh.rowj[ph][c];
    }
    // (d) reflector and updates.
    const Reflector rf = make_reflector(alpha, xn2);
    if (c > j && c < w) {
      const float wc = fmaf(rf.scale, d, ajc);
      const float cx = rf.tau * rf.scale * wc;
#pragma unroll
      for (int i = 0; i < RPL; ++i) {
        const int lr = lr0 + 32 * i;
        if (lr > j) a[i] = fmaf(-cx, x[i], a[i]);
        else if (lr == j) a[i] = fmaf(-rf.tau, wc, a[i]);
      }
    } else if (c == j) {
#pragma unroll
      for (int i = 0; i < RPL; ++i) {
        const int lr = lr0 + 32 * i;
        if (lr > j) a[i] *= rf.scale;
        else if (lr == j) a[i] = rf.diag;
      }
      if (p == 0 && lane == 0) {
        tau_out[j] = rf.tau;
        sh.tau[j] = rf.tau;
      }
    } else if (HAS_T && c < j && p == 0 && lane == 0) {
      sh.G[c][j] = fmaf(rf.scale, d, ajc);  // v_c . v_j = a[j][c] + scale * (x_j . v_c)
    }
  }
  if (HAS_T && p == 0) {
    __syncthreads();
    if (c == 0) larft_inverse_warp(sh.T, sh.G, sh.tau, jmax);
  }
}

// Single-CTA panel, "owner computes" form: used when the whole panel fits one CTA.
// NW = 32 / CPW warps; warp g owns columns g + NW q (q < CPW), interleaved so that the
// still-active columns stay spread over all warps. Reflector j:
//   the owner warp (j % NW) reduces ||x_j||^2 over its column, computes beta, tau and the
//   scale once, scales its tail into v_j and publishes v_j (unit at row j, zero above) and
//   tau in shared memory;  ONE __syncthreads;  every warp then forms v_j^T a_c for its
//   active columns c > j (warp all-reduce) and applies a_c -= tau (v_j^T a_c) v_j, and for
//   its finished columns c < j records G[c][j] = v_c^T v_j for the T factor.
// T is assembled after the loop by the LARFT recurrence over G (one warp).
template <int RPL, int CPW>
struct OwnerShared {
  float v[2][32 * RPL];
  float tau[32];
  float G[32][33];
  float T[32][33];
  int tiny;  // a column's alpha^2 + ||x||^2 fell below 2^-100
  int amax;  // bits of the panel's largest |entry| (rescaling pass only)
};

template <int RPL, int CPW, bool HAS_T>
__device__ __forceinline__ void factor_panel_owner(float (&a)[CPW][RPL], const int w, const int jmax,
                                                   OwnerShared<RPL, CPW>& sh, float* __restrict__ tau_out) {
  constexpr int NW = 32 / CPW;
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  for (int j = 0; j < jmax; ++j) {
    const int ph = j & 1;
    if (g == j % NW) {
      const int oq = j / NW;
      float x[RPL];
#pragma unroll
      for (int i = 0; i < RPL; ++i) {
        float t = a[0][i];
#pragma unroll
        for (int q = 1; q < CPW; ++q) t = (q == oq) ? a[q][i] : t;
        x[i] = t;
      }
      // Four independent partial sums shorten the dependent FMA chain.
      float sp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < RPL; ++i) sp[i & 3] = (lane + 32 * i > j) ? fmaf(x[i], x[i], sp[i & 3]) : sp[i & 3];
      float s = (sp[0] + sp[1]) + (sp[2] + sp[3]);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(kFullMask, s, o);
      const float alpha = __shfl_sync(kFullMask, x[0], j);
      const Reflector rf = make_reflector_fast(alpha, s);
      if (lane == 0 && fmaf(alpha, alpha, s) < kRescaleDown) sh.tiny = 1;  // see panel_owner_kernel
#pragma unroll
      for (int i = 0; i < RPL; ++i) {
        const int lr = lane + 32 * i;
        const float vi = (lr > j) ? x[i] * rf.scale : (lr == j ? 1.f : 0.f);
        sh.v[ph][lr] = vi;
        const float nx = (lr > j) ? vi : (lr == j ? rf.diag : x[i]);
#pragma unroll
        for (int q = 0; q < CPW; ++q)
          if (q == oq) a[q][i] = nx;
      }
      if (lane == 0) {
        sh.tau[j] = rf.tau;
        tau_out[j] = rf.tau;
      }
    }
    __syncthreads();
    const float tj = sh.tau[j];
    float v[RPL];
#pragma unroll
    for (int i = 0; i < RPL; ++i) v[i] = sh.v[ph][lane + 32 * i];
    float dq[CPW];
#pragma unroll
    for (int q = 0; q < CPW; ++q) {
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int i = 0; i < RPL; i += 2) {
        d0 = fmaf(v[i], a[q][i], d0);
        if (i + 1 < RPL) d1 = fmaf(v[i + 1], a[q][i + 1], d1);
      }
      dq[q] = d0 + d1;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
      for (int q = 0; q < CPW; ++q) dq[q] += __shfl_xor_sync(kFullMask, dq[q], o);
#pragma unroll
    for (int q = 0; q < CPW; ++q) {
      const int c = g + NW * q;
      if (c > j && c < w) {
        const float f = tj * dq[q];
#pragma unroll
        for (int i = 0; i < RPL; ++i) a[q][i] = fmaf(-f, v[i], a[q][i]);
      } else if (HAS_T && c < j) {
        if (lane == 0) sh.G[c][j] = dq[q];
      }
    }
  }
  // T (from sh.G and sh.tau) is built by the caller, after its next CTA barrier.
}

// Two CTAs per SM for the 8-warp shape (<= 128 registers), so one CTA's reflector latency
// overlaps another matrix's panel.
template <int RPL, int CPW, bool HAS_T>
__global__ void __launch_bounds__(32 * (32 / CPW), (CPW >= 4 ? (RPL <= 12 ? 3 : 2) : 1)) panel_owner_kernel(PanelParams P) {
  constexpr int NW = 32 / CPW;
  __shared__ OwnerShared<RPL, CPW> sh;
  const int bidx = blockIdx.y;
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int n = P.n, k = P.k, w = P.w;
  const int m = n - k;
  constexpr int R = 32 * RPL;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  float* stage = reinterpret_cast<float*>(smem_raw);  // 32 x (R + 1) floats
  const float* __restrict__ S = P.src + (long long)bidx * P.src_bstride;
  float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  if (HAS_T)
    for (int i = threadIdx.x; i < 32 * 33; i += 32 * NW) (&sh.T[0][0])[i] = 0.f;
  if (threadIdx.x == 0) {
    sh.tiny = 0;
    sh.amax = 0;
  }
  panel_stage_in<R, 32 * NW>(S, n, k, 0, min(R, m), w, stage);
  __syncthreads();
  float a[CPW][RPL];
#pragma unroll
  for (int q = 0; q < CPW; ++q) {
    const int c = g + NW * q;
#pragma unroll
    for (int i = 0; i < RPL; ++i) a[q][i] = stage[c * (R + 1) + lane + 32 * i];
  }
  __syncthreads();
  factor_panel_owner<RPL, CPW, HAS_T>(a, w, min(w, m), sh, P.tau + (long long)bidx * n + k);
  __syncthreads();  // every warp is done reading the stage; sh.tiny is final
  if (sh.tiny) {
    // A squared norm fell below 2^-100, where the squares lose digits to the subnormal range
    // (Q would lose orthogonality). Factor the panel again from its staged input scaled by a
    // power of two that brings its largest entry near 1, then scale R back: V and tau are
    // scale invariant and R scales exactly, so this is LAPACK's small-column rescaling done
    // once per panel. Uniformly small panels (a tiny matrix) are covered; a panel whose
    // largest entry is ordinary keeps its result. Ordinary inputs never enter this branch.
    float mx = 0.f;
#pragma unroll
    for (int q = 0; q < CPW; ++q)
#pragma unroll
      for (int i = 0; i < RPL; ++i) mx = fmaxf(mx, fabsf(stage[(g + NW * q) * (R + 1) + lane + 32 * i]));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, o));
    if (lane == 0) atomicMax(&sh.amax, __float_as_int(mx));  // non-negative: int order = float order
    __syncthreads();
    const float M = __int_as_float(sh.amax);
    if (M > 0.f && M < 0x1p-40f) {
      int ex;
      frexpf(M, &ex);  // M = f 2^ex, f in [0.5, 1)
      const int up = min(-ex, 126);
      const float scl = ldexpf(1.f, up), inv = ldexpf(1.f, -up);
#pragma unroll
      for (int q = 0; q < CPW; ++q)
#pragma unroll
        for (int i = 0; i < RPL; ++i) a[q][i] = stage[(g + NW * q) * (R + 1) + lane + 32 * i] * scl;
      __syncthreads();
      factor_panel_owner<RPL, CPW, HAS_T>(a, w, min(w, m), sh, P.tau + (long long)bidx * n + k);
#pragma unroll
      for (int q = 0; q < CPW; ++q)
#pragma unroll
        for (int i = 0; i < RPL; ++i)
          if (lane + 32 * i <= g + NW * q) a[q][i] *= inv;  // R: rows up to the diagonal
      __syncthreads();
    }
  }
#pragma unroll
  for (int q = 0; q < CPW; ++q) {
    const int c = g + NW * q;
#pragma unroll
    for (int i = 0; i < RPL; ++i) stage[c * (R + 1) + lane + 32 * i] = a[q][i];
  }
  __syncthreads();  // staged panel, Gram entries and tau are complete
  if (HAS_T && g == 0) {
    // Warp 0 builds and stores T while the other warps write the panel.
    larft_inverse_warp(sh.T, sh.G, sh.tau, min(w, m));
    __syncwarp();
    if (P.T != nullptr) {
      float* Tb = P.T + (long long)bidx * P.t_bstride;
      for (int i = lane; i < 32 * 32; i += 32) Tb[i] = sh.T[i / 32][i % 32];
    }
  } else {
    const int t0 = HAS_T ? (int)threadIdx.x - 32 : (int)threadIdx.x;
    panel_stage_out(Hb, n, k, 0, R, min(R, m), w, stage, HAS_T ? 32 * NW - 32 : 32 * NW, t0);
  }
}

template <int RPL, bool HAS_T>
__global__ void __launch_bounds__(kPanelThreads) panel_factor_kernel(PanelParams P) {
  constexpr int R = 32 * RPL;
  __shared__ PanelShared<RPL> sh;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  float* stage = reinterpret_cast<float*>(smem_raw);  // 32 x (R + 1) floats
  cg::cluster_group cluster = cg::this_cluster();
  const int CP = (int)cluster.num_blocks();
  const int p = (int)cluster.block_rank();
  const int bidx = blockIdx.y;
  const int lane = threadIdx.x & 31, c = threadIdx.x >> 5;
  const int n = P.n, k = P.k, w = P.w;
  const int m = n - k;
  const int r0 = p * R;
  const int rows_valid = max(0, min(R, m - r0));
  const float* __restrict__ S = P.src + (long long)bidx * P.src_bstride;
  float* __restrict__ Hb = P.H + (long long)bidx * n * n;

  if (HAS_T)
    for (int i = threadIdx.x; i < 32 * 33; i += kPanelThreads) (&sh.T[0][0])[i] = 0.f;
  panel_stage_in<R, kPanelThreads>(S, n, k, r0, rows_valid, w, stage);
  __syncthreads();
  float a[RPL];
#pragma unroll
  for (int i = 0; i < RPL; ++i) a[i] = stage[c * (R + 1) + lane + 32 * i];
  if (CP > 1) cluster.sync();  // every CTA of the cluster runs before any DSMEM access
  __syncthreads();

  factor_panel_cols<RPL, HAS_T>(a, w, min(w, m), sh, P.tau + (long long)bidx * n + k, CP, p);

  __syncthreads();
#pragma unroll
  for (int i = 0; i < RPL; ++i) stage[c * (R + 1) + lane + 32 * i] = a[i];
  __syncthreads();
  panel_stage_out(Hb, n, k, r0, R, rows_valid, w, stage, kPanelThreads);
  if (HAS_T && P.T != nullptr && p == 0) {
    float* Tb = P.T + (long long)bidx * P.t_bstride;
    for (int i = threadIdx.x; i < 32 * 32; i += kPanelThreads) Tb[i] = sh.T[i / 32][i % 32];
  }
  if (CP > 1) cluster.sync();  // keep this CTA's shared memory alive for remote readers
}

template <int RPL>
constexpr size_t panel_stage_bytes() { return (size_t)32 * (32 * RPL + 1) * sizeof(float); }

}  // namespace qrb200
