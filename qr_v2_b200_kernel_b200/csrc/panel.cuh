// Householder panel factorisation (larfg + larf over a panel of at most 32 columns) with the
// LARFT T factor, one CTA per panel of up to 512 rows: the "owner computes" panel
// (panel_owner_kernel) of the two-level schedule, plus the pieces the factor-warp and cluster
// panels share (coalesced staging of the panel through shared memory, the one-warp T).
//
// Reflector j (reference arithmetic, submission.py:91-107 for larfg, :100-103 for the rank-1
// update, :129-137 for LARFT): beta = -sign(alpha) ||(alpha, x)||, tau = (beta - alpha)/beta,
// v = (1, x / (alpha - beta)); every later column c gets a_c -= tau v (v^T a_c).
#pragma once

#include "common.cuh"

namespace qrb200 {

constexpr int kPanelW = 32;        // panel width (columns) == warps per panel CTA

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
                                                   OwnerShared<RPL, CPW>& sh) {
  constexpr int NW = 32 / CPW;
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  // Reflector j = NW oq + jg is owned by warp jg as its register column oq. The loop over oq is
  // unrolled, so the owner's column and, for every warp, whether each of its columns lies left
  // of, at or right of j are compile-time facts except within the group oq itself.
#pragma unroll
  for (int oq = 0; oq < CPW; ++oq) {
#pragma unroll 1
    for (int jg = 0; jg < NW; ++jg) {
      const int j = NW * oq + jg;
      if (j >= jmax) break;
      const int ph = j & 1;
      if (g == jg) {
        // Four independent partial sums shorten the dependent FMA chain.
        float sp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < RPL; ++i)
          sp[i & 3] = (lane + 32 * i > j) ? fmaf(a[oq][i], a[oq][i], sp[i & 3]) : sp[i & 3];
        float s = (sp[0] + sp[1]) + (sp[2] + sp[3]);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(kFullMask, s, o);
        const float alpha = __shfl_sync(kFullMask, a[oq][0], j);
        const Reflector rf = make_reflector_fast(alpha, s);
        if (lane == 0 && fmaf(alpha, alpha, s) < kRescaleDown) sh.tiny = 1;  // see panel_owner_kernel
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const int lr = lane + 32 * i;
          const float vi = (lr > j) ? a[oq][i] * rf.scale : (lr == j ? 1.f : 0.f);
          sh.v[ph][lr] = vi;
          a[oq][i] = (lr > j) ? vi : (lr == j ? rf.diag : a[oq][i]);
        }
        if (lane == 0) sh.tau[j] = rf.tau;  // to global memory after the loop
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
        // q > oq: c > j; q < oq: c < j; q == oq: decided by g against jg.
        const bool right = (q > oq) || (q == oq && g > jg);
        const bool left = (q < oq) || (q == oq && g < jg);
        if (right && c < w) {
          const float f = tj * dq[q];
#pragma unroll
          for (int i = 0; i < RPL; ++i) a[q][i] = fmaf(-f, v[i], a[q][i]);
        } else if (HAS_T && left) {
          if (lane == 0) sh.G[c][j] = dq[q];
        }
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
  factor_panel_owner<RPL, CPW, HAS_T>(a, w, min(w, m), sh);
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
      factor_panel_owner<RPL, CPW, HAS_T>(a, w, min(w, m), sh);
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
  if (g == 0 && lane < min(w, m)) P.tau[(long long)bidx * n + k + lane] = sh.tau[lane];
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

template <int RPL>
constexpr size_t panel_stage_bytes() { return (size_t)32 * (32 * RPL + 1) * sizeof(float); }

}  // namespace qrb200
