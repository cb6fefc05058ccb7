// Householder panel (m <= 32 * RPL rows, w <= 32 columns) as a factor warp fed by update warps
// -- the pipeline of small_fw.cuh applied to one 32-column panel, plus the panel's 32 x 32 T.
//
//   * warp 0 (factor warp) factors the panel in blocks of 4 columns with warp shuffles only
//     (larfg/larf, submission.py:91-107); block t arrives with V_0 .. V_{t-2} applied, the
//     factor warp applies V_{t-1}, factors, writes the block to H and publishes V_t (masked)
//     and its 4 x 4 T_t (LARFT, submission.py:129-137) in shared memory;
//   * update warps 1, 2, 3, 5, 6, 7, 9 own blocks 1 .. 7 (rows 32 q + 4 g + e of column c in
//     lane 4 g + c) and apply each V_s as it appears (compact WY, submission.py:453-480);
//     warps 4 and 8 have (almost) nothing to do, so the factor warp has its scheduler to itself;
//   * once its block is handed over, update warp u writes that block to H from shared memory
//     as soon as it is factored (the factor warp issues no global stores) and forms the Gram
//     entries V_u^T V_b as each later V_b appears (warp 4 writes block 0);
//   * warp 4 assembles T with the blocked LARFT recurrence, step b as soon as the Gram
//     entries of block column b are in (gcount[b]):
//       T[0:4b, 4b:4b+4] = -T[0:4b, 0:4b] (V_{0:4b}^T V_b) T_b      (b = 1 .. nb-1).
// Hand-offs are release/acquire counters in shared memory (vcount: V blocks out; bflag[2]:
// block held by each slot of the two-slot ring into the factor warp); every wait is bounded and
// a warp whose wait expires records a device status and leaves (there is no CTA barrier after
// the set-up).
#pragma once

#include "panel.cuh"
#include "small_fw.cuh"

namespace qrb200 {

// Volatile shared float4 load: issued where it stands, so a long unrolled loop does not hoist
// all of its loads ahead of the arithmetic (which would need a register per loaded value).
__device__ __forceinline__ float4 lds4_inorder(const float* p) {
  float4 v;
  asm volatile("ld.volatile.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

template <int RPL>
struct __align__(16) PanelFwShared {
  static constexpr int R = 32 * RPL;
  float V[8][4][R];     // masked V of every block, [block][column][row] (update warps, Gram)
  float Vr[2][R][4];    // the last two V blocks row-major (the factor warp's float4 reads)
  float B[2][R][4];     // blocks on their way to the factor warp, row-major
  float Tb[8][4][4];    // block T's
  float Rb[8][4][32];   // rows 0..31 of every factored block as written to H (R entries above V)
  float G[32][33];      // Gram entries V_a^T V_b (a < b blocks); then the T recurrence's Y
  float T[32][33];
  float tau[32];        // the factor warp's tau, written to global memory after its last block
  int vcount, bflag[2], gcount[8];
};

template <int RPL>
constexpr size_t panel_fw_smem() { return sizeof(PanelFwShared<RPL>); }

constexpr int kPanelFwWarps = 10;  // factor warp, update warps 1-3, 5-7, 9, idle 4 and 8

// Factor-warp layout, any RPL: a <- (I - V T V^T)^T a with V row-major in shared memory (one
// float4 per row), products summed with the transposed butterfly.
template <int R, int RPL>
__device__ __forceinline__ void fw_apply_rowmajor(float (&a)[4][RPL], const float (*__restrict__ Vr)[4],
                                                  const float* __restrict__ Ts) {
  const int lane = threadIdx.x & 31;
  float p[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) p[e] = 0.f;
#pragma unroll
  for (int i = 0; i < RPL; ++i) {
    const float4 v = *reinterpret_cast<const float4*>(Vr[lane + 32 * i]);
    const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int cp = 0; cp < 4; ++cp)
#pragma unroll
      for (int c = 0; c < 4; ++c) p[cp * 4 + c] = fmaf(vv[cp], a[c][i], p[cp * 4 + c]);
  }
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int o = 16 >> step, half = 8 >> step;
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int q = 0; q < half; ++q) {
      const float send = up ? p[q] : p[q + half];
      const float keep = up ? p[q + half] : p[q];
      p[q] = keep + __shfl_xor_sync(kFullMask, send, o);
    }
  }
  p[0] += __shfl_xor_sync(kFullMask, p[0], 1);
  float W[4][4];
#pragma unroll
  for (int v = 0; v < 16; ++v) W[v / 4][v % 4] = __shfl_sync(kFullMask, p[0], 2 * v);
  float Y[4][4];  // Y[cp][c] = sum_k T[k][cp] W[k][c]
#pragma unroll
  for (int cp = 0; cp < 4; ++cp)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k <= cp; ++k) acc = fmaf(Ts[k * 4 + cp], W[k][c], acc);
      Y[cp][c] = acc;
    }
#pragma unroll
  for (int i = 0; i < RPL; ++i) {
    const float4 v = *reinterpret_cast<const float4*>(Vr[lane + 32 * i]);
    const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int cp = 0; cp < 4; ++cp)
#pragma unroll
      for (int c = 0; c < 4; ++c) a[c][i] = fmaf(-vv[cp], Y[cp][c], a[c][i]);
  }
}

// Block b of the factored panel from shared memory to H: V below the diagonal, the rows
// 0..31 (R entries and the diagonal) from Rb. Lane l writes rows l + 32 i.
template <int RPL>
__device__ __forceinline__ void panel_fw_store_block(const PanelFwShared<RPL>& sh, float* __restrict__ Hp, int n,
                                                     int m, int pw, int b) {
  const int lane = threadIdx.x & 31, c0 = 4 * b;
  const bool vec = ((n & 3) == 0) && ((reinterpret_cast<uintptr_t>(Hp) & 15u) == 0) && c0 + 3 < pw;
#pragma unroll 4
  for (int i = 0; i < RPL; ++i) {
    const int r = lane + 32 * i;
    if (r >= m) break;
    float v[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) v[c] = (i == 0 && r <= c0 + c) ? sh.Rb[b][c][r] : sh.V[b][c][r];
    if (vec) {
      *reinterpret_cast<float4*>(Hp + (long long)r * n + c0) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c0 + c < pw) Hp[(long long)r * n + c0 + c] = v[c];
    }
  }
}

// Gram entries G[4 a + i][4 b + c] = V_a[:, i] . V_b[:, c] (a < b); lane 4 g + c sums rows
// 32 q + 4 g + e of column c of V_b against the four columns of V_a.
template <int RPL>
__device__ __forceinline__ void panel_fw_gram_pair(PanelFwShared<RPL>& sh, int a, int b) {
  constexpr int R = 32 * RPL, RPG = R / 8;
  const int lane = threadIdx.x & 31, g4 = 4 * (lane >> 2), cc = lane & 3;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int q = 0; q < RPG; q += 4) {
    const float4 vb = lds4_inorder(&sh.V[b][cc][8 * q + g4]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 va = lds4_inorder(&sh.V[a][i][8 * q + g4]);
      acc[i] = fmaf(va.x, vb.x, acc[i]);
      acc[i] = fmaf(va.y, vb.y, acc[i]);
      acc[i] = fmaf(va.z, vb.z, acc[i]);
      acc[i] = fmaf(va.w, vb.w, acc[i]);
    }
  }
#pragma unroll
  for (int o = 4; o <= 16; o <<= 1)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] += __shfl_xor_sync(kFullMask, acc[i], o);
  if (lane < 4)
#pragma unroll
    for (int i = 0; i < 4; ++i) sh.G[4 * a + i][4 * b + cc] = acc[i];
}

// One step of the blocked LARFT recurrence by one warp (lane r < 4b owns row r):
//   Y[r][j] = sum_l G[r][4b + l] T_b[l][j];  T[r][4b + j] = -sum_{r <= q < 4b} T[r][q] Y[q][j].
template <int RPL>
__device__ __forceinline__ void panel_fw_t_step(PanelFwShared<RPL>& sh, int b) {
  const int lane = threadIdx.x & 31;
  const bool act = lane < 4 * b;
  float y[4] = {0.f, 0.f, 0.f, 0.f};
  if (act) {
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      const float g = sh.G[lane][4 * b + l];
#pragma unroll
      for (int j = 0; j < 4; ++j) y[j] = fmaf(g, sh.Tb[b][l][j], y[j]);
    }
  }
  __syncwarp();
  if (act)
#pragma unroll
    for (int j = 0; j < 4; ++j) sh.G[lane][4 * b + j] = y[j];
  __syncwarp();
  if (act) {
    float acc[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
    for (int q = 0; q < 28; ++q) {
      if (q >= lane && q < 4 * b) {
        const float tq = sh.T[lane][q];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j][q & 1] = fmaf(tq, sh.G[q][4 * b + j], acc[j][q & 1]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) sh.T[lane][4 * b + j] = -(acc[j][0] + acc[j][1]);
  }
  __syncwarp();
}

template <int RPL>
__global__ void __launch_bounds__(32 * kPanelFwWarps) panel_fw_kernel(PanelParams P) {
  griddep_launch_wait();
  constexpr int R = 32 * RPL, RPG = R / 8;
  extern __shared__ __align__(16) unsigned char pfw_smem_raw[];
  PanelFwShared<RPL>& sh = *reinterpret_cast<PanelFwShared<RPL>*>(pfw_smem_raw);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int bidx = blockIdx.y;
  const int n = P.n, k = P.k, pw = P.w, m = n - k;
  const int jmax = min(pw, m);
  const int nb = (jmax + 3) / 4;
  const float* __restrict__ S = P.src + (long long)bidx * P.src_bstride + (long long)k * n + k;  // panel origin
  float* __restrict__ Hp = P.H + (long long)bidx * n * n + (long long)k * n + k;
  float* __restrict__ taub = P.tau + (long long)bidx * n + k;
  const bool vec = ((n & 3) == 0) && ((k & 3) == 0) &&
                   (((reinterpret_cast<uintptr_t>(P.src) | reinterpret_cast<uintptr_t>(P.H)) & 15u) == 0) &&
                   ((P.src_bstride & 3) == 0);
  if (threadIdx.x < 8) sh.gcount[threadIdx.x] = 0;
  if (threadIdx.x == 0) {
    sh.vcount = 0;
    sh.bflag[0] = sh.bflag[1] = -1;
  }
  for (int i = threadIdx.x; i < 32 * 33; i += blockDim.x) {
    (&sh.G[0][0])[i] = 0.f;
    (&sh.T[0][0])[i] = 0.f;
  }
  __syncthreads();  // the only CTA-wide barrier: after it, warps meet through the counters

  if (w == 0) {
    // ---------------- factor warp ----------------
    float a[4][RPL];
#pragma unroll
    for (int i = 0; i < RPL; ++i) {
      const int r = lane + 32 * i;
      if (vec && r < m && 3 < pw) {
        const float4 x = *reinterpret_cast<const float4*>(S + (long long)r * n);
        a[0][i] = x.x;
        a[1][i] = x.y;
        a[2][i] = x.z;
        a[3][i] = x.w;
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) a[c][i] = (r < m && c < pw) ? S[(long long)r * n + c] : 0.f;
      }
    }
    for (int t = 0; t < nb; ++t) {
      const int c0 = 4 * t;
      if (t >= 1) {
        const int sl = t & 1;
        if (!fw_wait_geq(&sh.bflag[sl], t)) return;
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const float4 x = *reinterpret_cast<const float4*>(sh.B[sl][lane + 32 * i]);
          a[0][i] = x.x;
          a[1][i] = x.y;
          a[2][i] = x.z;
          a[3][i] = x.w;
        }
        fw_apply_rowmajor<R, RPL>(a, sh.Vr[(t - 1) & 1], &sh.Tb[t - 1][0][0]);  // V_{t-1}
      }
      float Tw[4][4];
      // tau stays in shared memory: a global store here would hold up the fence of the
      // block's publication below (a fence waits for the thread's global stores).
      fw_factor_block<4, RPL, true>(a, c0, jmax, Tw, sh.tau);
      // V_t masked (rows >= 32 lie below every pivot of the panel), in both layouts.
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        sh.V[t][c][lane] = (lane > c0 + c) ? a[c][0] : (lane == c0 + c ? 1.f : 0.f);
        sh.Rb[t][c][lane] = a[c][0];
#pragma unroll
        for (int i = 1; i < RPL; ++i) sh.V[t][c][lane + 32 * i] = a[c][i];
      }
      {
        float v0[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) v0[c] = (lane > c0 + c) ? a[c][0] : (lane == c0 + c ? 1.f : 0.f);
        *reinterpret_cast<float4*>(sh.Vr[t & 1][lane]) = make_float4(v0[0], v0[1], v0[2], v0[3]);
#pragma unroll
        for (int i = 1; i < RPL; ++i)
          *reinterpret_cast<float4*>(sh.Vr[t & 1][lane + 32 * i]) = make_float4(a[0][i], a[1][i], a[2][i], a[3][i]);
      }
      if (lane == 0)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
          for (int c = 0; c < 4; ++c) sh.Tb[t][kk][c] = Tw[kk][c];
      fw_publish(&sh.vcount, t + 1);
    }
    __syncwarp();  // lane 0 wrote tau
    if (lane < jmax) taub[lane] = sh.tau[lane];
  } else if ((w & 3) != 0) {
    // ---------------- update warps ----------------
    // Warp u owns block t = u + 1: it applies V_0 .. V_{t-2} and hands the block over; then,
    // as V_b appear, it writes block t to H and forms the Gram entries V_u^T V_b (b > u).
    const int u = w - (w >> 2) - 1;  // 0 .. 6
    const int t = 1 + u;
    const int g4 = 4 * (lane >> 2), cc = lane & 3;
    if (t < nb) {
      float x[RPG];
      const int col = 4 * t + cc;
#pragma unroll
      for (int q = 0; q < RPG; ++q) {
        const int r = 8 * (q & ~3) + g4 + (q & 3);
        x[q] = (r < m && col < pw) ? S[(long long)r * n + col] : 0.f;
      }
      for (int s2 = 0; s2 <= t - 2; ++s2) {
        if (!fw_wait_geq(&sh.vcount, s2 + 1)) return;
        fw_apply_rows<R, 4, RPG>(x, &sh.V[s2][0][0], &sh.Tb[s2][0][0], g4);
      }
      // Slot t & 1 last held block t - 2, read before V_{t-2} was published (waited above).
      const int sl = t & 1;
#pragma unroll
      for (int q = 0; q < RPG; ++q) sh.B[sl][8 * (q & ~3) + g4 + (q & 3)][cc] = x[q];
      fw_publish(&sh.bflag[sl], t);
    }
    for (int b = u + 1; b < nb; ++b) {
      if (!fw_wait_geq(&sh.vcount, b + 1)) return;
      if (b == t) panel_fw_store_block<RPL>(sh, Hp, n, m, pw, b);
      panel_fw_gram_pair<RPL>(sh, u, b);
      __threadfence_block();
      __syncwarp();
      if (lane == 0) atomicAdd(&sh.gcount[b], 1);
    }
  } else if (w == 4) {
    // ---------------- block 0 to H, then T as the Gram block columns complete ----------------
    if (nb > 0 && fw_wait_geq(&sh.vcount, 1)) panel_fw_store_block<RPL>(sh, Hp, n, m, pw, 0);
    if (P.T == nullptr) return;
    for (int b = 0; b < nb; ++b) {
      // This warp shares the factor warp's scheduler: poll gently.
      if (!fw_wait_geq_sleep(&sh.vcount, b + 1)) return;  // T_b is out
      if (lane < 16) sh.T[4 * b + (lane >> 2)][4 * b + (lane & 3)] = sh.Tb[b][lane >> 2][lane & 3];
      __syncwarp();
      if (b == 0) continue;
      if (!fw_wait_geq_sleep(&sh.gcount[b], b)) return;  // all V_a^T V_b, a < b
      panel_fw_t_step<RPL>(sh, b);
    }
    float* Tg = P.T + (long long)bidx * P.t_bstride;
    for (int e = lane; e < 32 * 32; e += 32) Tg[e] = sh.T[e >> 5][e & 31];
  }
}

}  // namespace qrb200
