// One-launch compact-WY update of a few trailing columns by a 32-wide panel,
// C <- C - V T^T V^T C (milestones/01_eager_official123203us.py:102-107), for the short
// updates that sit on the critical path: the next panel's columns under look-ahead, or the
// narrow updates inside an outer block. Rows must start on 16-byte boundaries.
//
// A thread-block cluster of CP CTAs covers the m rows (256 per CTA, 512 threads: the few CTAs of
// this critical-path launch have their SMs to themselves, so every phase is spread over twice
// the threads of a resident-CTA design); blockIdx.y picks a 32-column slice of C, blockIdx.z the
// matrix. Each CTA
//   (1) stages its rows of V (unit lower trapezoid, masked) and of the C slice in shared memory
//       with coalesced 16-byte loads,
//   (2) forms its partial W_p = V_p^T C_p (32 x 32; each thread a 4 x 4 block over an eighth of
//       the rows, the eighths added in shared memory in a fixed order),
//   (3) after one cluster barrier adds the CP partials from the peers' shared memory in rank
//       order (two halves of the peers read by two thread halves, then added: every CTA gets
//       bitwise the same W) and forms W2 = T^T W,
//   (4) writes C_p - V_p W2 back (4 x 4 blocks per thread in shared memory, then coalesced).
// A second cluster barrier keeps every CTA's partial readable until all peers are done.
#pragma once

#include "common.cuh"
#include "panel_cl.cuh"
#include "tc.cuh"
#include "wy_simt.cuh"

namespace qrb200 {

constexpr int kU1Rows = 256, kU1Ld = 36, kU1Threads = 512;

// The row-eighth partials are dead once they are summed into W, which happens before the first
// cluster barrier; the buffers written after it share their space, so that two CTAs fit on an
// SM (112 KB each).
struct __align__(16) U1Shared {
  float V[kU1Rows][kU1Ld];
  float C[kU1Rows][kU1Ld];
  union {
    float Wq[8][32][32];  // row-eighth partials
    struct {
      float Wh[32][32];   // sum of the upper half of the peers' partials
      float Wt[32][33];   // the cluster total
      float W2[32][32];   // T^T W
    } s;
  } u;
  float W[32][32];        // this CTA's partial V^T C, read by the peers
  float T[32][33];
};
constexpr size_t kU1Smem = sizeof(U1Shared);

// Peer shared-memory load (the cluster barrier before it orders the peer's writes); not
// volatile, so independent loads are issued back to back.
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 x;
  asm("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w) : "r"(addr));
  return x;
}

__global__ void __launch_bounds__(kU1Threads) wy_u1_kernel(WyParams P) {
  griddep_launch_wait();
  extern __shared__ __align__(16) unsigned char u1_smem_raw[];
  U1Shared& sh = *reinterpret_cast<U1Shared*>(u1_smem_raw);
  uint32_t CP, p;
  asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(CP));
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(p));
  const int bidx = blockIdx.z;
  const int n = P.n, k = P.k, w = P.w, m = n - k, nc = P.cend - k - w;
  const int c0 = P.coff + blockIdx.y * 32;  // first trailing column of this slice
  const int r0 = (int)p * kU1Rows;
  const int tid = threadIdx.x;
  const float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  float* __restrict__ Ho = P.H + (long long)bidx * n * n;

  // (1) stage V, C and T (8 threads per row, 16 bytes each): every global load of the stage is
  // issued before the first shared-memory store, so the whole stage is in flight together.
  float tv[2];
#pragma unroll
  for (int it = 0; it < 2; ++it) tv[it] = P.T[(long long)bidx * P.t_bstride + it * kU1Threads + tid];
  float4 vs[4], xs[4];
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int e = it * kU1Threads + tid, rr = e >> 3, q = e & 7, r = r0 + rr, c = 4 * q;
    vs[it] = make_float4(0.f, 0.f, 0.f, 0.f);
    xs[it] = vs[it];
    if (r < m) {
      if (c < w) vs[it] = *reinterpret_cast<const float4*>(Hb + (long long)(k + r) * n + k + c);
      if (c0 + c < nc) xs[it] = *reinterpret_cast<const float4*>(Sb + (long long)(k + r) * n + k + w + c0 + c);
    }
  }
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int e = it * kU1Threads + tid, rr = e >> 3, q = e & 7, r = r0 + rr, c = 4 * q;
    float4 v = vs[it];
    const float4 x = xs[it];
    if (r < 32) {  // unit lower triangle at the top of the panel
      v.x = (c >= w) ? 0.f : (r > c ? v.x : (r == c ? 1.f : 0.f));
      v.y = (c + 1 >= w) ? 0.f : (r > c + 1 ? v.y : (r == c + 1 ? 1.f : 0.f));
      v.z = (c + 2 >= w) ? 0.f : (r > c + 2 ? v.z : (r == c + 2 ? 1.f : 0.f));
      v.w = (c + 3 >= w) ? 0.f : (r > c + 3 ? v.w : (r == c + 3 ? 1.f : 0.f));
    }
    *reinterpret_cast<float4*>(&sh.V[rr][c]) = v;
    *reinterpret_cast<float4*>(&sh.C[rr][c]) = x;
  }
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int e = it * kU1Threads + tid;
    sh.T[e >> 5][e & 31] = tv[it];
  }
  __syncthreads();
  // (2) partial W over the slab: thread (rq, ig, cg) sums rows rq, rq + 8, ... for a 4 x 4 block.
  {
    // Paired FMAs (two independent, individually rounded fmaf per instruction).
    const int cg = tid & 7, ig = (tid >> 3) & 7, rq = tid >> 6;
    float2 acc[4][2];
#pragma unroll
    for (int a = 0; a < 4; ++a) acc[a][0] = acc[a][1] = make_float2(0.f, 0.f);
#pragma unroll 4
    for (int r = rq; r < kU1Rows; r += 8) {
      const float4 v = *reinterpret_cast<const float4*>(&sh.V[r][4 * ig]);
      const float4 x = *reinterpret_cast<const float4*>(&sh.C[r][4 * cg]);
      const float vv[4] = {v.x, v.y, v.z, v.w};
      const float2 x01 = make_float2(x.x, x.y), x23 = make_float2(x.z, x.w);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const float2 va = make_float2(vv[a], vv[a]);
        acc[a][0] = __ffma2_rn(va, x01, acc[a][0]);
        acc[a][1] = __ffma2_rn(va, x23, acc[a][1]);
      }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
      *reinterpret_cast<float4*>(&sh.u.Wq[rq][4 * ig + a][4 * cg]) =
          make_float4(acc[a][0].x, acc[a][0].y, acc[a][1].x, acc[a][1].y);
  }
  __syncthreads();
  const int i = (tid >> 3) & 31, cq = tid & 7, half = tid >> 8;
  if (half == 0) {
    float4 s = *reinterpret_cast<const float4*>(&sh.u.Wq[0][i][4 * cq]);
#pragma unroll
    for (int q = 1; q < 8; ++q) {
      const float4 t = *reinterpret_cast<const float4*>(&sh.u.Wq[q][i][4 * cq]);
      s.x += t.x;
      s.y += t.y;
      s.z += t.z;
      s.w += t.w;
    }
    *reinterpret_cast<float4*>(&sh.W[i][4 * cq]) = s;
  }
  // (3) cluster total in rank order (peers 0..7 by the lower thread half, 8..15 by the upper
  // half, then the two half sums added), then W2 = T^T W.
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  {
    constexpr int kHalf = kClMaxCta / 2;
    float4 part[kHalf];
#pragma unroll
    for (int q = 0; q < kHalf; ++q) {
      const int src = half * kHalf + q;
      part[q] = (src < (int)CP) ? ld_cluster_f4(cl_map(&sh.W[i][4 * cq], (uint32_t)src)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float4 tot = part[0];
#pragma unroll
    for (int q = 1; q < kHalf; ++q) {
      tot.x += part[q].x;
      tot.y += part[q].y;
      tot.z += part[q].z;
      tot.w += part[q].w;
    }
    if (half == 1) *reinterpret_cast<float4*>(&sh.u.s.Wh[i][4 * cq]) = tot;
    __syncthreads();
    if (half == 0) {
      const float4 hi = *reinterpret_cast<const float4*>(&sh.u.s.Wh[i][4 * cq]);
      sh.u.s.Wt[i][4 * cq] = tot.x + hi.x;
      sh.u.s.Wt[i][4 * cq + 1] = tot.y + hi.y;
      sh.u.s.Wt[i][4 * cq + 2] = tot.z + hi.z;
      sh.u.s.Wt[i][4 * cq + 3] = tot.w + hi.w;
    }
  }
  __syncthreads();
  if (half == 0) {
    float y[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c <= i; ++c) {
      const float t = sh.T[c][i];
#pragma unroll
      for (int e = 0; e < 4; ++e) y[e] = fmaf(t, sh.u.s.Wt[c][4 * cq + e], y[e]);
    }
    *reinterpret_cast<float4*>(&sh.u.s.W2[i][4 * cq]) = make_float4(y[0], y[1], y[2], y[3]);
  }
  __syncthreads();
  // (4) C_p - V_p W2: thread (row group rg = tid / 8, column quad cg = tid % 8) updates rows
  // rg + 64 i (i < 4) of its four columns in place in the staged C (a 4 x 4 register block,
  // paired FMAs, columns of V in order), then the slab goes back through shared memory.
  {
    const int rg = tid >> 3, cg = tid & 7;
    float2 acc[4][2];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float4 x = *reinterpret_cast<const float4*>(&sh.C[rg + 64 * r][4 * cg]);
      acc[r][0] = make_float2(x.x, x.y);
      acc[r][1] = make_float2(x.z, x.w);
    }
#pragma unroll 2
    for (int c4 = 0; c4 < 32; c4 += 4) {
      float4 vr[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) vr[r] = *reinterpret_cast<const float4*>(&sh.V[rg + 64 * r][c4]);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const float4 y = *reinterpret_cast<const float4*>(&sh.u.s.W2[c4 + a][4 * cg]);
        const float2 y01 = make_float2(y.x, y.y), y23 = make_float2(y.z, y.w);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const float v = -(a == 0 ? vr[r].x : (a == 1 ? vr[r].y : (a == 2 ? vr[r].z : vr[r].w)));
          const float2 vv = make_float2(v, v);
          acc[r][0] = __ffma2_rn(vv, y01, acc[r][0]);
          acc[r][1] = __ffma2_rn(vv, y23, acc[r][1]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
      *reinterpret_cast<float4*>(&sh.C[rg + 64 * r][4 * cg]) =
          make_float4(acc[r][0].x, acc[r][0].y, acc[r][1].x, acc[r][1].y);
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int e = it * kU1Threads + tid, rr = e >> 3, q = e & 7, r = r0 + rr, c = 4 * q;
    if (r < m && c0 + c < nc)
      *reinterpret_cast<float4*>(Ho + (long long)(k + r) * n + k + w + c0 + c) =
          *reinterpret_cast<const float4*>(&sh.C[rr][c]);
  }
  // No CTA leaves while a peer may still read its partial. Relaxed: the peers' reads completed
  // (their values were consumed) before they arrive, and nothing written here is read by a peer.
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

}  // namespace qrb200
