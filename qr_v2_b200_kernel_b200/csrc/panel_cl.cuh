// Householder panel (larfg + larf over 32 columns, submission.py:415-449) on a thread-block
// cluster of CP CTAs with one cluster exchange per reflector and no CTA-wide barrier inside the
// reflector loop.
//
// Layout: 8 warps per CTA; warp g owns panel columns 4g .. 4g+3 and holds the CTA's R = 32 RPL
// rows of them in registers (lane l, register i <-> row l + 32 i of the CTA's row slab; CTA p
// holds panel rows [p R, p R + R)). Every warp also keeps a replica of the current pivot column.
//
// Reflector j:
//   (1) every warp forms, over its rows below j, d_c = x_j . a_c for its four columns (c == j
//       gives ||x_j||^2, c < j the LARFT dot x_j . v_c) and sums them across the warp;
//   (2) lanes 0 .. CP-1 store the four partials into CTA `lane`'s slot for this CTA (CTA 0 adds
//       the panel's row j) with st.shared::cluster and arrive there on the step's mbarrier with
//       release semantics -- a push, so no CTA waits for a barrier round trip;
//   (3) every warp waits (acquire) for the 8 x CP arrivals on its own CTA's mbarrier, adds the
//       CP partials in rank order (so every warp of every CTA holds bitwise the same totals),
//       derives beta, tau and scale = 1/(alpha - beta) (submission.py:91-107) and applies
//       a_c -= tau (v_j . a_c) v_j with v_j . a_c = a[j][c] + scale d_c (submission.py:100-103);
//   (4) every warp updates its replica of column j+1 with the same arithmetic, using the copy
//       the owner of column j+1 published in shared memory one step earlier, so the next
//       reduction needs no hand-off at all; the owner of column j+2 publishes that column.
// Slots, row buffers and mbarriers alternate by the parity of j. A CTA cannot run two steps
// ahead of any other: its step-(j+1) push happens after its step-j wait, which needs every
// CTA's step-j push, which every CTA makes after finishing step j-1 (the last use of the
// buffers of parity j+1). T (LARFT, submission.py:129-137) is assembled by CTA 0 after the
// loop from the Gram entries G[c][j] = v_c . v_j = a[j][c] + scale d_c collected on the way.
//
// Every wait is bounded: on expiry the CTA records a device status, stops pushing and waiting,
// and still takes the two cluster barriers every CTA takes (entry and exit), so nothing hangs.
#pragma once

#include <cooperative_groups.h>

#include "panel.cuh"
#include "small_fw.cuh"
#include "tc.cuh"

namespace qrb200 {

constexpr int kClWarps = 8;
constexpr int kClThreads = 32 * kClWarps;
constexpr int kClMaxCta = 16;
// Row stride of the partial-dot slots: 36 floats put the 16 source rows on different banks, so
// the lane-parallel totals read them without conflicts (a 32-float stride put them all on one).
constexpr int kClSlotLd = 36;

template <int RPL>
struct __align__(16) ClShared {
  float slot[2][kClMaxCta][kClSlotLd];  // partial dots, [parity][source CTA][column]
  float rowv[2][32];             // panel row j, [parity][column] (pushed by CTA 0)
  float xs[2][32 * RPL];         // pivot column published by its owner, [parity][row]
  uint64_t mbar[2];
  float tau[32];
  float G[32][33];
  float T[32][33];
};

__device__ __forceinline__ uint32_t cl_map(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cl_fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Store of four floats into a peer CTA's shared memory that also counts 16 bytes of
// transaction on the peer's mbarrier (no release fence on the sending side).
__device__ __forceinline__ void cl_st4_async(uint32_t addr, float a, float b, float c, float d, uint32_t mbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
               "f"(a), "f"(b), "f"(c), "f"(d), "r"(mbar)
               : "memory");
}
__device__ __forceinline__ void cl_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(mbar)), "r"(bytes) : "memory");
}
// Bounded acquire wait (cluster scope) for phase `parity` of a local mbarrier.
__device__ __forceinline__ bool cl_wait(uint64_t* mbar, uint32_t parity) {
  const uint32_t addr = smem_u32(mbar);
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  report_device_failure(kSiteCluster);
  return false;
}

__device__ __forceinline__ void cl_barrier_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cl_barrier_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Partials travel by st.async and complete transaction bytes on the receiver's mbarrier (one
// local expect_tx arrival per phase).
template <int RPL>
__global__ void __launch_bounds__(kClThreads) panel_cl_kernel(PanelParams P) {
  griddep_launch_wait();
  constexpr int R = 32 * RPL;
  __shared__ ClShared<RPL> sh;
  extern __shared__ __align__(16) unsigned char cl_smem_raw[];
  float* stage = reinterpret_cast<float*>(cl_smem_raw);  // 32 x (R + 1) floats
  uint32_t CP, p;
  asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(CP));
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(p));
  const int bidx = blockIdx.y;
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int n = P.n, k = P.k, w = P.w, m = n - k;
  const int r0 = (int)p * R;
  const int rows_valid = max(0, min(R, m - r0));
  const int jmax = min(w, m);
  const float* __restrict__ S = P.src + (long long)bidx * P.src_bstride;
  float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  float* __restrict__ tau_out = P.tau + (long long)bidx * n + k;

  // Bytes one step brings into this CTA: 16 per warp of every CTA, plus CTA 0's row j.
  const uint32_t step_bytes = (uint32_t)(16 * kClWarps * (CP + 1));
  if (threadIdx.x == 0) {
    mbar_init(&sh.mbar[0], 1);
    mbar_init(&sh.mbar[1], 1);
    cl_fence_mbar_init();
    if (jmax > 0) cl_expect_tx(&sh.mbar[0], step_bytes);
    if (jmax > 1) cl_expect_tx(&sh.mbar[1], step_bytes);
  }
  // Entry barrier split around the panel load: peers may push only after every CTA's
  // mbarriers are initialised.
  cl_barrier_arrive();
  for (int i = threadIdx.x; i < 32 * 33; i += kClThreads) (&sh.T[0][0])[i] = 0.f;
  panel_stage_in<R, kClThreads>(S, n, k, r0, rows_valid, w, stage);
  __syncthreads();
  float a[4][RPL];
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int i = 0; i < RPL; ++i) a[q][i] = stage[(4 * g + q) * (R + 1) + lane + 32 * i];
  float xj[RPL];  // replica of the pivot column (column 0 to start with)
#pragma unroll
  for (int i = 0; i < RPL; ++i) xj[i] = stage[lane + 32 * i];
  if (g == 0)
#pragma unroll
    for (int i = 0; i < RPL; ++i) sh.xs[1][lane + 32 * i] = a[1][i];
  __syncthreads();
  cl_barrier_wait();

  const bool top = (p == 0);  // the CTA holding panel rows 0 .. 31 (every pivot row)
  const uint32_t my_slot_off = (uint32_t)((p * kClSlotLd + 4 * g) * sizeof(float));
  const int src = lane & 15;  // source CTA whose partials this lane adds (lanes 16.. repeat 0..15)
  bool ok = true;
  for (int j = 0; j < jmax; ++j) {
    const int ph = j & 1;
    // (1) partial dots over this CTA's rows below j, summed across the warp. Only register 0
    //     of the top CTA holds rows <= j.
    const bool below0 = !top || lane > j;
    float d[4];
    {
      const float x0 = below0 ? xj[0] : 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) d[q] = x0 * a[q][0];
#pragma unroll
      for (int i = 1; i < RPL; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) d[q] = fmaf(xj[i], a[q][i], d[q]);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
      for (int q = 0; q < 4; ++q) d[q] += __shfl_xor_sync(kFullMask, d[q], o);
    float rj[4] = {0.f, 0.f, 0.f, 0.f};
    if (top)
#pragma unroll
      for (int q = 0; q < 4; ++q) rj[q] = __shfl_sync(kFullMask, a[q][0], j);  // row j is lane j, i = 0
    // (2) push to every CTA of the cluster (lane t -> CTA t).
    if (ok && lane < (int)CP) {
      const uint32_t base = cl_map(&sh.slot[ph][0][0], (uint32_t)lane) + my_slot_off;
      const uint32_t rmbar = cl_map(&sh.mbar[ph], (uint32_t)lane);
      cl_st4_async(base, d[0], d[1], d[2], d[3], rmbar);
      if (top) cl_st4_async(cl_map(&sh.rowv[ph][4 * g], (uint32_t)lane), rj[0], rj[1], rj[2], rj[3], rmbar);
    }
    // (3) totals: lane s adds source CTA s's partials; a 4-level butterfly leaves the sum over
    //     all sources, in one fixed order, in every lane of every warp.
    if (ok) ok = cl_wait(&sh.mbar[ph], (uint32_t)((j >> 1) & 1));
    // The phase of step j is complete for every thread of this CTA: the mbarrier's next phase
    // (step j + 2) cannot complete before this CTA's step-(j+1) pushes, so arming it now is safe.
    if (ok && threadIdx.x == 0 && j + 2 < jmax) cl_expect_tx(&sh.mbar[ph], step_bytes);
    const int j1 = min(j + 1, 31);
    const float4 rv = *reinterpret_cast<const float4*>(&sh.rowv[ph][4 * g]);
    const float alpha = sh.rowv[ph][j];
    const float rj1 = sh.rowv[ph][j1];
    float t[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (src < (int)CP) {
      const float4 v = *reinterpret_cast<const float4*>(&sh.slot[ph][src][4 * g]);
      t[0] = v.x;
      t[1] = v.y;
      t[2] = v.z;
      t[3] = v.w;
      t[4] = sh.slot[ph][src][j];
      t[5] = sh.slot[ph][src][j1];
    }
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1)
#pragma unroll
      for (int e = 0; e < 6; ++e) t[e] += __shfl_xor_sync(kFullMask, t[e], o);
    const float rjv[4] = {rv.x, rv.y, rv.z, rv.w};
    const float nrm2 = t[4], dj1 = t[5];
    const Reflector rf = make_reflector_fast(alpha, nrm2);
    const float sc = rf.scale;
    // (4) update: a_c -= tau (v_j . a_c) v_j, v_j = (.., 0, 1, scale x_j) on rows (<j, j, >j).
    const bool rowj = top && lane == j;  // register 0 of this lane is row j
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = 4 * g + q;
      if (c > j && c < w) {
        const float wc = fmaf(sc, t[q], rjv[q]);
        const float cx = rf.tau * sc * wc;
        a[q][0] = below0 ? fmaf(-cx, xj[0], a[q][0]) : (rowj ? fmaf(-rf.tau, wc, a[q][0]) : a[q][0]);
#pragma unroll
        for (int i = 1; i < RPL; ++i) a[q][i] = fmaf(-cx, xj[i], a[q][i]);
      } else if (c == j) {
        a[q][0] = below0 ? a[q][0] * sc : (rowj ? rf.diag : a[q][0]);
#pragma unroll
        for (int i = 1; i < RPL; ++i) a[q][i] *= sc;
        if (top && lane == 0) sh.tau[j] = rf.tau;  // to global after the loop
      } else if (c < j && top && lane == 0) {
        sh.G[c][j] = fmaf(sc, t[q], rjv[q]);  // v_c . v_j
      }
    }
    // (5) replica of column j + 1 (the same arithmetic its owner just applied).
    if (j + 1 < jmax) {
      const float wc1 = fmaf(sc, dj1, rj1);
      const float cx1 = rf.tau * sc * wc1;
      const float* xs = sh.xs[(j + 1) & 1];
      const float x0 = xs[lane];
      xj[0] = below0 ? fmaf(-cx1, xj[0], x0) : (rowj ? fmaf(-rf.tau, wc1, x0) : x0);
#pragma unroll
      for (int i = 1; i < RPL; ++i) xj[i] = fmaf(-cx1, xj[i], xs[lane + 32 * i]);
    }
    // The owner of column j + 2 publishes it (final through reflector j) for the next step.
    if (j + 2 < jmax && g == ((j + 2) >> 2)) {
      const int q2 = (j + 2) & 3;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (q == q2)
#pragma unroll
          for (int i = 0; i < RPL; ++i) sh.xs[j & 1][lane + 32 * i] = a[q][i];
      __threadfence_block();
    }
    __syncwarp();
  }
  // Exit barrier split around the write-out: every push into this CTA has landed once its last
  // wait returned, and no CTA leaves before every CTA got that far.
  cl_barrier_arrive();
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int i = 0; i < RPL; ++i) stage[(4 * g + q) * (R + 1) + lane + 32 * i] = a[q][i];
  __syncthreads();  // the staged panel, tau and the Gram entries are complete
  if (top && g == 0) {
    // Warp 0 of the top CTA builds and stores T and tau while the other warps write the panel.
    larft_inverse_warp(sh.T, sh.G, sh.tau, jmax);
    __syncwarp();
    if (ok) {
      if (lane < jmax) tau_out[lane] = sh.tau[lane];
      if (P.T != nullptr) {
        float* Tb = P.T + (long long)bidx * P.t_bstride;
        for (int i = lane; i < 32 * 32; i += 32) Tb[i] = sh.T[i / 32][i % 32];
      }
    }
  } else if (ok) {
    const int t0 = top ? (int)threadIdx.x - 32 : (int)threadIdx.x;
    panel_stage_out(Hb, n, k, r0, R, rows_valid, w, stage, top ? kClThreads - 32 : kClThreads, t0);
  }
  cl_barrier_wait();
}

template <int RPL>
constexpr size_t panel_cl_smem() { return (size_t)32 * (32 * RPL + 1) * sizeof(float); }

}  // namespace qrb200
