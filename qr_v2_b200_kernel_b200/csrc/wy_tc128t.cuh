// C -= V W' (the last product of the 128-wide compact-WY update, submission.py:367-373 for the
// reference's _mm_sub) with its operands fed by the tensor memory accelerator.
//
// Per 16-deep K stage one thread issues eight cp.async.bulk.tensor loads -- four 4-column boxes
// of 128 rows of V (rows of H) and four of W'^T -- that complete on the stage's mbarrier
// (transaction bytes). The boxes land raw, [column quad][row][4], in the stage's lo buffers; the
// converter threads then split each float4 into hi = tf32_rna(x) and lo = x - hi and write both
// into the K-major core-matrix layout the MMA reads (masking V to its unit lower trapezoid in the
// block's first 128 rows). Row-major boxes of natural strides keep the tensor maps plain; the
// quad-major landing makes both the converter's reads and its writes conflict-free.
// Three slots, loads one stage ahead, two CTAs per SM. The tiles, MMAs, 3xTF32 arithmetic and
// the staged epilogue are those of tc_gemm128_pipe_kernel<MODE_UPD> (wy_tc128p.cuh) with V in
// place of Y.
#pragma once

#include <cuda.h>

#include "wy_tc128p.cuh"

namespace qrb200 {

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* mbar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(mbar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(mbar)), "r"(bytes) : "memory");
}

struct TmaUpdShared {
  Gemm128Stage st[3];
  uint64_t mbar[3];  // the MMAs of the slot's stage are done
  uint64_t full[3];  // the slot's eight boxes have landed
  uint32_t tmem;
};
constexpr size_t tma_upd_smem() { return sizeof(TmaUpdShared) + 1024; }

// tmV: H as (columns n, rows n, matrices), box 4 x 128 x 1; tmW: the W'^T buffer as (128, rows n,
// matrices), box 4 x 128 x 1. Rows past n read as zero.
__global__ void __launch_bounds__(128) tc_upd_tma_kernel(Gemm128Params P, const __grid_constant__ CUtensorMap tmV,
                                                         const __grid_constant__ CUtensorMap tmW) {
  constexpr int S = 3, kAhead = 1;
  constexpr uint32_t RS = (kGChunk / 4) * 128, CS = 128;
  constexpr int NK = kOB / kGChunk;  // 8 K stages
  constexpr uint32_t kStageBytes = 2u * 128u * kGChunk * 4u;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  TmaUpdShared& sh = *reinterpret_cast<TmaUpdShared*>(align1024(smem_raw));
  const int tid = threadIdx.x, warp = tid >> 5;
  const int bidx = blockIdx.z;
  const int n = P.n, k = P.k, w = P.w, m = n - k;
  const int ncols = P.cend - k - w;
  const int col0 = P.coff + blockIdx.x * 128, row0 = blockIdx.y * 128;
  const int ldc = P.ldc > 0 ? P.ldc : n, ccol = P.ldc > 0 ? P.ccol : k + w;
  const long long hob = P.ldc > 0 ? P.hout_bstride : (long long)n * n;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      mbar_init(&sh.mbar[s], 1);
      mbar_init(&sh.full[s], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
  }
  if (warp == 0) tmem_alloc(&sh.tmem, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  constexpr uint32_t idesc = make_idesc_tf32(128, 128, false, false);
  bool ok = true;
  if (row0 + tid < m) {
    // The epilogue's slice of C starts moving HBM -> L2 under the K loop.
    const float* crow = P.src + (long long)bidx * P.src_bstride + (long long)(k + row0 + tid) * ldc + ccol + col0;
    const int last = min(ncols - col0, 128) - 1;
    if (last >= 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (32 * q <= last) prefetch_l2(crow + 32 * q);
      prefetch_l2(crow + last);
    }
  }
  // Stage kc into its slot (thread 0): four 4-column boxes of V and of W'^T.
  auto issue = [&](int kc) {
    Gemm128Stage& st = sh.st[kc % S];
    uint64_t* fb = &sh.full[kc % S];
    mbar_arrive_expect_tx(fb, kStageBytes);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      tma_load_3d(st.a_lo + q * 512, &tmV, fb, k + kc * kGChunk + 4 * q, k + row0, bidx);
      tma_load_3d(st.b_lo + q * 512, &tmW, fb, kc * kGChunk + 4 * q, col0, bidx);
    }
  };
  if (tid == 0)
#pragma unroll
    for (int s = 0; s < kAhead; ++s) issue(s);
  for (int kc = 0; kc < NK; ++kc) {
    // Refill: stage kc + 1 goes into the slot of stage kc - 2 once its MMAs are done; every other
    // thread learns of that through the slot's `full` barrier (the loads are issued after it).
    if (tid == 0 && kc + kAhead < NK) {
      if (kc >= 2) ok = mbar_wait(&sh.mbar[(kc - 2) % S], (uint32_t)(((kc - 2) / S) & 1)) && ok;
      issue(kc + kAhead);
    }
    ok = mbar_wait(&sh.full[kc % S], (uint32_t)((kc / S) & 1)) && ok;
    Gemm128Stage& st = sh.st[kc % S];
    // Thread piece it: row rr, column quad cq (8 lanes fill one 128-byte core matrix); the raw
    // float4 sits at [cq][rr] of the landing buffer.
    float4 xa[4], xb[4];
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int idx = it * 128 + tid;
      const int rr = (idx & 7) + 8 * (idx >> 5), cq = (idx >> 3) & 3;
      xa[it] = *reinterpret_cast<const float4*>(st.a_lo + cq * 512 + rr * 4);
      xb[it] = *reinterpret_cast<const float4*>(st.b_lo + cq * 512 + rr * 4);
    }
    __syncthreads();  // every raw piece is in registers before the lo buffers are overwritten
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int idx = it * 128 + tid;
      const int rr = (idx & 7) + 8 * (idx >> 5), cq = (idx >> 3) & 3;
      const uint32_t off = tile_off(rr, 4 * cq, RS, CS) >> 2;
      const int c = kc * kGChunk + 4 * cq, r = row0 + rr, j = col0 + rr;
      float4 x = xa[it];
      if (row0 == 0) {  // V is unit lower trapezoidal: rows <= column hold R in H
        x.x = (rr > c) ? x.x : (rr == c ? 1.f : 0.f);
        x.y = (rr > c + 1) ? x.y : (rr == c + 1 ? 1.f : 0.f);
        x.z = (rr > c + 2) ? x.z : (rr == c + 2 ? 1.f : 0.f);
        x.w = (rr > c + 3) ? x.w : (rr == c + 3 ? 1.f : 0.f);
      }
      if (c >= w || r >= m) x = make_float4(0.f, 0.f, 0.f, 0.f);
      float4 y = xb[it];
      if (c >= w || j >= ncols) y = make_float4(0.f, 0.f, 0.f, 0.f);
      float4 h, l;
      split4(x, h, l);
      *reinterpret_cast<float4*>(st.a_hi + off) = h;
      *reinterpret_cast<float4*>(st.a_lo + off) = l;
      split4(y, h, l);
      *reinterpret_cast<float4*>(st.b_hi + off) = h;
      *reinterpret_cast<float4*>(st.b_lo + off) = l;
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ah = smem_u32(st.a_hi), al = smem_u32(st.a_lo);
      const uint32_t bh = smem_u32(st.b_hi), bl = smem_u32(st.b_lo);
#pragma unroll
      for (int ks = 0; ks < kGChunk / 8; ++ks)
        mma_tf32x3(tmem, make_sdesc(ah + ks * 2 * CS, CS, RS), make_sdesc(al + ks * 2 * CS, CS, RS),
                   make_sdesc(bh + ks * 2 * CS, CS, RS), make_sdesc(bl + ks * 2 * CS, CS, RS), idesc,
                   kc > 0 || ks > 0);
      mma_commit(&sh.mbar[kc % S]);
    }
  }
  // Epilogue as tc_gemm128_pipe_kernel<MODE_UPD>'s: each 32-column chunk of the product goes through a
  // padded shared tile so that global traffic runs along rows; the next chunk's C is in flight
  // while the current one is processed.
  const int lane = tid & 31, lr = lane >> 3, lq = lane & 7;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  float* __restrict__ Ho = P.Hout + (long long)bidx * hob;
  constexpr int kPad = 36;
  float* stg = reinterpret_cast<float*>(&sh.st[0]) + warp * (32 * kPad);
  auto load_chunk = [&](int q, float4 (&cv)[8]) {
    const int c = col0 + q * 32 + 4 * lq;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = row0 + 32 * warp + 4 * i + lr;
      cv[i] = (r < m && c < ncols) ? *reinterpret_cast<const float4*>(Sb + (long long)(k + r) * ldc + ccol + c)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  float4 cA[8], cB[8];
  load_chunk(0, cA);
  {
    const int last = NK - 1;
    ok = mbar_wait(&sh.mbar[last % S], (uint32_t)((last / S) & 1)) && ok;
  }
  tc_fence_after();
  __syncthreads();  // every warp is past its ring reads before any staging write
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float pv[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + q * 32, pv);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      *reinterpret_cast<float4*>(stg + lane * kPad + 4 * e) =
          make_float4(pv[4 * e], pv[4 * e + 1], pv[4 * e + 2], pv[4 * e + 3]);
    __syncwarp();
    float4 (&cur)[8] = (q & 1) ? cB : cA;
    float4 (&nxt)[8] = (q & 1) ? cA : cB;
    if (q + 1 < 4) load_chunk(q + 1, nxt);
    const int c = col0 + q * 32 + 4 * lq;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rl = 4 * i + lr, r = row0 + 32 * warp + rl;
      const float4 p = *reinterpret_cast<const float4*>(stg + rl * kPad + 4 * lq);
      if (!ok || r >= m || c >= ncols) continue;
      *reinterpret_cast<float4*>(Ho + (long long)(k + r) * ldc + ccol + c) =
          make_float4(cur[i].x - p.x, cur[i].y - p.y, cur[i].z - p.z, cur[i].w - p.w);
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

}  // namespace qrb200
