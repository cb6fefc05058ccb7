// Tensor-core pieces of the two-level blocked update (outer blocks of 128 columns made of
// four 32-column panels). With V the 128 reflectors of an outer block (unit lower
// trapezoid in H) and T its 128 x 128 compact-WY factor, the trailing columns C get
//     C <- C - Y (V^T C),   Y = V T^T,
// the same product as C - V T^T V^T C (milestones/01_eager_official123203us.py:102-107) with
// the factor folded into V once per outer block:
//
//   tc_vtcw_kernel<128, false> : Wp[s]^T = C_s^T V_s  (row split s, MN-major SW128_32B operands)
//   tc_vtcw_kernel<128, true>  : Gp[s]   = V_s^T V_s  (Gram of the outer block, same tile as A and B)
//   tbuild_kernel               : T from the Gram and the four 32 x 32 panel factors
//   tc_gemm128_kernel<Y>        : Y = V T^T            (128-row tiles, K = 128)
//   tc_gemm128_kernel<UPD>      : C -= Y (sum_s Wp[s]) (128 x 128 tiles, K = 128)
//
// All products are 3xTF32 tcgen05 MMAs with FP32 accumulation in TMEM.
#pragma once

#include "tc.cuh"
#include "wy_simt.cuh"
#include "wy_tc.cuh"

namespace qrb200 {

constexpr int kOB = 128;  // outer block width (reflectors per fat update)

// ---------------------------------------------------------------------------------------
// W^T = C^T V (or G = V^T V) over one row split; M = 128 trailing columns (or V columns),
// N = W, K = rows in 16-row stages. Both operands MN-major SW128_32B (K atoms of 4 rows,
// SBO = (MN / 32) * 512). Two 32 KB stages (3 CTAs per SM); each thread prefetches the next
// stage's global data into registers before the current stage's MMAs are issued, so HBM
// latency overlaps tensor-core work.
constexpr int kWChunk = 16;
template <int W>
struct VtcwStage {
  float c_hi[kWChunk * kTcCols];
  float c_lo[kWChunk * kTcCols];
  float v_hi[kWChunk * W];
  float v_lo[kWChunk * W];
};
template <int W>
struct VtcwShared {
  VtcwStage<W> st[2];
  uint64_t mbar[2];
  uint32_t tmem;
};
template <int W>
constexpr size_t vtcw_smem() { return sizeof(VtcwShared<W>) + 1024; }

template <int W, bool GRAM>
__global__ void __launch_bounds__(128) tc_vtcw_kernel(WyParams P) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  VtcwShared<W>& sh = *reinterpret_cast<VtcwShared<W>*>(align1024(smem_raw));
  constexpr uint32_t LBO = 512, SBO_C = (kTcCols / 32) * 512, SBO_V = (W / 32) * 512;
  constexpr int NV = W / 32;        // float4 of V per thread per stage (16 x W / 4 / 128)
  constexpr int NC = GRAM ? 0 : 4;  // float4 of C per thread per stage (16 x 128 / 4 / 128)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bidx = blockIdx.z, split = blockIdx.y;
  const int n = P.n, k = P.k, w = P.w, m = n - k;
  const int nc = GRAM ? w : P.cend - k - w;
  const int col0 = (GRAM ? 0 : P.coff) + blockIdx.x * kTcCols;
  const float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  const int r_begin = split * P.rows_per_split;
  const int r_end = min(m, r_begin + P.rows_per_split);
  const int nchunks = r_end > r_begin ? (r_end - r_begin + kWChunk - 1) / kWChunk : 0;

  if (tid == 0) {
    mbar_init(&sh.mbar[0], 1);
    mbar_init(&sh.mbar[1], 1);
    fence_async_smem();
  }
  if (warp == 0) tmem_alloc(&sh.tmem, W);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  constexpr uint32_t idesc = make_idesc_tf32(128, W, true, true);
  bool ok = true;
  const int q8 = lane & 7, kr = lane >> 3;

  // Element coordinates of this thread's float4 pieces: atom a covers 4 rows x 32 columns and
  // is written by one warp (lane -> row a%4.., 16-byte piece).
  auto v_coord = [&](int it, int& c, int& kk) {
    const int atom = it * 4 + warp;
    c = (atom % NV) * 32 + 4 * q8;
    kk = (atom / NV) * 4 + kr;
  };
  auto c_coord = [&](int it, int& mn, int& kk) {
    const int atom = it * 4 + warp;
    mn = (atom & 3) * 32 + 4 * q8;
    kk = (atom >> 2) * 4 + kr;
  };
  float4 pv[NV], pc[NC > 0 ? NC : 1];
  auto load = [&](int ch) {
    const int r0 = r_begin + ch * kWChunk;
#pragma unroll
    for (int it = 0; it < NV; ++it) {
      int c, kk;
      v_coord(it, c, kk);
      const int r = r0 + kk;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < r_end && c < w) {
        const float4 h = *reinterpret_cast<const float4*>(Hb + (long long)(k + r) * n + k + c);
        x.x = (r > c) ? h.x : (r == c ? 1.f : 0.f);
        x.y = (c + 1 >= w) ? 0.f : ((r > c + 1) ? h.y : (r == c + 1 ? 1.f : 0.f));
        x.z = (c + 2 >= w) ? 0.f : ((r > c + 2) ? h.z : (r == c + 2 ? 1.f : 0.f));
        x.w = (c + 3 >= w) ? 0.f : ((r > c + 3) ? h.w : (r == c + 3 ? 1.f : 0.f));
      }
      pv[it] = x;
    }
#pragma unroll
    for (int it = 0; it < NC; ++it) {
      int mn, kk;
      c_coord(it, mn, kk);
      const int r = r0 + kk, col = col0 + mn;
      pc[it] = (r < r_end && col < nc) ? *reinterpret_cast<const float4*>(Sb + (long long)(k + r) * n + k + w + col)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  // C rows kPrefetchAhead chunks ahead are requested into L2 (one 128-byte line per thread).
  constexpr int kPrefetchAhead = 4;
  auto prefetch_chunk = [&](int ch) {
    if (GRAM || ch >= nchunks || tid >= kWChunk * 5) return;
    const int rr = tid / 5, q = tid % 5, r = r_begin + ch * kWChunk + rr;
    const int cl = min(32 * q, nc - col0 - 1);
    if (r < r_end && cl >= 0) prefetch_l2(Sb + (long long)(k + r) * n + k + w + col0 + cl);
  };
#pragma unroll
  for (int c = 1; c <= kPrefetchAhead; ++c) prefetch_chunk(c);
  if (nchunks > 0) load(0);
  for (int ch = 0; ch < nchunks; ++ch) {
    const int s = ch & 1;
    VtcwStage<W>& st = sh.st[s];
    prefetch_chunk(ch + 1 + kPrefetchAhead);
    if (ch >= 2) ok = mbar_wait(&sh.mbar[s], ((ch >> 1) - 1) & 1) && ok;
#pragma unroll
    for (int it = 0; it < NV; ++it) {
      int c, kk;
      v_coord(it, c, kk);
      float4 hi, lo;
      split4(pv[it], hi, lo);
      const uint32_t off = sw32_off(c, kk, LBO, SBO_V) >> 2;
      *reinterpret_cast<float4*>(st.v_hi + off) = hi;
      *reinterpret_cast<float4*>(st.v_lo + off) = lo;
    }
#pragma unroll
    for (int it = 0; it < NC; ++it) {
      int mn, kk;
      c_coord(it, mn, kk);
      float4 hi, lo;
      split4(pc[it], hi, lo);
      const uint32_t off = sw32_off(mn, kk, LBO, SBO_C) >> 2;
      *reinterpret_cast<float4*>(st.c_hi + off) = hi;
      *reinterpret_cast<float4*>(st.c_lo + off) = lo;
    }
    if (ch + 1 < nchunks) load(ch + 1);  // in flight while this stage's MMAs run
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      // Gram mode uses the V tile as A as well (M = W = 128 columns of V).
      const uint32_t ach = smem_u32(GRAM ? st.v_hi : st.c_hi), acl = smem_u32(GRAM ? st.v_lo : st.c_lo);
      const uint32_t sbo_a = GRAM ? SBO_V : SBO_C;
      const uint32_t bvh = smem_u32(st.v_hi), bvl = smem_u32(st.v_lo);
#pragma unroll
      for (int ks = 0; ks < kWChunk / 8; ++ks) {
        mma_tf32x3(tmem, make_sdesc_sw32(ach + ks * 2 * sbo_a, LBO, sbo_a), make_sdesc_sw32(acl + ks * 2 * sbo_a, LBO, sbo_a),
                   make_sdesc_sw32(bvh + ks * 2 * SBO_V, LBO, SBO_V), make_sdesc_sw32(bvl + ks * 2 * SBO_V, LBO, SBO_V),
                   idesc, ch > 0 || ks > 0);
      }
      mma_commit(&sh.mbar[s]);
    }
  }
  if (nchunks > 0) {
    const int last = nchunks - 1;
    ok = mbar_wait(&sh.mbar[last & 1], (last >> 1) & 1) && ok;
  }
  tc_fence_after();
  // Epilogue: thread t owns row col0 + t of the result (W^T or G), W values.
  const int col = col0 + tid;
  float* out = P.Wp + (((long long)bidx * P.nsplit + split) * P.ncmax + col) * W;
#pragma unroll 1
  for (int q = 0; q < W / 32; ++q) {
    float wv[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + q * 32, wv);
    if (nchunks == 0 || !ok) {
#pragma unroll
      for (int i = 0; i < 32; ++i) wv[i] = 0.f;
    }
    if (col < (GRAM ? W : nc)) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(out + q * 32 + i) = make_float4(wv[i], wv[i + 1], wv[i + 2], wv[i + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, W);
}

// ---------------------------------------------------------------------------------------
// T of the outer block from its Gram matrix and the four 32 x 32 panel factors:
//   T[0:32b, 32b:32b+32] = -T[0:32b, 0:32b] (G[0:32b, 32b:32b+32] T_b),   b = 1, 2, 3
// (the block form of the LARFT recurrence of submission.py:129-137). One CTA per matrix.
struct TbuildParams {
  const float* Gp;        // batch x nsplit x 128 x 128 Gram partials
  int nsplit;
  const float* Tin;       // batch x 4 x 32 x 32 panel factors
  float* Tout;            // batch x 128 x 128
  int ow;                 // outer block width (multiple of 32, <= 128)
};
// T's strictly lower part is zero, so it holds the Gram blocks the recurrence reads instead:
// G[i][j] (block(i) < block(j)) lives at T[j][i]; and each step's intermediate X sits in the
// block column T[0:r, r:r+32] that the step then overwrites with its result. 66 KB: three CTAs
// per SM.
struct TbuildShared {
  float T[kOB][kOB + 1];
};
constexpr size_t kTbuildSmem = sizeof(TbuildShared);

__global__ void __launch_bounds__(256, 3) tbuild_kernel(TbuildParams P) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  TbuildShared& sh = *reinterpret_cast<TbuildShared*>(smem_raw);
  const int b = blockIdx.x, tid = threadIdx.x;
  const int ow = P.ow;
  // The panel factors (diagonal blocks) land by cp.async while the Gram partials are summed.
#pragma unroll
  for (int it = 0; it < 16; ++it) {
    const int e = it * 256 + tid;
    const int blk = e >> 10, i = (e >> 5) & 31, j = e & 31;
    if (32 * blk < ow) cp_async4(&sh.T[32 * blk + i][32 * blk + j], P.Tin + (long long)b * 4096 + e);
  }
  cp_async_commit();
  // Sum the Gram partials: 16 float4 per thread, all loads of a split issued together.
  {
    float4 g[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) g[t] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < P.nsplit; ++q) {
      const float4* src = reinterpret_cast<const float4*>(P.Gp + ((long long)b * P.nsplit + q) * kOB * kOB);
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const float4 x = src[t * 256 + tid];
        g[t].x += x.x; g[t].y += x.y; g[t].z += x.z; g[t].w += x.w;
      }
    }
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      const int e = 4 * (t * 256 + tid), i = e / kOB, j = e % kOB;
      if ((i >> 5) < (j >> 5)) {  // cross-panel Gram block, stored transposed below the diagonal
        sh.T[j][i] = g[t].x; sh.T[j + 1][i] = g[t].y; sh.T[j + 2][i] = g[t].z; sh.T[j + 3][i] = g[t].w;
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  // Register-tiled block steps: thread (ti, tj) owns rows ti + 8 q (q < r/8... up to 12) of
  // column tj of the new 32-column block, so every shared load feeds several independent
  // FMA chains.
  const int tj = tid & 31, ti = tid >> 5;  // 32 columns x 8 row phases
  for (int bb = 1; bb * 32 < ow; ++bb) {
    const int r = 32 * bb;  // rows of the new column block
    const int nq = r / 8;   // rows per thread: 4, 8 or 12
    // X = G[0:r, r:r+32] T_bb     (T_bb upper triangular: c <= tj), into T[0:r, r:r+32]
    {
      float acc[12];
#pragma unroll
      for (int q = 0; q < 12; ++q) acc[q] = 0.f;
      for (int c = 0; c <= tj; ++c) {
        const float t = sh.T[r + c][r + tj];
#pragma unroll
        for (int q = 0; q < 12; ++q)
          if (q < nq) acc[q] = fmaf(sh.T[r + c][ti + 8 * q], t, acc[q]);  // G[ti + 8q][r + c]
      }
#pragma unroll
      for (int q = 0; q < 12; ++q)
        if (q < nq) sh.T[ti + 8 * q][r + tj] = acc[q];
    }
    __syncthreads();
    // T[0:r, r:r+32] = -T[0:r, 0:r] X   (T[0:r, 0:r] upper triangular: c >= row)
    {
      float acc[12];
#pragma unroll
      for (int q = 0; q < 12; ++q) acc[q] = 0.f;
      for (int c = ti; c < r; ++c) {
        const float x = sh.T[c][r + tj];
#pragma unroll
        for (int q = 0; q < 12; ++q) {
          const int i = ti + 8 * q;
          if (q < nq && c >= i) acc[q] = fmaf(sh.T[i][c], x, acc[q]);
        }
      }
      __syncthreads();  // every thread is done reading X
#pragma unroll
      for (int q = 0; q < 12; ++q)
        if (q < nq) sh.T[ti + 8 * q][r + tj] = -acc[q];
    }
    __syncthreads();
  }
  // Upper triangle of the first ow columns; the Gram storage below the diagonal and any block
  // column the recurrence did not reach are zero in T.
  for (int e = tid; e < kOB * kOB; e += 256) {
    const int i = e / kOB, j = e % kOB;
    P.Tout[(long long)b * kOB * kOB + e] = (i > j || j >= ow) ? 0.f : sh.T[i][j];
  }
}

// ---------------------------------------------------------------------------------------
// 128 x 128 x 128 3xTF32 GEMM tile, K = 128 in four 32-wide double-buffered stages, both
// operands K-major (no swizzle).
//   MODE_Y  : P = V T^T  -> Y rows   (A = V rows of H, unit lower; B rows = T rows)
//   MODE_UPD: P = Y W    -> C -= P   (A = Y rows; B rows = trailing columns, sum of the
//                                     row-split partials W^T[col][0:128])
enum Gemm128Mode { MODE_Y = 0, MODE_UPD = 1 };

struct Gemm128Params {
  const float* H;         // matrices (V source for MODE_Y; C destination for MODE_UPD)
  const float* src;       // C source for MODE_UPD (A for the first outer block, else H)
  long long src_bstride;
  float* Hout;
  const float* T;         // batch x 128 x 128 (MODE_Y)
  float* Y;               // batch x ldy x 128 (row r of the outer block at r * 128)
  long long y_bstride;
  const float* Wp;        // batch x nsplit x ncmax x 128 (MODE_UPD)
  int nsplit, ncmax;
  int n, k, w;            // outer block: rows/columns from k, width w (<= 128)
  int cend;               // MODE_UPD: trailing columns [k + w, cend)
  int coff;               // MODE_UPD: first trailing column of this launch (tile-aligned)
};

// Stages hold a 16-wide K slice of both operands (K-major, no swizzle: CS = 128 B between
// column quads, RS = 512 B between 8-row groups): 32 KB per stage, two stages, 3 CTAs per SM.
constexpr int kGChunk = 16;
struct Gemm128Stage {
  float a_hi[128 * kGChunk];
  float a_lo[128 * kGChunk];
  float b_hi[128 * kGChunk];
  float b_lo[128 * kGChunk];
};
struct Gemm128Shared {
  Gemm128Stage st[2];
  uint64_t mbar[2];
  uint32_t tmem;
};
constexpr size_t kGemm128Smem = sizeof(Gemm128Shared) + 1024;

template <int MODE>
__global__ void __launch_bounds__(128) tc_gemm128_kernel(Gemm128Params P) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Gemm128Shared& sh = *reinterpret_cast<Gemm128Shared*>(align1024(smem_raw));
  constexpr uint32_t RS = (kGChunk / 4) * 128, CS = 128;
  constexpr int NK = kOB / kGChunk;  // K stages
  const int tid = threadIdx.x, warp = tid >> 5;
  const int bidx = blockIdx.z;
  const int n = P.n, k = P.k, w = P.w, m = n - k;
  const int ncols = (MODE == MODE_Y) ? kOB : P.cend - k - w;  // B rows (N extent)
  const int col0 = (MODE == MODE_UPD ? P.coff : 0) + blockIdx.x * 128, row0 = blockIdx.y * 128;
  const float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  const float* __restrict__ Yb = P.Y + (long long)bidx * P.y_bstride;

  if (tid == 0) {
    mbar_init(&sh.mbar[0], 1);
    mbar_init(&sh.mbar[1], 1);
    fence_async_smem();
  }
  if (warp == 0) tmem_alloc(&sh.tmem, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  constexpr uint32_t idesc = make_idesc_tf32(128, 128, false, false);
  bool ok = true;

  // Piece it of this thread: row rr of the tile, column quad cq of the K slice (8 lanes fill
  // one 128-byte core matrix).
  auto coord = [&](int it, int& rr, int& cq) {
    const int idx = it * 128 + tid;
    rr = (idx & 7) + 8 * (idx >> 5);
    cq = (idx >> 3) & 3;
  };
  float4 pa[4], pb[4];
  auto load = [&](int kc) {
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      int rr, cq;
      coord(it, rr, cq);
      const int c = kc * kGChunk + 4 * cq;
      // A: rows of V (unit lower, MODE_Y) or of Y (MODE_UPD)
      const int r = row0 + rr;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < m && c < w) {
        if (MODE == MODE_Y) {
          const float4 h = *reinterpret_cast<const float4*>(Hb + (long long)(k + r) * n + k + c);
          x.x = (r > c) ? h.x : (r == c ? 1.f : 0.f);
          x.y = (c + 1 >= w) ? 0.f : ((r > c + 1) ? h.y : (r == c + 1 ? 1.f : 0.f));
          x.z = (c + 2 >= w) ? 0.f : ((r > c + 2) ? h.z : (r == c + 2 ? 1.f : 0.f));
          x.w = (c + 3 >= w) ? 0.f : ((r > c + 3) ? h.w : (r == c + 3 ? 1.f : 0.f));
        } else {
          x = *reinterpret_cast<const float4*>(Yb + (long long)r * kOB + c);
        }
      }
      pa[it] = x;
      // B: rows of T (MODE_Y) or trailing columns of sum_s W^T (MODE_UPD)
      const int j = col0 + rr;
      float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j < ncols && c < w) {
        if (MODE == MODE_Y) {
          y = *reinterpret_cast<const float4*>(P.T + ((long long)bidx * kOB + j) * kOB + c);
        } else {
          for (int q = 0; q < P.nsplit; ++q) {
            const float4 t = *reinterpret_cast<const float4*>(
                P.Wp + (((long long)bidx * P.nsplit + q) * P.ncmax + j) * kOB + c);
            y.x += t.x; y.y += t.y; y.z += t.z; y.w += t.w;
          }
        }
      }
      pb[it] = y;
    }
  };

  load(0);
  for (int kc = 0; kc < NK; ++kc) {
    const int s = kc & 1;
    Gemm128Stage& st = sh.st[s];
    if (kc >= 2) ok = mbar_wait(&sh.mbar[s], ((kc >> 1) - 1) & 1) && ok;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      int rr, cq;
      coord(it, rr, cq);
      const uint32_t off = tile_off(rr, 4 * cq, RS, CS) >> 2;
      float4 hi, lo;
      split4(pa[it], hi, lo);
      *reinterpret_cast<float4*>(st.a_hi + off) = hi;
      *reinterpret_cast<float4*>(st.a_lo + off) = lo;
      split4(pb[it], hi, lo);
      *reinterpret_cast<float4*>(st.b_hi + off) = hi;
      *reinterpret_cast<float4*>(st.b_lo + off) = lo;
    }
    if (kc + 1 < NK) load(kc + 1);  // in flight while this stage's MMAs run
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
      mma_commit(&sh.mbar[s]);
    }
  }
  // Epilogue: thread t owns tile row t (TMEM lane t). The C slice for the next 32 columns is
  // requested before the current one is processed.
  const int r = row0 + tid;
  const bool row_ok = r < m;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  float* __restrict__ Ho = P.Hout + (long long)bidx * n * n;
  const long long roff = (long long)(k + r) * n + k + w;
  float4 cv[8];
  auto load_c = [&](int q) {
    const int cbase = col0 + q * 32;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      cv[e] = (MODE == MODE_UPD && row_ok && cbase + 4 * e < ncols)
                  ? *reinterpret_cast<const float4*>(Sb + roff + cbase + 4 * e)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  if (MODE == MODE_UPD) load_c(0);
  {
    const int last = NK - 1;
    ok = mbar_wait(&sh.mbar[last & 1], (last >> 1) & 1) && ok;
  }
  tc_fence_after();
#pragma unroll 1
  for (int q = 0; q < 4; ++q) {
    float pv[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + q * 32, pv);
    float4 cur[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) cur[e] = cv[e];
    if (MODE == MODE_UPD && q + 1 < 4) load_c(q + 1);
    if (!ok || !row_ok) continue;
    const int cbase = col0 + q * 32;
    if (MODE == MODE_Y) {
      float* yrow = P.Y + (long long)bidx * P.y_bstride + (long long)r * kOB + cbase;
#pragma unroll
      for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4*>(yrow + e) = make_float4(pv[e], pv[e + 1], pv[e + 2], pv[e + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (cbase + 4 * e < ncols)
          *reinterpret_cast<float4*>(Ho + roff + cbase + 4 * e) =
              make_float4(cur[e].x - pv[4 * e], cur[e].y - pv[4 * e + 1], cur[e].z - pv[4 * e + 2], cur[e].w - pv[4 * e + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

}  // namespace qrb200
