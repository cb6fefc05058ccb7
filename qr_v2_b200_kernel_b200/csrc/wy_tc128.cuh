// Tensor-core pieces of the two-level blocked update (outer blocks of 128 columns made of
// four 32-column panels). With V the 128 reflectors of an outer block (unit lower
// trapezoid in H) and T its 128 x 128 compact-WY factor, the trailing columns C get
//     C <- C - Y (V^T C),   Y = V T^T,
// the same product as C - V T^T V^T C (milestones/01_eager_official123203us.py:102-107) with
// the factor folded into V once per outer block:
//
//   tc_vtcw_pipe_kernel<128, false> : Wp[s]^T = C_s^T V_s  (row split s; wy_tc128p.cuh)
//   tc_vtcw_pipe_kernel<128, true>  : Gp[s]   = V_s^T V_s  (Gram of the outer block)
//   tbuild_kernel                   : T from the Gram and the four 32 x 32 panel factors
//   tc_gemm128_pipe_kernel<Y>       : Y = V T^T            (128-row tiles, K = 128)
//   tc_gemm128_pipe_kernel<UPD>     : C -= Y (sum_s Wp[s]) (128 x 128 tiles, K = 128)
//
// All products are 3xTF32 tcgen05 MMAs with FP32 accumulation in TMEM.
#pragma once

#include "tc.cuh"
#include "wy_simt.cuh"

namespace qrb200 {

constexpr int kOB = 128;  // outer block width (reflectors per fat update)

// Rows of one K stage of the V^T C / Gram products.
constexpr int kWChunk = 16;

// ---------------------------------------------------------------------------------------
// T of the outer block from its Gram matrix and the four 32 x 32 panel factors:
//   T[0:32b, 32b:32b+32] = -T[0:32b, 0:32b] (G[0:32b, 32b:32b+32] T_b),   b = 1, 2, 3
// (the block form of the LARFT recurrence of submission.py:129-137). One CTA per matrix.
struct TbuildParams {
  const float* Gp;        // batch x nsplit x 128 x 128 Gram partials
  int nsplit;
  const float* Tin;       // batch x 4 x 32 x 32 panel factors
  float* Tout;            // batch x 128 x 128
  int ow;                 // outer block width (<= 128)
  int transpose;          // store T^T (applying Q = H_0 H_1 ... needs V T, i.e. Y = V (T^T)^T)
};
// T's strictly lower part is zero, so it holds the Gram blocks the recurrence reads instead:
// G[i][j] (block(i) < block(j)) lives at T[j][i]; and each step's intermediate X sits in the
// block column T[0:r, r:r+32] that the step then overwrites with its result. Rows are 132 floats
// apart so that four consecutive columns form one aligned float4; 66 KB: three CTAs per SM.
constexpr int kTbLd = kOB + 4;
struct TbuildShared {
  float T[kOB][kTbLd];
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
  // Register-tiled block steps: thread (ti, tj) owns rows ti nq .. ti nq + nq - 1 (nq = r / 8:
  // 4, 8 or 12 consecutive rows) of column tj of the new 32-column block. Its rows of a column
  // of G or T are one or more float4 loads shared by the whole warp (same ti), so every shared
  // load feeds four to twelve FMAs instead of one.
  const int tj = tid & 31, ti = tid >> 5;  // 32 columns x 8 row groups
  for (int bb = 1; bb * 32 < ow; ++bb) {
    const int r = 32 * bb;  // rows of the new column block
    const int nq = r / 8;   // rows per thread: 4, 8 or 12
    const int i0 = ti * nq;
    // X = G[0:r, r:r+32] T_bb into T[0:r, r:r+32]. T_bb is upper triangular with zeros stored
    // below its diagonal, so the sum runs over all 32 rows of it (the extra terms are exact zeros).
    {
      float acc[12];
#pragma unroll
      for (int q = 0; q < 12; ++q) acc[q] = 0.f;
#pragma unroll 4
      for (int c = 0; c < 32; ++c) {
        const float t = sh.T[r + c][r + tj];
        const float* gc = &sh.T[r + c][i0];  // G[i0 + q][r + c], stored transposed
#pragma unroll
        for (int q4 = 0; q4 < 3; ++q4) {
          if (4 * q4 < nq) {
            const float4 g4 = *reinterpret_cast<const float4*>(gc + 4 * q4);
            acc[4 * q4 + 0] = fmaf(g4.x, t, acc[4 * q4 + 0]);
            acc[4 * q4 + 1] = fmaf(g4.y, t, acc[4 * q4 + 1]);
            acc[4 * q4 + 2] = fmaf(g4.z, t, acc[4 * q4 + 2]);
            acc[4 * q4 + 3] = fmaf(g4.w, t, acc[4 * q4 + 3]);
          }
        }
      }
      // X goes to rows 0 .. r - 1, which this phase does not read.
#pragma unroll
      for (int q = 0; q < 12; ++q)
        if (q < nq) sh.T[i0 + q][r + tj] = acc[q];
    }
    __syncthreads();
    // T[0:r, r:r+32] = -T[0:r, 0:r] X   (T[0:r, 0:r] upper triangular: c >= row; its storage
    // below the diagonal holds Gram entries, masked here)
    {
      float acc[12];
#pragma unroll
      for (int q = 0; q < 12; ++q) acc[q] = 0.f;
      // The first nq columns meet the thread's own rows (masked); beyond them every term counts.
      for (int c = i0; c < i0 + nq; c += 4) {
        float x[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = sh.T[c + e][r + tj];
#pragma unroll
        for (int q = 0; q < 12; ++q) {
          if (q < nq) {
            const int i = i0 + q;
            const float4 t4 = *reinterpret_cast<const float4*>(&sh.T[i][c]);
            acc[q] = fmaf(c + 0 >= i ? t4.x : 0.f, x[0], acc[q]);
            acc[q] = fmaf(c + 1 >= i ? t4.y : 0.f, x[1], acc[q]);
            acc[q] = fmaf(c + 2 >= i ? t4.z : 0.f, x[2], acc[q]);
            acc[q] = fmaf(c + 3 >= i ? t4.w : 0.f, x[3], acc[q]);
          }
        }
      }
      for (int c = i0 + nq; c < r; c += 4) {
        float x[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = sh.T[c + e][r + tj];
#pragma unroll
        for (int q = 0; q < 12; ++q) {
          if (q < nq) {
            const float4 t4 = *reinterpret_cast<const float4*>(&sh.T[i0 + q][c]);
            acc[q] = fmaf(t4.x, x[0], acc[q]);
            acc[q] = fmaf(t4.y, x[1], acc[q]);
            acc[q] = fmaf(t4.z, x[2], acc[q]);
            acc[q] = fmaf(t4.w, x[3], acc[q]);
          }
        }
      }
      __syncthreads();  // every thread is done reading X
#pragma unroll
      for (int q = 0; q < 12; ++q)
        if (q < nq) sh.T[i0 + q][r + tj] = -acc[q];
    }
    __syncthreads();
  }
  // Upper triangle of the first ow columns; the Gram storage below the diagonal and any block
  // column the recurrence did not reach are zero in T.
  // Stored row by row (coalesced); the transposed form reads shared memory transposed instead.
  for (int e = tid; e < kOB * kOB; e += 256) {
    const int oi = e / kOB, oj = e % kOB;
    const int i = P.transpose ? oj : oi, j = P.transpose ? oi : oj;  // element T[i][j]
    P.Tout[(long long)b * kOB * kOB + e] = (i > j || j >= ow) ? 0.f : sh.T[i][j];
  }
}

// ---------------------------------------------------------------------------------------
// 128 x 128 x 128 3xTF32 GEMM tile, K = 128 in four 32-wide double-buffered stages, both
// operands K-major (no swizzle).
//   MODE_Y  : P = V T^T  -> Y rows   (A = V rows of H, unit lower; B rows = T rows)
//   MODE_UPD: P = Y W    -> C -= P   (A = Y rows; B rows = trailing columns, sum of the
//                                     row-split partials W^T[col][0:128])
// MODE_Y   : Y = V T^T (rows of V)                  -> Y
// MODE_UPD : C -= Y W  (B = one or two W^T partials) -> C
// MODE_WT  : W'^T = W^T T (rows = trailing columns; A = one or two W^T partials, B = T^T rows),
//            so that W' = T^T V^T C                   -> the W'^T buffer (P.Y)
// (C -= V W', A = V rows of H and B = W'^T, is tc_upd_tma_kernel in wy_tc128t.cuh.)
enum Gemm128Mode { MODE_Y = 0, MODE_UPD = 1, MODE_WT = 2 };

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
  // C outside H (applying Q or Q^T to another matrix): row stride, the column of C that holds
  // trailing column 0, and the batch stride of Hout. ldc == 0: C is H itself (row stride n,
  // trailing column 0 at column k + w, batch stride n * n).
  int ldc, ccol;
  long long hout_bstride;
};

// One K stage of the 128 x 128 GEMM tiles: a 16-wide K slice of both operands (K-major, no
// swizzle: CS = 128 B between column quads, RS = 512 B between 8-row groups), hi and lo, 32 KB.
constexpr int kGChunk = 16;
struct Gemm128Stage {
  float a_hi[128 * kGChunk];
  float a_lo[128 * kGChunk];
  float b_hi[128 * kGChunk];
  float b_lo[128 * kGChunk];
};

}  // namespace qrb200
