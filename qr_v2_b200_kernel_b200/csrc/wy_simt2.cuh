// Streaming FP32 kernels for the 32-wide compact-WY update C <- C - V T^T V^T C
// (milestones/01_eager_official123203us.py:102-107, submission.py:453-480), for rows whose
// starts are 16-byte aligned (n % 4 == 0 and a 16-byte aligned batch):
//
//   wy_vtc2_kernel : Wp[s] = V_s^T C_s  over a row split s; 32 x 128 outputs per CTA, the rows
//                    streamed in 32-row stages by cp.async (three stages in flight), 4 x 4
//                    outputs per thread;
//   wy_vtcn_kernel : the same for updates of 32 or 64 columns;
//   wy_tw2_kernel  : W2 = T^T sum_s Wp[s];
//   wy_upd3_kernel : C <- C - V W2 over persistent tiles, cp.async ring; wy_upd4_kernel: one tile per CTA.
// Same arithmetic per output as wy_simt.cuh except for the summation order inside each
// partial product.
#pragma once

#include "common.cuh"
#include "tc.cuh"
#include "wy_simt.cuh"

namespace qrb200 {

constexpr int kV2Cols = 128, kV2Rows = 32, kV2Stages = 3;
struct Vtc2Stage {
  float C[kV2Rows][kV2Cols];
  float V[kV2Rows][32];
};
constexpr size_t kVtc2Smem = sizeof(Vtc2Stage) * kV2Stages;

__global__ void __launch_bounds__(256) wy_vtc2_kernel(WyParams P) {
  griddep_launch_wait();
  extern __shared__ __align__(16) unsigned char v2_smem_raw[];
  Vtc2Stage* st = reinterpret_cast<Vtc2Stage*>(v2_smem_raw);
  const int bidx = blockIdx.z, split = blockIdx.y;
  const int n = P.n, k = P.k, w = P.w, nc = P.cend - k - w;
  const int col0 = P.coff + blockIdx.x * kV2Cols;
  const float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  const int tid = threadIdx.x, tx = tid & 31, ty = tid >> 5;
  const int r_begin = split * P.rows_per_split;
  const int r_end = min(n - k, r_begin + P.rows_per_split);
  const int nchunks = r_end > r_begin ? (r_end - r_begin + kV2Rows - 1) / kV2Rows : 0;

  auto issue = [&](int ch) {
    Vtc2Stage& s = st[ch % kV2Stages];
    const int rb = r_begin + ch * kV2Rows;
#pragma unroll
    for (int it = 0; it < 4; ++it) {  // C: 32 rows x 32 float4
      const int e = it * 256 + tid, rr = e >> 5, q = e & 31, r = rb + rr, col = col0 + 4 * q;
      const bool ok = r < r_end && col < nc;
      cp_async16(&s.C[rr][4 * q], ok ? Sb + (long long)(k + r) * n + k + w + col : Sb, ok);
    }
    {  // V: 32 rows x 8 float4
      const int rr = tid >> 3, q = tid & 7, r = rb + rr;
      const bool ok = r < r_end && 4 * q < w;
      cp_async16(&s.V[rr][4 * q], ok ? Hb + (long long)(k + r) * n + k + 4 * q : Hb, ok);
    }
  };

  // acc[i][h]: output row 4 ty + i, columns 4 tx + 2 h and the next (paired FMAs: two
  // independent, individually rounded fmaf per instruction).
  float2 acc[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = make_float2(0.f, 0.f);
#pragma unroll
  for (int s = 0; s < kV2Stages - 1; ++s) {
    if (s < nchunks) issue(s);
    cp_async_commit();
  }
  for (int ch = 0; ch < nchunks; ++ch) {
    cp_async_wait<kV2Stages - 2>();
    __syncthreads();
    if (ch + kV2Stages - 1 < nchunks) issue(ch + kV2Stages - 1);
    cp_async_commit();
    Vtc2Stage& s = st[ch % kV2Stages];
    if (split == 0 && ch == 0) {
      // Rows 0..31 of the panel: V is unit lower triangular there (R sits above the diagonal).
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int e = it * 256 + tid, rr = e >> 5, c = e & 31;
        const float v = s.V[rr][c];
        s.V[rr][c] = (c >= w) ? 0.f : (rr > c ? v : (rr == c ? 1.f : 0.f));
      }
      __syncthreads();
    }
#pragma unroll 8
    for (int rr = 0; rr < kV2Rows; ++rr) {
      const float4 v = *reinterpret_cast<const float4*>(&s.V[rr][4 * ty]);
      const float4 c = *reinterpret_cast<const float4*>(&s.C[rr][4 * tx]);
      const float vv[4] = {v.x, v.y, v.z, v.w};
      const float2 c01 = make_float2(c.x, c.y), c23 = make_float2(c.z, c.w);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 vi = make_float2(vv[i], vv[i]);
        acc[i][0] = __ffma2_rn(vi, c01, acc[i][0]);
        acc[i][1] = __ffma2_rn(vi, c23, acc[i][1]);
      }
    }
  }
  cp_async_wait<0>();
  const int col = col0 + 4 * tx;
  if (col < nc) {
    float* out = P.Wp + ((long long)bidx * P.nsplit + split) * 32 * P.ncmax;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<float4*>(out + (long long)(4 * ty + i) * P.ncmax + col) =
          make_float4(acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y);
  }
}

// ---------------------------------------------------------------------------------------
// Persistent C <- C - V W2 over TR x TC tiles (64 x 64, or 128 x 32 for the narrowest
// updates): each CTA walks tiles blockIdx.x, + gridDim.x, ..., with the next tile's C, V and W2
// slices already streaming into the other half of a two-stage cp.async ring while the current
// one is computed (4 x 4 outputs per thread, paired FMAs).
template <int TR, int TC>
struct Upd3Stage {
  float C[TR][TC];
  float V[TR][32 + 4];
  float W[32][TC];
};
constexpr int kU3Rows = 64, kU3Cols = 64;
template <int TR, int TC>
constexpr size_t upd3_smem() { return sizeof(Upd3Stage<TR, TC>) * 2; }

template <int TR, int TC>
__global__ void __launch_bounds__(256) wy_upd3_kernel(WyParams P, int tiles_c, int tiles_r, int ntiles) {
  griddep_launch_wait();
  static_assert(TR * TC == 4096, "256 threads x 4 x 4 outputs");
  constexpr int CG = TC / 4;  // column groups of 4
  extern __shared__ __align__(16) unsigned char u3_smem_raw[];
  Upd3Stage<TR, TC>* st = reinterpret_cast<Upd3Stage<TR, TC>*>(u3_smem_raw);
  const int n = P.n, k = P.k, w = P.w, m = n - k, nc = P.cend - k - w;
  const int tid = threadIdx.x, cg = tid % CG, rg = tid / CG;
  auto tile_of = [&](int t, int& b, int& row0, int& col0) {
    const int per_b = tiles_c * tiles_r;
    b = t / per_b;
    const int rem = t - b * per_b;
    row0 = (rem / tiles_c) * TR;
    col0 = P.coff + (rem % tiles_c) * TC;
  };
  auto issue = [&](int t, int slot) {
    int b, row0, col0;
    tile_of(t, b, row0, col0);
    Upd3Stage<TR, TC>& s = st[slot];
    const float* __restrict__ Sb = P.src + (long long)b * P.src_bstride;
    const float* __restrict__ Hb = P.H + (long long)b * n * n;
    const float* __restrict__ W2b = P.W2 + (long long)b * 32 * P.ncmax;
#pragma unroll
    for (int it = 0; it < TR * CG / 256; ++it) {  // C: TR rows x CG float4
      const int e = it * 256 + tid, rr = e / CG, q = e % CG, r = row0 + rr, col = col0 + 4 * q;
      const bool ok = r < m && col < nc;
      cp_async16(&s.C[rr][4 * q], ok ? Sb + (long long)(k + r) * n + k + w + col : Sb, ok);
    }
#pragma unroll
    for (int it = 0; it < TR * 8 / 256; ++it) {  // V: TR rows x 8 float4
      const int e = it * 256 + tid, rr = e >> 3, q = e & 7, r = row0 + rr;
      const bool ok = r < m && 4 * q < w;
      cp_async16(&s.V[rr][4 * q], ok ? Hb + (long long)(k + r) * n + k + 4 * q : Hb, ok);
    }
#pragma unroll
    for (int it = 0; it < 32 * CG / 256; ++it) {  // W2: 32 rows x CG float4
      const int e = it * 256 + tid, c = e / CG, q = e % CG, col = col0 + 4 * q;
      const bool ok = col < nc;
      cp_async16(&s.W[c][4 * q], ok ? W2b + (long long)c * P.ncmax + col : W2b, ok);
    }
  };
  int t = blockIdx.x;
  if (t < ntiles) issue(t, 0);
  cp_async_commit();
  for (int it = 0; t < ntiles; t += gridDim.x, ++it) {
    const int slot = it & 1;
    const int tn = t + gridDim.x;
    if (tn < ntiles) issue(tn, slot ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    int b, row0, col0;
    tile_of(t, b, row0, col0);
    Upd3Stage<TR, TC>& s = st[slot];
    if (row0 == 0) {
      // Panel rows 0..31: V is unit lower triangular there.
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int e = q * 256 + tid, rr = e >> 5, c = e & 31;
        const float v = s.V[rr][c];
        s.V[rr][c] = (c >= w) ? 0.f : (rr > c ? v : (rr == c ? 1.f : 0.f));
      }
      __syncthreads();
    }
    // acc[i][h] holds columns 4 cg + 2 h, 4 cg + 2 h + 1 of row 4 rg + i (paired FMAs).
    float2 acc[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = make_float2(0.f, 0.f);
#pragma unroll 2
    for (int c4 = 0; c4 < 32; c4 += 4) {
      float4 vr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) vr[i] = *reinterpret_cast<const float4*>(&s.V[4 * rg + i][c4]);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const float4 x = *reinterpret_cast<const float4*>(&s.W[c4 + cc][4 * cg]);
        const float2 x0 = make_float2(x.x, x.y), x1 = make_float2(x.z, x.w);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float v = cc == 0 ? vr[i].x : (cc == 1 ? vr[i].y : (cc == 2 ? vr[i].z : vr[i].w));
          const float2 vv = make_float2(v, v);
          acc[i][0] = __ffma2_rn(vv, x0, acc[i][0]);
          acc[i][1] = __ffma2_rn(vv, x1, acc[i][1]);
        }
      }
    }
    const int col = col0 + 4 * cg;
    if (col < nc) {
      float* __restrict__ Ho = P.H + (long long)b * n * n;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = row0 + 4 * rg + i;
        if (r < m) {
          const float4 c = *reinterpret_cast<const float4*>(&s.C[4 * rg + i][4 * cg]);
          *reinterpret_cast<float4*>(Ho + (long long)(k + r) * n + k + w + col) =
              make_float4(c.x - acc[i][0].x, c.y - acc[i][0].y, c.z - acc[i][1].x, c.w - acc[i][1].y);
        }
      }
    }
    __syncthreads();  // the slot is refilled by the next iteration's issue
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------------------
// V^T C for narrow updates (COLS = 32 or 64 trailing columns): the 32 x COLS outputs of a CTA
// are 4 x 4 per thread, and the 128 / COLS thread phases take alternate rows of every 32-row
// stage (so no thread works on padding columns); the phase partials are added in shared
// memory in phase order at the end. Stages as wy_vtc2_kernel.
template <int COLS>
struct VtcnStage {
  float C[kV2Rows][COLS];
  float V[kV2Rows][32];
};
template <int COLS>
constexpr size_t vtcn_smem() { return sizeof(VtcnStage<COLS>) * kV2Stages + (size_t)(128 / COLS) * 32 * COLS * 4; }

template <int COLS>
__global__ void __launch_bounds__(256) wy_vtcn_kernel(WyParams P) {
  griddep_launch_wait();
  constexpr int CG = COLS / 4, NPH = 128 / COLS;
  extern __shared__ __align__(16) unsigned char vn_smem_raw[];
  VtcnStage<COLS>* st = reinterpret_cast<VtcnStage<COLS>*>(vn_smem_raw);
  float* red = reinterpret_cast<float*>(vn_smem_raw + sizeof(VtcnStage<COLS>) * kV2Stages);  // [NPH][32][COLS]
  const int bidx = blockIdx.z, split = blockIdx.y;
  const int n = P.n, k = P.k, w = P.w, nc = P.cend - k - w;
  const int col0 = P.coff + blockIdx.x * COLS;
  const float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  const int tid = threadIdx.x, tx = tid % CG, ty = (tid / CG) % 8, ph = tid / (CG * 8);
  const int r_begin = split * P.rows_per_split;
  const int r_end = min(n - k, r_begin + P.rows_per_split);
  const int nchunks = r_end > r_begin ? (r_end - r_begin + kV2Rows - 1) / kV2Rows : 0;

  auto issue = [&](int ch) {
    VtcnStage<COLS>& s = st[ch % kV2Stages];
    const int rb = r_begin + ch * kV2Rows;
#pragma unroll
    for (int it = 0; it < kV2Rows * CG / 256; ++it) {  // C: 32 rows x CG float4
      const int e = it * 256 + tid, rr = e / CG, q = e % CG, r = rb + rr, col = col0 + 4 * q;
      const bool ok = r < r_end && col < nc;
      cp_async16(&s.C[rr][4 * q], ok ? Sb + (long long)(k + r) * n + k + w + col : Sb, ok);
    }
    {  // V: 32 rows x 8 float4
      const int rr = tid >> 3, q = tid & 7, r = rb + rr;
      const bool ok = r < r_end && 4 * q < w;
      cp_async16(&s.V[rr][4 * q], ok ? Hb + (long long)(k + r) * n + k + 4 * q : Hb, ok);
    }
  };

  // acc[i][h]: output row 4 ty + i, columns 4 tx + 2 h and the next (paired FMAs: two
  // independent, individually rounded fmaf per instruction).
  float2 acc[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = make_float2(0.f, 0.f);
#pragma unroll
  for (int s = 0; s < kV2Stages - 1; ++s) {
    if (s < nchunks) issue(s);
    cp_async_commit();
  }
  for (int ch = 0; ch < nchunks; ++ch) {
    cp_async_wait<kV2Stages - 2>();
    __syncthreads();
    if (ch + kV2Stages - 1 < nchunks) issue(ch + kV2Stages - 1);
    cp_async_commit();
    VtcnStage<COLS>& s = st[ch % kV2Stages];
    if (split == 0 && ch == 0) {
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int e = it * 256 + tid, rr = e >> 5, c = e & 31;
        const float v = s.V[rr][c];
        s.V[rr][c] = (c >= w) ? 0.f : (rr > c ? v : (rr == c ? 1.f : 0.f));
      }
      __syncthreads();
    }
#pragma unroll 4
    for (int rr = ph; rr < kV2Rows; rr += NPH) {
      const float4 v = *reinterpret_cast<const float4*>(&s.V[rr][4 * ty]);
      const float4 c = *reinterpret_cast<const float4*>(&s.C[rr][4 * tx]);
      const float vv[4] = {v.x, v.y, v.z, v.w};
      const float2 c01 = make_float2(c.x, c.y), c23 = make_float2(c.z, c.w);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 vi = make_float2(vv[i], vv[i]);
        acc[i][0] = __ffma2_rn(vi, c01, acc[i][0]);
        acc[i][1] = __ffma2_rn(vi, c23, acc[i][1]);
      }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<float4*>(&red[(ph * 32 + 4 * ty + i) * COLS + 4 * tx]) =
        make_float4(acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y);
  __syncthreads();
  // Threads of phase 0 add the phases in order and store.
  if (ph == 0) {
    const int col = col0 + 4 * tx;
    if (col < nc) {
      float* out = P.Wp + ((long long)bidx * P.nsplit + split) * 32 * P.ncmax;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float4 sum = *reinterpret_cast<const float4*>(&red[(4 * ty + i) * COLS + 4 * tx]);
#pragma unroll
        for (int q = 1; q < NPH; ++q) {
          const float4 x = *reinterpret_cast<const float4*>(&red[(q * 32 + 4 * ty + i) * COLS + 4 * tx]);
          sum.x += x.x;
          sum.y += x.y;
          sum.z += x.z;
          sum.w += x.w;
        }
        *reinterpret_cast<float4*>(out + (long long)(4 * ty + i) * P.ncmax + col) = sum;
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// W2 = T^T sum_s Wp[s] for 32 columns per CTA: thread (row group g, column c) adds the row-split
// partials of W rows 4 g .. 4 g + 3 (independent, coalesced loads), then forms the same rows
// of T^T W from shared memory.
__global__ void __launch_bounds__(256) wy_tw2_kernel(WyParams P) {
  griddep_launch_wait();
  __shared__ float Ts[32][33];
  __shared__ float Ws[32][33];
  const int bidx = blockIdx.y;
  const int nc = P.cend - P.k - P.w;
  const int tid = threadIdx.x, c = tid & 31, g = tid >> 5;
  const int col = P.coff + blockIdx.x * 32 + c;
  const float* Tb = P.T + (long long)bidx * P.t_bstride;
  {
    float tv[4];  // all four loads in flight before the stores
#pragma unroll
    for (int it = 0; it < 4; ++it) tv[it] = Tb[it * 256 + tid];
#pragma unroll
    for (int it = 0; it < 4; ++it) Ts[(it * 256 + tid) >> 5][tid & 31] = tv[it];
  }
  float wv[4] = {0.f, 0.f, 0.f, 0.f};
  if (col < nc) {
    // Splits in groups of four: sixteen independent loads in flight before the adds (which
    // keep the split order).
    const float* W0 = P.Wp + (long long)bidx * P.nsplit * 32 * P.ncmax + (long long)(4 * g) * P.ncmax + col;
    const long long sstride = 32LL * P.ncmax;
    int s = 0;
    for (; s + 4 <= P.nsplit; s += 4) {
      float x[4][4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int a = 0; a < 4; ++a) x[u][a] = W0[(s + u) * sstride + (long long)a * P.ncmax];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int a = 0; a < 4; ++a) wv[a] += x[u][a];
    }
    for (; s < P.nsplit; ++s)
#pragma unroll
      for (int a = 0; a < 4; ++a) wv[a] += W0[s * sstride + (long long)a * P.ncmax];
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) Ws[4 * g + a][c] = wv[a];
  __syncthreads();
  if (col >= nc) return;
  float* out = P.W2 + (long long)bidx * 32 * P.ncmax;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int i = 4 * g + a;
    float acc = 0.f;
    for (int cc = 0; cc <= i; ++cc) acc = fmaf(Ts[cc][i], Ws[cc][c], acc);
    out[(long long)i * P.ncmax + col] = acc;
  }
}

// ---------------------------------------------------------------------------------------
// Persistent C <- C - V W2 over 64 x 128 tiles (4 x 8 outputs per thread: columns 4 cg .. and
// 64 + 4 cg ..), same two-stage cp.async ring as wy_upd3_kernel; two CTAs per SM.
constexpr int kU4Rows = 64, kU4Cols = 128;
struct Upd4Stage {
  float C[kU4Rows][kU4Cols];
  float V[kU4Rows][32];
  float W[32][kU4Cols];
};
// One 64 x 128 tile per CTA (57 KB: several CTAs per SM, so one CTA's loads overlap another's
// arithmetic; a persistent grid that filled every SM held the next high-priority panel back).
constexpr size_t kUpd4Smem = sizeof(Upd4Stage);

// C -= V W2 for tile blockIdx.x (matrix-major, then row tiles, then column tiles).
__global__ void __launch_bounds__(256) wy_upd4_kernel(WyParams P, int tiles_c, int tiles_r) {
  griddep_launch_wait();
  extern __shared__ __align__(16) unsigned char u4_smem_raw[];
  Upd4Stage& s = *reinterpret_cast<Upd4Stage*>(u4_smem_raw);
  const int n = P.n, k = P.k, w = P.w, m = n - k, nc = P.cend - k - w;
  const int tid = threadIdx.x, cg = tid & 15, rg = tid >> 4;
  const int t = blockIdx.x, per_b = tiles_c * tiles_r;
  const int b = t / per_b, rem = t - b * per_b;
  const int row0 = (rem / tiles_c) * kU4Rows, col0 = P.coff + (rem % tiles_c) * kU4Cols;
  {
    const float* __restrict__ Sb = P.src + (long long)b * P.src_bstride;
    const float* __restrict__ Hb = P.H + (long long)b * n * n;
    const float* __restrict__ W2b = P.W2 + (long long)b * 32 * P.ncmax;
#pragma unroll
    for (int it = 0; it < 8; ++it) {  // C: 64 rows x 32 float4
      const int e = it * 256 + tid, rr = e >> 5, q = e & 31, r = row0 + rr, col = col0 + 4 * q;
      const bool ok = r < m && col < nc;
      cp_async16(&s.C[rr][4 * q], ok ? Sb + (long long)(k + r) * n + k + w + col : Sb, ok);
    }
#pragma unroll
    for (int it = 0; it < 2; ++it) {  // V: 64 rows x 8 float4
      const int e = it * 256 + tid, rr = e >> 3, q = e & 7, r = row0 + rr;
      const bool ok = r < m && 4 * q < w;
      cp_async16(&s.V[rr][4 * q], ok ? Hb + (long long)(k + r) * n + k + 4 * q : Hb, ok);
    }
#pragma unroll
    for (int it = 0; it < 4; ++it) {  // W2: 32 rows x 32 float4
      const int e = it * 256 + tid, c = e >> 5, q = e & 31, col = col0 + 4 * q;
      const bool ok = col < nc;
      cp_async16(&s.W[c][4 * q], ok ? W2b + (long long)c * P.ncmax + col : W2b, ok);
    }
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  if (row0 == 0) {
    // Panel rows 0..31: V is unit lower triangular there.
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = q * 256 + tid, rr = e >> 5, c = e & 31;
      const float v = s.V[rr][c];
      s.V[rr][c] = (c >= w) ? 0.f : (rr > c ? v : (rr == c ? 1.f : 0.f));
    }
    __syncthreads();
  }
  // acc[i][h]: row 4 rg + i, column pair h of this thread's eight (h < 2: 4 cg + 2 h ..;
  // h >= 2: 64 + 4 cg + 2 (h - 2) ..).
  float2 acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int h = 0; h < 4; ++h) acc[i][h] = make_float2(0.f, 0.f);
#pragma unroll 2
  for (int c4 = 0; c4 < 32; c4 += 4) {
    float4 vr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) vr[i] = *reinterpret_cast<const float4*>(&s.V[4 * rg + i][c4]);
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const float4 xa = *reinterpret_cast<const float4*>(&s.W[c4 + cc][4 * cg]);
      const float4 xb = *reinterpret_cast<const float4*>(&s.W[c4 + cc][64 + 4 * cg]);
      const float2 xp[4] = {make_float2(xa.x, xa.y), make_float2(xa.z, xa.w), make_float2(xb.x, xb.y),
                            make_float2(xb.z, xb.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float v = cc == 0 ? vr[i].x : (cc == 1 ? vr[i].y : (cc == 2 ? vr[i].z : vr[i].w));
        const float2 vv = make_float2(v, v);
#pragma unroll
        for (int h = 0; h < 4; ++h) acc[i][h] = __ffma2_rn(vv, xp[h], acc[i][h]);
      }
    }
  }
  float* __restrict__ Ho = P.H + (long long)b * n * n;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int cl = 64 * hh + 4 * cg, col = col0 + cl;
    if (col < nc) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = row0 + 4 * rg + i;
        if (r < m) {
          const float4 c = *reinterpret_cast<const float4*>(&s.C[4 * rg + i][cl]);
          *reinterpret_cast<float4*>(Ho + (long long)(k + r) * n + k + w + col) =
              make_float4(c.x - acc[i][2 * hh].x, c.y - acc[i][2 * hh].y, c.z - acc[i][2 * hh + 1].x,
                          c.w - acc[i][2 * hh + 1].y);
        }
      }
    }
  }
}

}  // namespace qrb200
