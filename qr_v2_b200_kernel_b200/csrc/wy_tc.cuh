// Compact-WY trailing update on the 5th-generation tensor cores (tcgen05, TMEM accumulators,
// 3xTF32 for FP32 accuracy), replacing the CUDA-core path for panels of width 32:
//
//   tc_vtc_kernel : Wp[s]^T = C_s^T V_s                 (one row split s per CTA)
//                   M = 128 trailing columns, N = 32, K = the split's rows (32-row chunks,
//                   double-buffered shared-memory stages, MMA completion on mbarriers)
//   tc_upd_kernel : W2 = T^T sum_s Wp[s]  on CUDA cores (thread = trailing column), then
//                   P = V W2 with M = 128 rows, N = 128 columns, K = 32 on the tensor cores,
//                   and the epilogue C <- C - P
//
// i.e. C <- (I - V T^T V^T) C = Q_panel^T C, the application of
// milestones/01_eager_official123203us.py:102-107 / submission.py:453-480.
// V is read implicitly from the factored panel in H; C is read from `src` (A for the first
// panel) and written to H. Requires n % 4 == 0 (16-byte row segments).
#pragma once

#include "tc.cuh"
#include "wy_simt.cuh"

namespace qrb200 {

constexpr int kTcCols = 128;  // trailing columns per CTA (MMA M of V^T C, N of V W2)
constexpr int kTcRows = 128;  // rows per CTA in tc_upd (MMA M of V W2)
constexpr int kTcChunk = 32;  // rows per stage in tc_vtc (K of one stage)

// ---- tc_vtc: shared layout ------------------------------------------------------------
// Both operands are MN-major (A = C^T: M = trailing columns; B = V: N = panel columns; K =
// rows), stored in the SW128_32B layout:
//   C chunk: 32 rows x 128 columns: 4 MN atoms (LBO = 512) x 8 K atoms (SBO = 2048), 16 KB,
//   V chunk: 32 rows x 32 columns:  1 MN atom             x 8 K atoms (SBO = 512),   4 KB,
// each as hi and lo. A warp stores one 512-byte atom per instruction (lane -> 16-byte piece).
struct VtcStage {
  float c_hi[kTcChunk * kTcCols];
  float c_lo[kTcChunk * kTcCols];
  float v_hi[kTcChunk * 32];
  float v_lo[kTcChunk * 32];
};
struct VtcShared {
  VtcStage st[2];
  uint64_t mbar[2];
  uint32_t tmem;
};
constexpr size_t kVtcSmem = sizeof(VtcShared) + 1024;  // + alignment slack

__device__ __forceinline__ unsigned char* align1024(unsigned char* p) {
  const uint32_t s = smem_u32(p);
  return p + ((1024u - (s & 1023u)) & 1023u);
}

__global__ void __launch_bounds__(128) tc_vtc_kernel(WyParams P) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  VtcShared& sh = *reinterpret_cast<VtcShared*>(align1024(smem_raw));
  constexpr uint32_t LBO = 512, SBO_C = 2048, SBO_V = 512;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bidx = blockIdx.z, split = blockIdx.y;
  const int n = P.n, k = P.k, w = P.w, m = n - k, nc = n - k - w;
  const int col0 = blockIdx.x * kTcCols;
  const float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  const int r_begin = split * P.rows_per_split;
  const int r_end = min(m, r_begin + P.rows_per_split);
  const int nchunks = r_end > r_begin ? (r_end - r_begin + kTcChunk - 1) / kTcChunk : 0;

  if (tid == 0) {
    mbar_init(&sh.mbar[0], 1);
    mbar_init(&sh.mbar[1], 1);
    fence_async_smem();
  }
  if (warp == 0) tmem_alloc(&sh.tmem, 32);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  constexpr uint32_t idesc = make_idesc_tf32(128, 32, true, true);
  bool ok = true;
  const int q8 = lane & 7, kr = lane >> 3;  // 16-byte piece within a 128-byte row, row within atom

  for (int ch = 0; ch < nchunks; ++ch) {
    const int s = ch & 1;
    VtcStage& st = sh.st[s];
    if (ch >= 2) ok = mbar_wait(&sh.mbar[s], ((ch >> 1) - 1) & 1) && ok;
    const int r0 = r_begin + ch * kTcChunk;
    // C chunk: 32 atoms (4 MN x 8 K), 8 per warp.
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int atom = it * 4 + warp;
      const int mn = (atom & 3) * 32 + 4 * q8, kk = (atom >> 2) * 4 + kr;
      const int r = r0 + kk, col = col0 + mn;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < r_end && col < nc) x = *reinterpret_cast<const float4*>(Sb + (long long)(k + r) * n + k + w + col);
      float4 hi, lo;
      split4(x, hi, lo);
      const uint32_t off = sw32_off(mn, kk, LBO, SBO_C) >> 2;
      *reinterpret_cast<float4*>(st.c_hi + off) = hi;
      *reinterpret_cast<float4*>(st.c_lo + off) = lo;
    }
    // V chunk: 8 atoms (1 MN x 8 K) of the unit lower trapezoid, 2 per warp.
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int kk = (it * 4 + warp) * 4 + kr;
      const int c = 4 * q8;
      const int r = r0 + kk;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < r_end) {
        const float4 h = *reinterpret_cast<const float4*>(Hb + (long long)(k + r) * n + k + c);
        x.x = (r > c) ? h.x : (r == c ? 1.f : 0.f);
        x.y = (r > c + 1) ? h.y : (r == c + 1 ? 1.f : 0.f);
        x.z = (r > c + 2) ? h.z : (r == c + 2 ? 1.f : 0.f);
        x.w = (r > c + 3) ? h.w : (r == c + 3 ? 1.f : 0.f);
      }
      float4 hi, lo;
      split4(x, hi, lo);
      const uint32_t off = sw32_off(c, kk, LBO, SBO_V) >> 2;
      *reinterpret_cast<float4*>(st.v_hi + off) = hi;
      *reinterpret_cast<float4*>(st.v_lo + off) = lo;
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ach = smem_u32(st.c_hi), acl = smem_u32(st.c_lo);
      const uint32_t bvh = smem_u32(st.v_hi), bvl = smem_u32(st.v_lo);
#pragma unroll
      for (int ks = 0; ks < kTcChunk / 8; ++ks) {
        mma_tf32x3(tmem, make_sdesc_sw32(ach + ks * 2 * SBO_C, LBO, SBO_C),
                   make_sdesc_sw32(acl + ks * 2 * SBO_C, LBO, SBO_C), make_sdesc_sw32(bvh + ks * 2 * SBO_V, LBO, SBO_V),
                   make_sdesc_sw32(bvl + ks * 2 * SBO_V, LBO, SBO_V), idesc, ch > 0 || ks > 0);
      }
      mma_commit(&sh.mbar[s]);
    }
  }
  if (nchunks > 0) {
    const int last = nchunks - 1;
    ok = mbar_wait(&sh.mbar[last & 1], (last >> 1) & 1) && ok;
  }
  tc_fence_after();
  // Epilogue: thread t holds W^T[col0 + t][0..32) in TMEM lane t.
  float wv[32];
  tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16), wv);
  if (nchunks == 0 || !ok) {
#pragma unroll
    for (int i = 0; i < 32; ++i) wv[i] = 0.f;
  }
  const int col = col0 + tid;
  if (col < nc) {
    float* out = P.Wp + (((long long)bidx * P.nsplit + split) * P.ncmax + col) * 32;
#pragma unroll
    for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(out + i) = make_float4(wv[i], wv[i + 1], wv[i + 2], wv[i + 3]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 32);
}

// ---- tc_upd: shared layout ------------------------------------------------------------
// B = W2^T: 128 trailing columns x 32 (K), CS = 128 B, RS = 1024 B, 16 KB (hi and lo).
// A = V tile: 128 rows x 32 (K),            CS = 128 B, RS = 1024 B, 16 KB (hi and lo).
struct UpdShared {
  float b_hi[kTcCols * 32];  // K-major operands: no-swizzle core-matrix layout
  float b_lo[kTcCols * 32];
  float a_hi[kTcRows * 32];
  float a_lo[kTcRows * 32];
  float T[32][33];
  uint64_t mbar;
  uint32_t tmem;
};

constexpr size_t kUpdSmem = sizeof(UpdShared) + 1024;

__global__ void __launch_bounds__(128) tc_upd_kernel(WyParams P) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  UpdShared& sh = *reinterpret_cast<UpdShared*>(align1024(smem_raw));
  constexpr uint32_t RS = 1024, CS = 128;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int bidx = blockIdx.z;
  const int n = P.n, k = P.k, w = P.w, m = n - k, nc = n - k - w;
  const int col0 = blockIdx.x * kTcCols, row0 = blockIdx.y * kTcRows;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  const float* __restrict__ Tb = P.T + (long long)bidx * 32 * 32;

  if (tid == 0) {
    mbar_init(&sh.mbar, 1);
    fence_async_smem();
  }
  if (warp == 0) tmem_alloc(&sh.tmem, 128);
  for (int e = tid; e < 32 * 32; e += 128) sh.T[e >> 5][e & 31] = Tb[e];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;

  // W2^T row of trailing column col0 + tid: W2[i] = sum_{c <= i} T[c][i] W[c].
  {
    const int col = col0 + tid;
    float wv[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) wv[c] = 0.f;
    if (col < nc) {
      for (int s = 0; s < P.nsplit; ++s) {
        const float* src = P.Wp + (((long long)bidx * P.nsplit + s) * P.ncmax + col) * 32;
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          const float4 t = *reinterpret_cast<const float4*>(src + c);
          wv[c] += t.x; wv[c + 1] += t.y; wv[c + 2] += t.z; wv[c + 3] += t.w;
        }
      }
    }
#pragma unroll
    for (int i0 = 0; i0 < 32; i0 += 4) {
      float o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int i = i0 + q;
        float acc = 0.f;
#pragma unroll
        for (int c = 0; c <= i; ++c) acc = fmaf(sh.T[c][i], wv[c], acc);
        o[q] = acc;
      }
      float4 hi, lo;
      split4(make_float4(o[0], o[1], o[2], o[3]), hi, lo);
      const uint32_t off = tile_off(tid, i0, RS, CS) >> 2;
      *reinterpret_cast<float4*>(sh.b_hi + off) = hi;
      *reinterpret_cast<float4*>(sh.b_lo + off) = lo;
    }
  }
  // V tile: rows row0 .. row0 + 127 of the panel, 8 column quads.
  const float* __restrict__ Hin = P.H + (long long)bidx * n * n;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int idx = it * 128 + tid;
    const int rr = (idx & 7) + 8 * (idx >> 6);
    const int cq = (idx >> 3) & 7;
    const int r = row0 + rr;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < m) {
      const float4 h = *reinterpret_cast<const float4*>(Hin + (long long)(k + r) * n + k + 4 * cq);
      const int c = 4 * cq;
      x.x = (r > c) ? h.x : (r == c ? 1.f : 0.f);
      x.y = (r > c + 1) ? h.y : (r == c + 1 ? 1.f : 0.f);
      x.z = (r > c + 2) ? h.z : (r == c + 2 ? 1.f : 0.f);
      x.w = (r > c + 3) ? h.w : (r == c + 3 ? 1.f : 0.f);
    }
    float4 hi, lo;
    split4(x, hi, lo);
    const uint32_t off = tile_off(rr, 4 * cq, RS, CS) >> 2;
    *reinterpret_cast<float4*>(sh.a_hi + off) = hi;
    *reinterpret_cast<float4*>(sh.a_lo + off) = lo;
  }
  fence_async_smem();
  __syncthreads();
  if (tid == 0) {
    tc_fence_after();
    constexpr uint32_t idesc = make_idesc_tf32(128, 128, false, false);
    const uint32_t ah = smem_u32(sh.a_hi), al = smem_u32(sh.a_lo);
    const uint32_t bh = smem_u32(sh.b_hi), bl = smem_u32(sh.b_lo);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      // K-major operands: SBO = row-group stride, LBO = column-quad stride, K step = 2 quads.
      mma_tf32x3(tmem, make_sdesc(ah + ks * 2 * CS, CS, RS), make_sdesc(al + ks * 2 * CS, CS, RS),
                 make_sdesc(bh + ks * 2 * CS, CS, RS), make_sdesc(bl + ks * 2 * CS, CS, RS), idesc, ks > 0);
    }
    mma_commit(&sh.mbar);
  }
  const bool ok = mbar_wait(&sh.mbar, 0);
  tc_fence_after();
  // Epilogue: thread t owns tile row t (TMEM lane t): C[r][cols] -= P[t][cols].
  const int r = row0 + tid;
#pragma unroll 1
  for (int q = 0; q < kTcCols / 32; ++q) {
    float pv[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + q * 32, pv);
    if (!ok || r >= m) continue;
    const int cbase = col0 + q * 32;
    const long long off = (long long)(k + r) * n + k + w + cbase;
#pragma unroll
    for (int e = 0; e < 32; e += 4) {
      if (cbase + e < nc) {  // nc and cbase are multiples of 4
        const float4 c = *reinterpret_cast<const float4*>(Sb + off + e);
        *reinterpret_cast<float4*>(Hb + off + e) =
            make_float4(c.x - pv[e], c.y - pv[e + 1], c.z - pv[e + 2], c.w - pv[e + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

}  // namespace qrb200
