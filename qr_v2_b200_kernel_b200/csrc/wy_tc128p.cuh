// 128 x 128 x 128 3xTF32 tcgen05 tile (Y = V T^T, or C -= Y W) with its operands streamed by
// cp.async: each 16-byte piece of raw fp32 lands directly at its place in the K-major
// core-matrix layout of the MMA operand (the hi buffer of a four-slot ring), two K stages ahead
// of the MMAs. The thread that requested a piece splits it in place once it has arrived
// (hi = tf32_rna(x) over x, lo = x - hi beside it), so no operand passes through registers while
// its load is in flight and the load latency is covered by two stages of tensor-core work.
// Same tiles, same arithmetic as tc_gemm128_kernel (wy_tc128.cuh), so results agree bit for bit.
// MODE_UPD takes W^T as one or two row-split partials (nsplit <= 2).
#pragma once

#include "wy_simt2.cuh"
#include "wy_tc128.cuh"

namespace qrb200 {

// SLOTS K stages of 16 resident; loads run SLOTS - 2 stages ahead (a slot is refilled once the
// MMAs of the stage two before the current one are done). Four slots: one CTA per SM; three:
// two CTAs per SM.
template <int SLOTS>
struct Pipe128Shared {
  Gemm128Stage st[SLOTS];
  uint64_t mbar[SLOTS];
  uint32_t tmem;
};
template <int SLOTS>
constexpr size_t pipe128_smem() { return sizeof(Pipe128Shared<SLOTS>) + 1024; }

template <int MODE, int SLOTS>
__global__ void __launch_bounds__(128) tc_gemm128_pipe_kernel(Gemm128Params P) {
  constexpr int kPipeSlots = SLOTS, kAhead = SLOTS - 2;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Pipe128Shared<SLOTS>& sh = *reinterpret_cast<Pipe128Shared<SLOTS>*>(align1024(smem_raw));
  constexpr uint32_t RS = (kGChunk / 4) * 128, CS = 128;
  constexpr int NK = kOB / kGChunk;  // 8 K stages
  const int tid = threadIdx.x, warp = tid >> 5;
  const int bidx = blockIdx.z;
  const int n = P.n, k = P.k, w = P.w, m = n - k;
  constexpr bool kStore = (MODE == MODE_Y || MODE == MODE_WT);  // P to a buffer, not C -= P
  constexpr bool kUpd = !kStore;
  constexpr bool kAV = (MODE == MODE_Y);                         // A = V rows of H
  const int ncols = kStore ? kOB : P.cend - k - w;
  const int mrows = (MODE == MODE_WT) ? P.cend - k - w : m;      // valid A rows
  const int col0 = (kUpd ? P.coff : 0) + blockIdx.x * 128, row0 = (MODE == MODE_WT ? P.coff : 0) + blockIdx.y * 128;
  const int ldc = P.ldc > 0 ? P.ldc : n, ccol = P.ldc > 0 ? P.ccol : k + w;
  const long long hob = P.ldc > 0 ? P.hout_bstride : (long long)n * n;
  const float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  const float* __restrict__ Yb = P.Y + (long long)bidx * P.y_bstride;
  const float* __restrict__ Bsrc = (MODE == MODE_Y || MODE == MODE_WT) ? P.T + (long long)bidx * kOB * kOB
                                                                       : P.Wp + (long long)bidx * P.nsplit * P.ncmax * kOB;
  const float* __restrict__ Wsrc = P.Wp + (long long)bidx * P.nsplit * P.ncmax * kOB;  // MODE_WT's A

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kPipeSlots; ++s) mbar_init(&sh.mbar[s], 1);
    fence_async_smem();
  }
  if (warp == 0) tmem_alloc(&sh.tmem, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  constexpr uint32_t idesc = make_idesc_tf32(128, 128, false, false);
  bool ok = true;
  if (kUpd && row0 + tid < m) {
    // The epilogue's slice of C (this thread's row, 128 columns) starts moving HBM -> L2 now,
    // under the K loop, instead of after it.
    const float* crow = P.src + (long long)bidx * P.src_bstride + (long long)(k + row0 + tid) * ldc + ccol + col0;
    const int last = min(ncols - col0, 128) - 1;
    if (last >= 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (32 * q <= last) prefetch_l2(crow + 32 * q);
      prefetch_l2(crow + last);
    }
  }

  // Piece it of this thread: row rr of the tile, column quad cq of the K slice (8 lanes fill
  // one 128-byte core matrix) -- the mapping of tc_gemm128_kernel.
  auto coord = [&](int it, int& rr, int& cq) {
    const int idx = it * 128 + tid;
    rr = (idx & 7) + 8 * (idx >> 5);
    cq = (idx >> 3) & 3;
  };
  auto issue = [&](int kc) {
    Gemm128Stage& st = sh.st[kc % kPipeSlots];
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      int rr, cq;
      coord(it, rr, cq);
      const int c = kc * kGChunk + 4 * cq;
      const uint32_t off = tile_off(rr, 4 * cq, RS, CS) >> 2;
      const int r = row0 + rr;
      const bool va = r < mrows && c < w;
      const float* sa = kAV ? Hb + (long long)(k + r) * n + k + c
                            : (MODE == MODE_WT ? Wsrc : Yb) + (long long)r * kOB + c;
      cp_async16(st.a_hi + off, va ? sa : Hb, va);
      if (MODE == MODE_WT && P.nsplit == 2)  // second row-split partial, parked in a_lo
        cp_async16(st.a_lo + off, va ? Wsrc + (long long)P.ncmax * kOB + (long long)r * kOB + c : Hb, va);
      const int j = col0 + rr;
      const bool vb = j < ncols && c < w;
      cp_async16(st.b_hi + off, vb ? Bsrc + (long long)j * kOB + c : Bsrc, vb);
      if (MODE == MODE_UPD && P.nsplit == 2)  // second row-split partial, parked in b_lo
        cp_async16(st.b_lo + off, vb ? Bsrc + (long long)P.ncmax * kOB + (long long)j * kOB + c : Bsrc, vb);
    }
  };
  auto split_inplace = [](float* hi, float* lo, uint32_t off) {
    const float4 x = *reinterpret_cast<const float4*>(hi + off);
    float4 h, l;
    split4(x, h, l);
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) = l;
  };

#pragma unroll
  for (int s = 0; s < kAhead; ++s) {
    issue(s);
    cp_async_commit();
  }
  for (int kc = 0; kc < NK; ++kc) {
    // Refill: stage kc + kAhead goes into the slot of stage kc - 2, once its MMAs are done.
    if (kc + kAhead < NK) {
      if (kc >= 2) ok = mbar_wait(&sh.mbar[(kc - 2) % kPipeSlots], (uint32_t)(((kc - 2) / kPipeSlots) & 1)) && ok;
      issue(kc + kAhead);
    }
    cp_async_commit();
    cp_async_wait<kAhead>();  // this thread's pieces of stage kc have landed
    Gemm128Stage& st = sh.st[kc % kPipeSlots];
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      int rr, cq;
      coord(it, rr, cq);
      const uint32_t off = tile_off(rr, 4 * cq, RS, CS) >> 2;
      if (kAV && row0 == 0) {
        // V is unit lower trapezoidal: rows <= column hold R in H.
        const int r = rr, c = kc * kGChunk + 4 * cq;
        float4 x = *reinterpret_cast<const float4*>(st.a_hi + off);
        x.x = (r > c) ? x.x : (r == c ? 1.f : 0.f);
        x.y = (r > c + 1) ? x.y : (r == c + 1 ? 1.f : 0.f);
        x.z = (r > c + 2) ? x.z : (r == c + 2 ? 1.f : 0.f);
        x.w = (r > c + 3) ? x.w : (r == c + 3 ? 1.f : 0.f);
        if (c >= w) x = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(st.a_hi + off) = x;
      }
      if (MODE == MODE_WT && P.nsplit == 2) {  // W^T = partial 0 + partial 1, then split
        const float4 x0 = *reinterpret_cast<const float4*>(st.a_hi + off);
        const float4 x1 = *reinterpret_cast<const float4*>(st.a_lo + off);
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        x.x += x0.x; x.y += x0.y; x.z += x0.z; x.w += x0.w;
        x.x += x1.x; x.y += x1.y; x.z += x1.z; x.w += x1.w;
        float4 h, l;
        split4(x, h, l);
        *reinterpret_cast<float4*>(st.a_hi + off) = h;
        *reinterpret_cast<float4*>(st.a_lo + off) = l;
      } else {
        split_inplace(st.a_hi, st.a_lo, off);
      }
      if (MODE == MODE_UPD && P.nsplit == 2) {  // W = partial 0 + partial 1, then split
        const float4 x0 = *reinterpret_cast<const float4*>(st.b_hi + off);
        const float4 x1 = *reinterpret_cast<const float4*>(st.b_lo + off);
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        x.x += x0.x; x.y += x0.y; x.z += x0.z; x.w += x0.w;
        x.x += x1.x; x.y += x1.y; x.z += x1.z; x.w += x1.w;
        float4 h, l;
        split4(x, h, l);
        *reinterpret_cast<float4*>(st.b_hi + off) = h;
        *reinterpret_cast<float4*>(st.b_lo + off) = l;
      } else {
        split_inplace(st.b_hi, st.b_lo, off);
      }
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
      mma_commit(&sh.mbar[kc % kPipeSlots]);
    }
  }
  cp_async_wait<0>();
  // Epilogue: warp w owns tile rows 32 w .. 32 w + 31 (its TMEM lanes). Each 32-column chunk of
  // the product goes through a padded shared tile (the operand ring is free once the last MMA
  // is done), so that global traffic runs along rows: lane l handles row 4 i + (l >> 3),
  // columns 4 (l & 7) .. + 3, and one warp access covers four whole 128-byte rows instead of
  // 32 partial ones. The next chunk's C is in flight while the current one is processed.
  const int lane = tid & 31, lr = lane >> 3, lq = lane & 7;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  float* __restrict__ Ho = P.Hout + (long long)bidx * hob;
  constexpr int kPad = 36;  // row stride of the staging tile (floats): conflict-free float4 rows
  float* stg = reinterpret_cast<float*>(&sh.st[0]) + warp * (32 * kPad);
  auto load_chunk = [&](int q, float4 (&cv)[8]) {
    const int c = col0 + q * 32 + 4 * lq;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = row0 + 32 * warp + 4 * i + lr;
      cv[i] = (kUpd && r < m && c < ncols)
                  ? *reinterpret_cast<const float4*>(Sb + (long long)(k + r) * ldc + ccol + c)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  float4 cA[8], cB[8];
  if (kUpd) load_chunk(0, cA);
  {
    const int last = NK - 1;
    ok = mbar_wait(&sh.mbar[last % kPipeSlots], (uint32_t)((last / kPipeSlots) & 1)) && ok;
  }
  tc_fence_after();
  __syncthreads();  // every warp is past its ring reads (splits) before any staging write
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float pv[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + q * 32, pv);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      *reinterpret_cast<float4*>(stg + lane * kPad + 4 * e) = make_float4(pv[4 * e], pv[4 * e + 1], pv[4 * e + 2], pv[4 * e + 3]);
    __syncwarp();
    float4 (&cur)[8] = (q & 1) ? cB : cA;
    float4 (&nxt)[8] = (q & 1) ? cA : cB;
    if (kUpd && q + 1 < 4) load_chunk(q + 1, nxt);
    const int c = col0 + q * 32 + 4 * lq;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rl = 4 * i + lr, r = row0 + 32 * warp + rl;
      const float4 p = *reinterpret_cast<const float4*>(stg + rl * kPad + 4 * lq);
      if (!ok || r >= mrows || c >= ncols) continue;
      if (kStore) {
        *reinterpret_cast<float4*>(P.Y + (long long)bidx * P.y_bstride + (long long)r * kOB + c) = p;
      } else {
        *reinterpret_cast<float4*>(Ho + (long long)(k + r) * ldc + ccol + c) =
            make_float4(cur[i].x - p.x, cur[i].y - p.y, cur[i].z - p.z, cur[i].w - p.w);
      }
    }
    __syncwarp();  // the staging rows are read before the next chunk overwrites them
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// ---------------------------------------------------------------------------------------
// W^T = C^T V (or the Gram G = V^T V) over one row split, as tc_vtcw_kernel (wy_tc128.cuh),
// with the rows streamed by cp.async straight into the SW128_32B operand layout and split in
// place (V masked to its unit lower trapezoid in the panel's first 128 rows). Same tiles and
// arithmetic, so results agree bit for bit.
// One K stage of the pipelined V^T C / Gram kernel: V first, then C (the Gram reads V as both
// operands, so its C buffers shrink to a placeholder: 18 KB per stage instead of 32, four CTAs
// per SM). Every buffer starts on a 1 KB boundary.
template <int W, bool GRAM>
struct VtcwPipeStage {
  float v_hi[kWChunk * W];
  float v_lo[kWChunk * W];
  float c_hi[GRAM ? 256 : kWChunk * kTcCols];
  float c_lo[GRAM ? 256 : kWChunk * kTcCols];
};

template <int W, bool GRAM, int SLOTS>
struct VtcwPipeShared {
  VtcwPipeStage<W, GRAM> st[SLOTS];
  uint64_t mbar[SLOTS];
  uint32_t tmem;
};
template <int W, bool GRAM, int SLOTS>
constexpr size_t vtcw_pipe_smem() { return sizeof(VtcwPipeShared<W, GRAM, SLOTS>) + 1024; }

template <int W, bool GRAM, int SLOTS>
__global__ void __launch_bounds__(128) tc_vtcw_pipe_kernel(WyParams P) {
  constexpr int kAhead = SLOTS - 2;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  VtcwPipeShared<W, GRAM, SLOTS>& sh = *reinterpret_cast<VtcwPipeShared<W, GRAM, SLOTS>*>(align1024(smem_raw));
  constexpr uint32_t LBO = 512, SBO_C = (kTcCols / 32) * 512, SBO_V = (W / 32) * 512;
  constexpr int NV = W / 32;
  constexpr int NC = GRAM ? 0 : 4;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bidx = blockIdx.z, split = blockIdx.y;
  const int n = P.n, k = P.k, w = P.w, m = n - k;
  const int nc = GRAM ? w : P.cend - k - w;
  const int col0 = (GRAM ? 0 : P.coff) + blockIdx.x * kTcCols;
  const int ldc = P.ldc > 0 ? P.ldc : n, ccol = P.ldc > 0 ? P.ccol : k + w;
  const float* __restrict__ Hb = P.H + (long long)bidx * n * n;
  const float* __restrict__ Sb = P.src + (long long)bidx * P.src_bstride;
  const int r_begin = split * P.rows_per_split;
  const int r_end = min(m, r_begin + P.rows_per_split);
  const int nchunks = r_end > r_begin ? (r_end - r_begin + kWChunk - 1) / kWChunk : 0;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < SLOTS; ++s) mbar_init(&sh.mbar[s], 1);
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
  auto issue = [&](int ch) {
    VtcwPipeStage<W, GRAM>& st = sh.st[ch % SLOTS];
    const int r0 = r_begin + ch * kWChunk;
#pragma unroll
    for (int it = 0; it < NV; ++it) {
      int c, kk;
      v_coord(it, c, kk);
      const int r = r0 + kk;
      const bool ok_v = r < r_end && c < w;
      cp_async16(st.v_hi + (sw32_off(c, kk, LBO, SBO_V) >> 2), ok_v ? Hb + (long long)(k + r) * n + k + c : Hb, ok_v);
    }
#pragma unroll
    for (int it = 0; it < NC; ++it) {
      int mn, kk;
      c_coord(it, mn, kk);
      const int r = r0 + kk, col = col0 + mn;
      const bool ok_c = r < r_end && col < nc;
      cp_async16(st.c_hi + (sw32_off(mn, kk, LBO, SBO_C) >> 2),
                 ok_c ? Sb + (long long)(k + r) * ldc + ccol + col : Sb, ok_c);
    }
  };
  auto split_inplace = [](float* hi, float* lo, uint32_t off) {
    const float4 x = *reinterpret_cast<const float4*>(hi + off);
    float4 h, l;
    split4(x, h, l);
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) = l;
  };

#pragma unroll
  for (int s = 0; s < kAhead; ++s) {
    if (s < nchunks) issue(s);
    cp_async_commit();
  }
  for (int ch = 0; ch < nchunks; ++ch) {
    if (ch + kAhead < nchunks) {
      if (ch >= 2) ok = mbar_wait(&sh.mbar[(ch - 2) % SLOTS], (uint32_t)(((ch - 2) / SLOTS) & 1)) && ok;
      issue(ch + kAhead);
    }
    cp_async_commit();
    cp_async_wait<kAhead>();
    VtcwPipeStage<W, GRAM>& st = sh.st[ch % SLOTS];
    const int r0 = r_begin + ch * kWChunk;
#pragma unroll
    for (int it = 0; it < NV; ++it) {
      int c, kk;
      v_coord(it, c, kk);
      const uint32_t off = sw32_off(c, kk, LBO, SBO_V) >> 2;
      const int r = r0 + kk;
      if (r < c + 4) {  // unit lower trapezoid: R sits on and above the diagonal in H
        float4 x = *reinterpret_cast<const float4*>(st.v_hi + off);
        x.x = (c >= w) ? 0.f : ((r > c) ? x.x : (r == c ? 1.f : 0.f));
        x.y = (c + 1 >= w) ? 0.f : ((r > c + 1) ? x.y : (r == c + 1 ? 1.f : 0.f));
        x.z = (c + 2 >= w) ? 0.f : ((r > c + 2) ? x.z : (r == c + 2 ? 1.f : 0.f));
        x.w = (c + 3 >= w) ? 0.f : ((r > c + 3) ? x.w : (r == c + 3 ? 1.f : 0.f));
        if (r >= r_end) x = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(st.v_hi + off) = x;
      }
      split_inplace(st.v_hi, st.v_lo, off);
    }
#pragma unroll
    for (int it = 0; it < NC; ++it) {
      int mn, kk;
      c_coord(it, mn, kk);
      split_inplace(st.c_hi, st.c_lo, sw32_off(mn, kk, LBO, SBO_C) >> 2);
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ach = smem_u32(GRAM ? st.v_hi : st.c_hi), acl = smem_u32(GRAM ? st.v_lo : st.c_lo);
      const uint32_t sbo_a = GRAM ? SBO_V : SBO_C;
      const uint32_t bvh = smem_u32(st.v_hi), bvl = smem_u32(st.v_lo);
#pragma unroll
      for (int ks = 0; ks < kWChunk / 8; ++ks) {
        mma_tf32x3(tmem, make_sdesc_sw32(ach + ks * 2 * sbo_a, LBO, sbo_a), make_sdesc_sw32(acl + ks * 2 * sbo_a, LBO, sbo_a),
                   make_sdesc_sw32(bvh + ks * 2 * SBO_V, LBO, SBO_V), make_sdesc_sw32(bvl + ks * 2 * SBO_V, LBO, SBO_V),
                   idesc, ch > 0 || ks > 0);
      }
      mma_commit(&sh.mbar[ch % SLOTS]);
    }
  }
  cp_async_wait<0>();
  if (nchunks > 0) {
    const int last = nchunks - 1;
    ok = mbar_wait(&sh.mbar[last % SLOTS], (uint32_t)((last / SLOTS) & 1)) && ok;
  }
  tc_fence_after();
  __syncthreads();  // every warp is past its stage reads before any staging write
  // Output row `col` (W floats) belongs to thread col - col0, i.e. to the TMEM lane of warp
  // (col - col0) / 32. Each 32-float chunk of a warp's 32 rows goes through a padded shared
  // tile so that lane l stores row 4 i + (l >> 3), floats 4 (l & 7) .. + 3: one warp store
  // covers four whole 128-byte rows instead of 32 partial ones.
  const int lr = lane >> 3, lq = lane & 7;
  constexpr int kPad = 36;
  float* stg = reinterpret_cast<float*>(&sh.st[0]) + warp * (32 * kPad);
  const int ncol = GRAM ? W : nc;
  float* outb = P.Wp + ((long long)bidx * P.nsplit + split) * P.ncmax * W;
#pragma unroll 1
  for (int q = 0; q < W / 32; ++q) {
    float wv[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + q * 32, wv);
    if (nchunks == 0 || !ok) {
#pragma unroll
      for (int i = 0; i < 32; ++i) wv[i] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e)
      *reinterpret_cast<float4*>(stg + lane * kPad + 4 * e) = make_float4(wv[4 * e], wv[4 * e + 1], wv[4 * e + 2], wv[4 * e + 3]);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rl = 4 * i + lr, col = col0 + 32 * warp + rl;
      if (col < ncol)
        *reinterpret_cast<float4*>(outb + (long long)col * W + q * 32 + 4 * lq) =
            *reinterpret_cast<const float4*>(stg + rl * kPad + 4 * lq);
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, W);
}

// ---------------------------------------------------------------------------------------
// W2 = T^T sum_s Wp[s] for partials stored transposed (Wp[s][col][0..32), as
// tc_vtcw_pipe_kernel<32, ...> writes them): 32 columns per CTA. Thread (column tid >> 3, row
// quad tid & 7) adds its float4 of every split (eight lanes read one whole 128-byte row), in
// split order; then the T^T product as wy_tw2_kernel.
__global__ void __launch_bounds__(256) wy_tw2t_kernel(WyParams P) {
  griddep_launch_wait();
  __shared__ float Ts[32][33];
  __shared__ float Ws[32][33];
  const int bidx = blockIdx.y;
  const int nc = P.cend - P.k - P.w;
  const int tid = threadIdx.x;
  const float* Tb = P.T + (long long)bidx * P.t_bstride;
  float tv[4];
#pragma unroll
  for (int it = 0; it < 4; ++it) tv[it] = Tb[it * 256 + tid];
  {
    const int cl = tid >> 3, g = tid & 7;
    const int col = P.coff + blockIdx.x * 32 + cl;
    float4 wv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (col < nc) {
      const float* W0 = P.Wp + ((long long)bidx * P.nsplit * P.ncmax + col) * 32 + 4 * g;
      const long long sstride = 32LL * P.ncmax;
      int s = 0;
      for (; s + 4 <= P.nsplit; s += 4) {
        float4 x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = *reinterpret_cast<const float4*>(W0 + (s + u) * sstride);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          wv.x += x[u].x; wv.y += x[u].y; wv.z += x[u].z; wv.w += x[u].w;
        }
      }
      for (; s < P.nsplit; ++s) {
        const float4 x = *reinterpret_cast<const float4*>(W0 + s * sstride);
        wv.x += x.x; wv.y += x.y; wv.z += x.z; wv.w += x.w;
      }
    }
    Ws[4 * g + 0][cl] = wv.x;
    Ws[4 * g + 1][cl] = wv.y;
    Ws[4 * g + 2][cl] = wv.z;
    Ws[4 * g + 3][cl] = wv.w;
  }
#pragma unroll
  for (int it = 0; it < 4; ++it) Ts[(it * 256 + tid) >> 5][tid & 31] = tv[it];
  __syncthreads();
  const int c = tid & 31, g = tid >> 5;
  const int col = P.coff + blockIdx.x * 32 + c;
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

}  // namespace qrb200
