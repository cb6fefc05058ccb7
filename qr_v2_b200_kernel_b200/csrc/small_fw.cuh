// Fully fused QR of a small matrix (n <= NMAX <= 128), one CTA per matrix, the whole matrix in
// registers -- the one-CTA-per-matrix path of the reference's fused kernel
// (submission.py:72-175), restructured as a factor warp fed by update warps.
//
// The columns are cut into blocks of 4. Warp 0, the factor warp, runs the serial chain: for
// block t it takes the block (every earlier block reflector but the last already applied),
// applies the last one itself, factors the 4 columns with warp shuffles only (larfg/larf,
// submission.py:91-107, and the LARFT recurrence for the 4 x 4 T, :129-137), writes the
// finished block to H and publishes V_t and T_t in shared memory. Update warps own the later
// blocks (block t0 = u + 1, then t0 + NU when the matrix has that many) and apply each
// published block reflector to them (compact WY, C <- C - V T^T (V^T C),
// milestones/01_eager_official123203us.py:102-107), handing block t to the factor warp once
// V_0 .. V_{t-2} are in. Warps 4, 8, ... stay idle: warps share a scheduler when their indices
// agree mod 4, so the factor warp gets one of the four schedulers to itself.
//
// Hand-offs are counters in shared memory written with release and polled with acquire
// semantics: vcount (V blocks published; every V stays in shared memory, so a consumer can
// fall behind without holding up the factor warp) and bflag[2] (the block in each slot of the
// two-slot B ring; a slot is reused for block t + 2 only after V_t is out, i.e. after the factor
// warp has read block t). Every wait is bounded; on expiry the warp records a device status
// and leaves.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace qrb200 {

__device__ __forceinline__ int ld_acquire_cta(const int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_cta(int* p, int v) {
  asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

// Wait (all lanes) until *p >= v; false after 2^24 polls, with the device status set.
__device__ __forceinline__ bool fw_wait_geq(const int* p, int v) {
  for (uint32_t it = 0; it < (1u << 24); ++it)
    if (ld_acquire_cta(p) >= v) return true;
  report_device_failure(kSiteHandoff);
  return false;
}

// As fw_wait_geq, with a pause between polls (for warps off the critical path that share a
// scheduler with it); at most 2^20 polls of about 0.1 us.
__device__ __forceinline__ bool fw_wait_geq_sleep(const int* p, int v) {
  for (uint32_t it = 0; it < (1u << 20); ++it) {
    if (ld_acquire_cta(p) >= v) return true;
    __nanosleep(100);
  }
  report_device_failure(kSiteHandoff);
  return false;
}

// As fw_wait_geq with a short pause of ns nanoseconds between polls (update warps: fewer
// shared-memory polls competing with the factor warp); at most 2^22 polls.
__device__ __forceinline__ bool fw_wait_geq_pause(const int* p, int v, int ns) {
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    if (ld_acquire_cta(p) >= v) return true;
    __nanosleep(ns);
  }
  report_device_failure(kSiteHandoff);
  return false;
}

// Publish by lane 0 after every lane's shared-memory writes.
__device__ __forceinline__ void fw_publish(int* p, int v) {
  __threadfence_block();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) st_release_cta(p, v);
}

// Factor-warp layout: lane l holds rows l + 32 i (i < RPL) of the block's CPW columns.
// Factor the block (global columns c0 ..); T (every lane holds all of it), tau written.
// J32: every pivot row is < 32 (a panel of at most 32 columns), so rows 32 i, i >= 1, are
// always below the pivot and register 0 holds the pivot row.
template <int CPW, int RPL, bool J32 = false>
__device__ __forceinline__ void fw_factor_block(float (&a)[CPW][RPL], const int c0, const int n, float (&Tw)[CPW][CPW],
                                                float* __restrict__ taub) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < CPW; ++k)
#pragma unroll
    for (int c = 0; c < CPW; ++c) Tw[k][c] = 0.f;
#pragma unroll
  for (int jj = 0; jj < CPW; ++jj) {
    const int j = c0 + jj;
    if (j >= n) break;
    const int ij = J32 ? 0 : (j >> 5), lj = j & 31;
    float xm[RPL];
#pragma unroll
    for (int i = 0; i < RPL; ++i) xm[i] = ((J32 && i > 0) || lane + 32 * i > j) ? a[jj][i] : 0.f;
    // d[CPW] carries the squared norm of the tail scaled by 2^100 through the same butterfly,
    // so the rare rescaled reflector needs no warp collective of its own (a shuffle inside a
    // data-dependent branch costs the hot path a convergence barrier).
    float d[CPW + 1], rowj[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < RPL; ++i) acc = fmaf(xm[i], c == jj ? xm[i] : a[c][i], acc);
      d[c] = acc;  // d[jj] = ||x||^2; c > jj: x . a_c; c < jj: x . v_c
      float t = a[c][0];
      if (!J32)
#pragma unroll
        for (int i = 1; i < RPL; ++i) t = (i == ij) ? a[c][i] : t;
      rowj[c] = t;
    }
    {
      float su = 0.f;
#pragma unroll
      for (int i = 0; i < RPL; ++i) {
        const float xu = xm[i] * kRescaleUp;
        su = fmaf(xu, xu, su);
      }
      d[CPW] = su;
    }
#pragma unroll
    for (int c = 0; c < CPW; ++c) rowj[c] = __shfl_sync(kFullMask, rowj[c], lj);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
      for (int c = 0; c <= CPW; ++c) d[c] += __shfl_xor_sync(kFullMask, d[c], o);
    const Reflector rf = make_reflector_fast(rowj[jj], d[jj], d[CPW]);
    float z[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      z[c] = fmaf(rf.scale, d[c], rowj[c]);  // v_j . a_c (c > jj) or v_c . v_j (c < jj)
      if (c > jj) {
        const float f = rf.tau * z[c];
        const float fs = f * rf.scale;
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          a[c][i] = fmaf(-fs, xm[i], a[c][i]);
          if ((!J32 || i == 0) && lane + 32 * i == j) a[c][i] -= f;
        }
      }
    }
#pragma unroll
    for (int c = 0; c < jj; ++c) {
      float t = 0.f;
#pragma unroll
      for (int k = c; k < jj; ++k) t = fmaf(Tw[c][k], z[k], t);
      Tw[c][jj] = -rf.tau * t;
    }
    Tw[jj][jj] = rf.tau;
#pragma unroll
    for (int i = 0; i < RPL; ++i) {
      const int r = lane + 32 * i;
      a[jj][i] = (J32 && i > 0) ? xm[i] * rf.scale : ((r > j) ? xm[i] * rf.scale : (r == j ? rf.diag : a[jj][i]));
    }
    if (lane == 0) taub[j] = rf.tau;
  }
}

// Factor-warp layout: a <- (I - V T V^T)^T a, V (masked: unit diagonal, zeros above;
// [column][row]) and T (row-major) in shared memory. The 16 partial products W[cp][c] are
// summed across the warp with a transposed butterfly (each xor step halves the live values:
// 16 shuffles instead of 80), then broadcast back from the lanes that hold them.
template <int NMAX, int CPW, int RPL>
__device__ __forceinline__ void fw_apply_cols(float (&a)[CPW][RPL], const float* __restrict__ Vs,
                                              const float* __restrict__ Ts) {
  static_assert(CPW == 4, "transposed reduction assumes 4 x 4 products");
  const int lane = threadIdx.x & 31;
  float vm[CPW][RPL];
#pragma unroll
  for (int cp = 0; cp < CPW; ++cp)
#pragma unroll
    for (int i = 0; i < RPL; ++i) vm[cp][i] = Vs[cp * NMAX + lane + 32 * i];
  float p[16];  // p[4 cp + c] = this lane's share of V[:, cp] . a[:, c]
#pragma unroll
  for (int cp = 0; cp < CPW; ++cp)
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < RPL; ++i) acc = fmaf(vm[cp][i], a[c][i], acc);
      p[cp * CPW + c] = acc;
    }
  // Steps o = 16, 8, 4, 2 keep the half of the values selected by the lane's bit; after them
  // lane l holds value ((l >> 1) & 15) summed over 16 lanes, and o = 1 completes the sum.
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
  // Value v sits in the lanes whose bits 4..1 spell v: bit 4 chose the upper half first, so
  // v = 8 b4 + 4 b3 + 2 b2 + b1.
  float W[CPW][CPW];
#pragma unroll
  for (int v = 0; v < 16; ++v) W[v / CPW][v % CPW] = __shfl_sync(kFullMask, p[0], 2 * v);
#pragma unroll
  for (int c = 0; c < CPW; ++c)
#pragma unroll
    for (int cp = 0; cp < CPW; ++cp) {
      float y = 0.f;
#pragma unroll
      for (int k = 0; k <= cp; ++k) y = fmaf(Ts[k * CPW + cp], W[k][c], y);
#pragma unroll
      for (int i = 0; i < RPL; ++i) a[c][i] = fmaf(-vm[cp][i], y, a[c][i]);
    }
}

// Volatile shared float4 load: issued where it stands, so a long unrolled loop does not hoist
// all of its loads ahead of the arithmetic (which would need a register per loaded value).
__device__ __forceinline__ float4 lds4_inorder(const float* p) {
  float4 v;
  asm volatile("ld.volatile.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

// Update-warp layout: lane 4 g + c holds column c, rows 32 q + 4 g + e (q < RPG / 4, e < 4) in
// x[4 q + e]. The dot products V^T x reduce over the 8 lanes of a column (3 shuffle levels), and
// the 8 row groups of one float4 load are 8 consecutive 16-byte pieces (no bank conflicts).
template <int NMAX, int CPW, int RPG>
__device__ __forceinline__ void fw_apply_rows(float (&x)[RPG], const float* __restrict__ Vs,
                                              const float* __restrict__ Ts, int g4) {
  float W[CPW];
#pragma unroll
  for (int cp = 0; cp < CPW; ++cp) W[cp] = 0.f;
#pragma unroll
  for (int k = 0; k < RPG; k += 4) {
#pragma unroll
    for (int cp = 0; cp < CPW; ++cp) {
      const float4 v = lds4_inorder(Vs + cp * NMAX + 8 * k + g4);
      W[cp] = fmaf(v.x, x[k], W[cp]);
      W[cp] = fmaf(v.y, x[k + 1], W[cp]);
      W[cp] = fmaf(v.z, x[k + 2], W[cp]);
      W[cp] = fmaf(v.w, x[k + 3], W[cp]);
    }
  }
#pragma unroll
  for (int o = 4; o <= 16; o <<= 1)
#pragma unroll
    for (int cp = 0; cp < CPW; ++cp) W[cp] += __shfl_xor_sync(kFullMask, W[cp], o);
  float Y[CPW];
#pragma unroll
  for (int cp = 0; cp < CPW; ++cp) {
    float y = 0.f;
#pragma unroll
    for (int k = 0; k <= cp; ++k) y = fmaf(Ts[k * CPW + cp], W[k], y);
    Y[cp] = y;
  }
#pragma unroll
  for (int k = 0; k < RPG; k += 4) {
#pragma unroll
    for (int cp = 0; cp < CPW; ++cp) {
      const float4 v = lds4_inorder(Vs + cp * NMAX + 8 * k + g4);
      x[k] = fmaf(-v.x, Y[cp], x[k]);
      x[k + 1] = fmaf(-v.y, Y[cp], x[k + 1]);
      x[k + 2] = fmaf(-v.z, Y[cp], x[k + 2]);
      x[k + 3] = fmaf(-v.w, Y[cp], x[k + 3]);
    }
  }
}

template <int NMAX, int CPW>
struct __align__(16) SmallFwShared {
  float V[NMAX / CPW][CPW][NMAX];  // every block's masked V ([column][row])
  float T[NMAX / CPW][CPW][CPW];
  float B[2][CPW][NMAX];           // blocks on their way to the factor warp
  int vcount, bflag[2];
};

template <int NMAX>
constexpr size_t small_fw_smem() { return sizeof(SmallFwShared<NMAX, 4>); }

// NWL warps are launched: the factor warp, idle warps 4, 8, .. and NU update warps.
template <int NMAX, int NWL>
__global__ void __launch_bounds__(32 * NWL) small_fw_kernel(const float* __restrict__ A, long long a_bstride,
                                                            float* __restrict__ H, float* __restrict__ tau, int n,
                                                            int P_SLEEP_NS = 0) {
  constexpr int CPW = 4;
  constexpr int RPL = NMAX / 32;               // factor-warp rows per lane
  constexpr int RPG = NMAX / 8;                // update-warp rows per lane
  constexpr int NU = NWL - 1 - (NWL - 1) / 4;  // update warps: w % 4 != 0
  extern __shared__ __align__(16) unsigned char fw_smem_raw[];
  SmallFwShared<NMAX, CPW>& sh = *reinterpret_cast<SmallFwShared<NMAX, CPW>*>(fw_smem_raw);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int nb = (n + CPW - 1) / CPW;  // blocks
  const int b = blockIdx.x;
  const float* __restrict__ Ab = A + (long long)b * a_bstride;
  float* __restrict__ Hb = H + (long long)b * n * n;
  float* __restrict__ taub = tau + (long long)b * n;
  const bool vec = (n & 3) == 0 && (a_bstride & 3) == 0 &&
                   ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(H)) & 15u) == 0;
  if (threadIdx.x == 0) {
    sh.vcount = 0;
    sh.bflag[0] = sh.bflag[1] = -1;
  }
  __syncthreads();

  if (w == 0) {
    // ---------------- factor warp ----------------
    float a[CPW][RPL];
#pragma unroll
    for (int i = 0; i < RPL; ++i) {
      const int r = lane + 32 * i;
      if (vec && r < n) {
        const float4 x = *reinterpret_cast<const float4*>(Ab + (long long)r * n);
        a[0][i] = x.x;
        a[1][i] = x.y;
        a[2][i] = x.z;
        a[3][i] = x.w;
      } else {
#pragma unroll
        for (int c = 0; c < CPW; ++c) a[c][i] = (r < n && c < n) ? Ab[(long long)r * n + c] : 0.f;
      }
    }
    // Block t's H store is issued after the wait for block t + 1, so that no global store is
    // in flight while the warp polls (the acquire poll would wait for it).
    float hprev[CPW][RPL];
    auto store_block = [&](int tb) {
      const int cb = tb * CPW;
#pragma unroll
      for (int i = 0; i < RPL; ++i) {
        const int r = lane + 32 * i;
        if (r >= n) continue;
        if (vec) {
          *reinterpret_cast<float4*>(Hb + (long long)r * n + cb) =
              make_float4(hprev[0][i], hprev[1][i], hprev[2][i], hprev[3][i]);
        } else {
#pragma unroll
          for (int c = 0; c < CPW; ++c)
            if (cb + c < n) Hb[(long long)r * n + cb + c] = hprev[c][i];
        }
      }
    };
    for (int t = 0; t < nb; ++t) {
      const int c0 = t * CPW;
      if (t >= 1) {
        const int sl = t & 1;
        if (!fw_wait_geq(&sh.bflag[sl], t)) return;
#pragma unroll
        for (int c = 0; c < CPW; ++c)
#pragma unroll
          for (int i = 0; i < RPL; ++i) a[c][i] = sh.B[sl][c][lane + 32 * i];
        store_block(t - 1);
        fw_apply_cols<NMAX, CPW, RPL>(a, &sh.V[t - 1][0][0], &sh.T[t - 1][0][0]);  // V_{t-1}
      }
      float Tw[CPW][CPW];
      fw_factor_block<CPW, RPL>(a, c0, n, Tw, taub);
      if (t + 1 < nb) {  // publish V_t (masked) and T_t
#pragma unroll
        for (int c = 0; c < CPW; ++c)
#pragma unroll
          for (int i = 0; i < RPL; ++i) {
            const int r = lane + 32 * i;
            sh.V[t][c][r] = (r > c0 + c) ? a[c][i] : (r == c0 + c ? 1.f : 0.f);
          }
        if (lane == 0)
#pragma unroll
          for (int k = 0; k < CPW; ++k)
#pragma unroll
            for (int c = 0; c < CPW; ++c) sh.T[t][k][c] = Tw[k][c];
        fw_publish(&sh.vcount, t + 1);
      }
#pragma unroll
      for (int c = 0; c < CPW; ++c)
#pragma unroll
        for (int i = 0; i < RPL; ++i) hprev[c][i] = a[c][i];
    }
    store_block(nb - 1);
    return;
  }
  if ((w & 3) == 0) return;  // idle: keeps the factor warp's scheduler free

  // ---------------- update warps ----------------
  const int u = w - (w >> 2) - 1;  // 0 .. NU-1
  const int g4 = 4 * (lane >> 2), cc = lane & 3;
  for (int t = 1 + u; t < nb; t += NU) {
    float x[RPG];
    const int col = t * CPW + cc;
#pragma unroll
    for (int k = 0; k < RPG; ++k) {
      const int r = 8 * (k & ~3) + g4 + (k & 3);
      x[k] = (r < n && col < n) ? Ab[(long long)r * n + col] : 0.f;
    }
    for (int s = 0; s <= t - 2; ++s) {
      if (!(P_SLEEP_NS > 0 ? fw_wait_geq_pause(&sh.vcount, s + 1, P_SLEEP_NS) : fw_wait_geq(&sh.vcount, s + 1))) return;
      fw_apply_rows<NMAX, CPW, RPG>(x, &sh.V[s][0][0], &sh.T[s][0][0], g4);
    }
    // Slot t & 1 last held block t - 2, which the factor warp read before publishing V_{t-2}:
    // the wait for V_{t-2} above already covers its reuse.
    const int sl = t & 1;
#pragma unroll
    for (int k = 0; k < RPG; k += 4)
      *reinterpret_cast<float4*>(&sh.B[sl][cc][8 * k + g4]) = make_float4(x[k], x[k + 1], x[k + 2], x[k + 3]);
    fw_publish(&sh.bflag[sl], t);
  }
}

}  // namespace qrb200
