// Fully fused QR of a small matrix (n <= NMAX <= 128), one CTA per matrix, the whole matrix in
// registers -- the one-CTA-per-matrix path of the reference's fused kernel
// (submission.py:72-175), restructured as a factor warp fed by update warps.
//
// The columns are cut into blocks of 4. Warp 0, the factor warp, runs the serial chain: it takes
// block t with every earlier reflector already applied, factors its 4 columns with warp shuffles
// only (larfg/larf, submission.py:91-107, and the LARFT recurrence for the 4 x 4 T, :129-137) and
// publishes each reflector v_j and tau_j in shared memory the moment it is formed, then the
// block's T_t, and writes the finished block to H. Update warps own the later blocks (block
// t0 = u + 1, then t0 + NU when the matrix has that many). The update warp holding block t + 1
// applies V_0 .. V_{t-1} as block reflectors (compact WY, C <- C - V T^T (V^T C),
// milestones/01_eager_official123203us.py:102-107) as they are published, then the reflectors of
// block t one by one (x <- x - tau v (v^T x)) while the factor warp is still forming them, and
// hands the block over: when the factor warp finishes block t, block t + 1 is ready but for the
// last reflector's rank-one update, and the factor warp itself applies nothing. Warps 4, 8, ...
// stay idle: warps share a scheduler when their indices agree mod 4, so the factor warp gets one
// of the four schedulers to itself.
//
// Hand-offs are counters in shared memory written with release and polled with acquire
// semantics: rcount (reflectors published), vcount (blocks whose V and T are complete; every V
// stays in shared memory, so a consumer can fall behind without holding up the factor warp) and
// bflag[2] (the block in each slot of the two-slot B ring; a slot is reused for block t + 2 only
// after the factor warp has read block t, which precedes V_t). Every wait is bounded; on expiry
// the warp records a device failure and leaves.
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
// Vpub (may be null): [column][row] storage of the block's masked reflectors; each column's
// v_j and tau_j go there (and to tpub[j]) and *rcount is released to j + 1 as soon as the
// reflector is formed.
template <int CPW, int RPL, bool J32 = false>
__device__ __forceinline__ void fw_factor_block(float (&a)[CPW][RPL], const int c0, const int n, float (&Tw)[CPW][CPW],
                                                float* __restrict__ taub, float* Vpub = nullptr,
                                                float* tpub = nullptr, int* rcount = nullptr) {
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
    if (Vpub != nullptr) {
      constexpr int LD = 32 * RPL;
#pragma unroll
      for (int i = 0; i < RPL; ++i) {
        const int r = lane + 32 * i;
        Vpub[jj * LD + r] = (r > j) ? xm[i] * rf.scale : (r == j ? 1.f : 0.f);
      }
      if (lane == 0) tpub[j] = rf.tau;
      fw_publish(rcount, j + 1);
    }
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
      const float4 v = *reinterpret_cast<const float4*>(Vs + cp * NMAX + 8 * k + g4);
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
      const float4 v = *reinterpret_cast<const float4*>(Vs + cp * NMAX + 8 * k + g4);
      x[k] = fmaf(-v.x, Y[cp], x[k]);
      x[k + 1] = fmaf(-v.y, Y[cp], x[k + 1]);
      x[k + 2] = fmaf(-v.z, Y[cp], x[k + 2]);
      x[k + 3] = fmaf(-v.w, Y[cp], x[k + 3]);
    }
  }
}

// Update-warp layout: x <- (I - tau v v^T) x for one published reflector (v in shared memory,
// masked); the dot v^T x reduces over the 8 lanes of a column (3 shuffle levels).
template <int NMAX, int RPG>
__device__ __forceinline__ void fw_apply_reflector_rows(float (&x)[RPG], const float* __restrict__ v, float tau,
                                                        int g4) {
  float wv = 0.f;
#pragma unroll
  for (int k = 0; k < RPG; k += 4) {
    const float4 vv = *reinterpret_cast<const float4*>(v + 8 * k + g4);
    wv = fmaf(vv.x, x[k], wv);
    wv = fmaf(vv.y, x[k + 1], wv);
    wv = fmaf(vv.z, x[k + 2], wv);
    wv = fmaf(vv.w, x[k + 3], wv);
  }
#pragma unroll
  for (int o = 4; o <= 16; o <<= 1) wv += __shfl_xor_sync(kFullMask, wv, o);
  const float f = tau * wv;
#pragma unroll
  for (int k = 0; k < RPG; k += 4) {
    const float4 vv = *reinterpret_cast<const float4*>(v + 8 * k + g4);
    x[k] = fmaf(-vv.x, f, x[k]);
    x[k + 1] = fmaf(-vv.y, f, x[k + 1]);
    x[k + 2] = fmaf(-vv.z, f, x[k + 2]);
    x[k + 3] = fmaf(-vv.w, f, x[k + 3]);
  }
}

template <int NMAX, int CPW>
struct __align__(16) SmallFwShared {
  float V[NMAX / CPW][CPW][NMAX];  // every block's masked V ([column][row])
  float T[NMAX / CPW][CPW][CPW];
  float B[2][CPW][NMAX];           // blocks on their way to the factor warp
  float tauv[NMAX];                // tau of every published reflector
  int rcount, vcount, bflag[2];
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
    sh.rcount = 0;
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
      if (t >= 1) {  // block t arrives with every earlier reflector applied
        const int sl = t & 1;
        if (!fw_wait_geq(&sh.bflag[sl], t)) return;
#pragma unroll
        for (int c = 0; c < CPW; ++c)
#pragma unroll
          for (int i = 0; i < RPL; ++i) a[c][i] = sh.B[sl][c][lane + 32 * i];
        store_block(t - 1);
        // The last reflector of block t - 1 (v below its diagonal in hprev[CPW - 1], tau in
        // tauv): a <- a - tau v (v^T a), one butterfly for the four dots.
        const int jl = c0 - 1;
        const float tl = sh.tauv[jl];
        float vl[RPL];
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const int r = lane + 32 * i;
          vl[i] = (r > jl) ? hprev[CPW - 1][i] : (r == jl ? 1.f : 0.f);
        }
        float dl[CPW];
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
          float acc = 0.f;
#pragma unroll
          for (int i = 0; i < RPL; ++i) acc = fmaf(vl[i], a[c][i], acc);
          dl[c] = acc;
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
          for (int c = 0; c < CPW; ++c) dl[c] += __shfl_xor_sync(kFullMask, dl[c], o);
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
          const float f = tl * dl[c];
#pragma unroll
          for (int i = 0; i < RPL; ++i) a[c][i] = fmaf(-f, vl[i], a[c][i]);
        }
      }
      float Tw[CPW][CPW];
      const bool more = t + 1 < nb;  // a later block needs this one's reflectors
      fw_factor_block<CPW, RPL>(a, c0, n, Tw, taub, more ? &sh.V[t][0][0] : nullptr, sh.tauv, &sh.rcount);
      if (more) {  // publish T_t (V_t went out column by column)
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
    // Block t - 1 is being factored: apply its reflectors one by one as they come out, all but
    // the last, which the factor warp applies itself once it has the block.
#pragma unroll 1
    for (int jj = 0; jj < CPW - 1; ++jj) {
      const int j = (t - 1) * CPW + jj;
      if (j >= n) break;
      if (!fw_wait_geq(&sh.rcount, j + 1)) return;
      fw_apply_reflector_rows<NMAX, RPG>(x, &sh.V[t - 1][jj][0], sh.tauv[j], g4);
    }
    // Slot t & 1 last held block t - 2, which the factor warp read before it published the
    // first reflector of block t - 1: the waits above already cover its reuse.
    const int sl = t & 1;
#pragma unroll
    for (int k = 0; k < RPG; k += 4)
      *reinterpret_cast<float4*>(&sh.B[sl][cc][8 * k + g4]) = make_float4(x[k], x[k + 1], x[k + 2], x[k + 3]);
    fw_publish(&sh.bflag[sl], t);
  }
}

}  // namespace qrb200
