// Factor-warp building blocks (a warp that holds a block of 4 columns, lane l owning rows
// l + 32 i, forms the block's reflectors with warp shuffles only) and the fully fused QR of a
// small matrix (n <= 128) built from them: one CTA per matrix, the whole matrix on chip -- the
// one-CTA-per-matrix path of the reference's fused kernel (submission.py:72-175), restructured
// as two factor warps taking the 4-column blocks in turn, fed by update warps
// (small_pp_kernel, below). panel_fw.cuh builds its panels from the same pieces.
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


// ---------------------------------------------------------------------------------------
// Whole-matrix QR with two factor warps in turn (n <= NMAX <= 128, one CTA per matrix).
//
// Blocks of 4 columns go alternately to factor warp 0 (even blocks) and factor warp 1 (odd
// blocks). While one factor warp forms the reflectors of block t, the other already holds
// block t + 1 in its registers and applies each reflector of block t the moment it is
// published (x <- x - tau v (v^T x), one butterfly for the four dots), so when the last
// reflector of block t comes out, block t + 1 is one rank-one update away from being factored:
// the reflector chain never waits for a block to be handed over. Before that, the warp brings
// block t + 1 up to date through block t - 2 (its own block, whose reflectors it still holds
// in registers); the update warps deliver it with every block up to t - 3 applied (compact
// WY, C <- C - V T^T (V^T C), milestones/01_eager_official123203us.py:102-107) through a
// three-slot ring. larfg/larf and the 4 x 4 LARFT follow submission.py:91-107 / :129-137.
//
// The factor warps issue no global memory access inside the chain: reflectors, tau and the
// finished columns go to shared memory (a fence or release store waits for the thread's global
// stores in flight), and the whole H and tau are written out, coalesced, once every block is
// done. Reflectors pass between the factor warps with no flag and no fence: every reflector
// slot starts as a NaN pattern that arithmetic never produces (kPpEmpty) and the consumer polls
// the data itself. Block-level hand-offs are counters in shared memory written with release and
// polled with acquire semantics: vcount[f] (blocks of factor warp f whose V and T are complete,
// for the update warps) and bflag[3] (the block in each ring slot). Every wait is bounded; a
// wait that runs out records a device failure and raises `abort`, which every other wait
// checks, so the CTA reaches its final barrier and skips the output.
//
// Measured on B200 (C1: 8 matrices of 128 x 128): 57.3 us per call against 65.5 us for a single
// factor warp fed block by block (same box); ~700 cycles per reflector in the factor warp.
template <int NMAX>
struct __align__(16) SmallPpShared {
  float V[NMAX / 4][4][NMAX];  // every block's masked reflectors, [block][column][row]
  float T[NMAX / 4][4][4];     // every block's T (for the update warps)
  float B[3][4][NMAX];         // blocks delivered by the update warps, [slot][column][row]
  float Hs[NMAX][NMAX + 4];    // the finished factorisation, row-major (padding: conflict-free float4 rows)
  float tauv[NMAX];
  int vcount[2], bflag[3], abort;
};

template <int NMAX>
constexpr size_t small_pp_smem() { return sizeof(SmallPpShared<NMAX>); }

__device__ __forceinline__ int ld_volatile_int(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Wait until *p >= v (acquire). Returns false if `abort` was raised or after 2^24 polls, in
// which case the device failure is recorded and `abort` raised.
__device__ __forceinline__ bool pp_wait(const int* p, int v, int* abort, int pause_ns) {
  for (uint32_t it = 0; it < (1u << 24); ++it) {
    if (ld_acquire_cta(p) >= v) return true;
    if ((it & 63u) == 63u && ld_volatile_int(abort)) return false;
    if (pause_ns > 0) __nanosleep(pause_ns);
  }
  report_device_failure(kSiteHandoff);
  *reinterpret_cast<volatile int*>(abort) = 1;
  return false;
}

// Reflector slots (V and tau) start as this NaN pattern. Arithmetic never produces it (GPU
// arithmetic returns the canonical NaN), so a slot holding anything else holds its final value:
// each 32-bit store is single-copy atomic, and a consumer that polls the data itself needs no
// flag, and the producer no fence.
constexpr uint32_t kPpEmpty = 0x7fbadbadu;

__device__ __forceinline__ float ld_volatile_f(const float* p) { return *reinterpret_cast<const volatile float*>(p); }

// Wait until reflector j (its masked column vcol[row] and tau) is published, and load it: every
// lane polls its own rows (the rows the producer's lane of the same index wrote) and tau.
// False if `abort` was raised or after 2^24 polls (device failure recorded, `abort` raised).
template <int RPL>
__device__ __forceinline__ bool pp_wait_reflector(const float* vcol, const float* tptr, float (&v)[RPL], float& tj,
                                                  int* abort) {
  const int lane = threadIdx.x & 31;
  for (uint32_t it = 0; it < (1u << 24); ++it) {
    tj = ld_volatile_f(tptr);
    bool ready = __float_as_uint(tj) != kPpEmpty;
#pragma unroll
    for (int i = 0; i < RPL; ++i) {
      v[i] = ld_volatile_f(vcol + lane + 32 * i);
      ready = ready && (__float_as_uint(v[i]) != kPpEmpty);
    }
    if (__all_sync(kFullMask, ready)) return true;
    if ((it & 63u) == 63u && ld_volatile_int(abort)) return false;
  }
  report_device_failure(kSiteHandoff);
  *reinterpret_cast<volatile int*>(abort) = 1;
  return false;
}

// One block of 4 columns by a factor warp (lane l holds rows l + 32 i): larfg + larf per column
// (submission.py:91-107) and the block's T (LARFT, :129-137; every lane holds it). Reflector j's
// masked column goes to Vpub (if not null) and its tau to tauv[j] as soon as it is formed,
// without a fence (see kPpEmpty). FULL: all four columns exist (no bound check in the chain).
template <int RPL, bool FULL>
__device__ __forceinline__ void pp_factor_block(float (&a)[4][RPL], const int c0, const int n, float (&Tw)[4][4],
                                                float* __restrict__ tauv, float* __restrict__ Vpub) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int c = 0; c < 4; ++c) Tw[k][c] = 0.f;
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const int j = c0 + jj;
    if (!FULL && j >= n) break;
    const int ij = j >> 5, lj = j & 31;
    float xm[RPL];
#pragma unroll
    for (int i = 0; i < RPL; ++i) xm[i] = (lane + 32 * i > j) ? a[jj][i] : 0.f;
    // d[4] carries the squared norm of the tail scaled by 2^100 through the same butterfly
    // (the rescaled reflector of make_reflector_outside).
    float d[5], rowj[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < RPL; ++i) acc = fmaf(xm[i], c == jj ? xm[i] : a[c][i], acc);
      d[c] = acc;  // d[jj] = ||x||^2; c > jj: x . a_c; c < jj: x . v_c
      float t = a[c][0];
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
      d[4] = su;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) rowj[c] = __shfl_sync(kFullMask, rowj[c], lj);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
      for (int c = 0; c < 5; ++c) d[c] += __shfl_xor_sync(kFullMask, d[c], o);
    const Reflector rf = make_reflector_fast(rowj[jj], d[jj], d[4]);
    if (Vpub != nullptr) {
#pragma unroll
      for (int i = 0; i < RPL; ++i) {
        const int r = lane + 32 * i;
        Vpub[jj * 32 * RPL + r] = (r > j) ? xm[i] * rf.scale : (r == j ? 1.f : 0.f);
      }
    }
    if (lane == 0) tauv[j] = rf.tau;
    float z[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      z[c] = fmaf(rf.scale, d[c], rowj[c]);  // v_j . a_c (c > jj) or v_c . v_j (c < jj)
      if (c > jj) {
        const float f = rf.tau * z[c];
        const float fs = f * rf.scale;
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          a[c][i] = fmaf(-fs, xm[i], a[c][i]);
          if (lane + 32 * i == j) a[c][i] -= f;
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
      a[jj][i] = (r > j) ? xm[i] * rf.scale : (r == j ? rf.diag : a[jj][i]);
    }
  }
}

// a <- (I - tau v v^T) a for the four columns of a factor-warp block (v masked: zero above its
// pivot row, one on it).
template <int RPL>
__device__ __forceinline__ void pp_apply_reflector(float (&a)[4][RPL], const float (&v)[RPL], float tj) {
  float d[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float d0 = 0.f, d1 = 0.f;
#pragma unroll
    for (int i = 0; i < RPL; i += 2) {
      d0 = fmaf(v[i], a[c][i], d0);
      if (i + 1 < RPL) d1 = fmaf(v[i + 1], a[c][i + 1], d1);
    }
    d[c] = d0 + d1;
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
    for (int c = 0; c < 4; ++c) d[c] += __shfl_xor_sync(kFullMask, d[c], o);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float f = tj * d[c];
#pragma unroll
    for (int i = 0; i < RPL; ++i) a[c][i] = fmaf(-f, v[i], a[c][i]);
  }
}

// NW warps: factor warps 0 and 1 (schedulers 0 and 1), update warps w with w % 4 >= 2
// (schedulers 2 and 3); the others only join the write-out.
template <int NMAX, int NW>
__global__ void __launch_bounds__(32 * NW) small_pp_kernel(const float* __restrict__ A, long long a_bstride,
                                                           float* __restrict__ H, float* __restrict__ tau, int n,
                                                           int poll_ns) {
  constexpr int RPL = NMAX / 32;  // factor-warp rows per lane
  constexpr int RPG = NMAX / 8;   // update-warp rows per lane
  constexpr int NU = NW / 2;      // update warps
  extern __shared__ __align__(16) unsigned char pp_smem_raw[];
  SmallPpShared<NMAX>& sh = *reinterpret_cast<SmallPpShared<NMAX>*>(pp_smem_raw);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int nb = (n + 3) / 4;
  const float* __restrict__ Ab = A + (long long)blockIdx.x * a_bstride;
  float* __restrict__ Hb = H + (long long)blockIdx.x * n * n;
  float* __restrict__ taub = tau + (long long)blockIdx.x * n;
  const bool vec_in = (n & 3) == 0 && (a_bstride & 3) == 0 && (reinterpret_cast<uintptr_t>(A) & 15u) == 0;
  const bool vec_out = (n & 3) == 0 && (reinterpret_cast<uintptr_t>(H) & 15u) == 0;
  if (threadIdx.x == 0) {
    sh.vcount[0] = sh.vcount[1] = 0;
    sh.bflag[0] = sh.bflag[1] = sh.bflag[2] = -1;
    sh.abort = 0;
  }
  {
    const float e = __uint_as_float(kPpEmpty);
    float4* v4 = reinterpret_cast<float4*>(&sh.V[0][0][0]);
    for (int i = threadIdx.x; i < NMAX * NMAX / 4; i += 32 * NW) v4[i] = make_float4(e, e, e, e);
    for (int i = threadIdx.x; i < NMAX; i += 32 * NW) sh.tauv[i] = e;
  }
  __syncthreads();

  if (w < 2) {
    // ---------------- factor warp w: blocks w, w + 2, w + 4, ... ----------------
    // Raw block t (t <= 2 needs no update-warp work) in the factor-warp layout.
    auto load_raw = [&](float (&x)[4][RPL], int t) {
      const int c0 = 4 * t;
#pragma unroll
      for (int i = 0; i < RPL; ++i) {
        const int r = lane + 32 * i;
        if (vec_in && r < n) {
          const float4 q = *reinterpret_cast<const float4*>(Ab + (long long)r * n + c0);
          x[0][i] = q.x;
          x[1][i] = q.y;
          x[2][i] = q.z;
          x[3][i] = q.w;
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) x[c][i] = (r < n && c0 + c < n) ? Ab[(long long)r * n + c0 + c] : 0.f;
        }
      }
    };
    float a[4][RPL], hp[4][RPL];
    if (w < nb) load_raw(a, w);
    if (w == 0 && nb > 2) load_raw(hp, 2);  // block 2, parked in hp until block 0 is done
    bool ok = true;
    for (int t = w; t < nb && ok; t += 2) {
      const int c0 = 4 * t;
      if (t >= 2) {
        // (1) block t with every block up to t - 3 applied; hp <- block t - 2 (final values)
        float x[4][RPL];
        if (t == 2) {
          // after block 0, a holds block 2 (raw) and hp block 0 (final): see (5)
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < RPL; ++i) x[c][i] = a[c][i];
        } else {
          const int sl = t % 3;
          if (!pp_wait(&sh.bflag[sl], t, &sh.abort, 0)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < RPL; ++i) x[c][i] = sh.B[sl][c][lane + 32 * i];
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < RPL; ++i) hp[c][i] = a[c][i];
        }
        // (2) own block t - 2, reflector by reflector from registers
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = 4 * (t - 2) + jj;
          float v[RPL];
#pragma unroll
          for (int i = 0; i < RPL; ++i) {
            const int r = lane + 32 * i;
            v[i] = (r > j) ? hp[jj][i] : (r == j ? 1.f : 0.f);
          }
          pp_apply_reflector<RPL>(x, v, sh.tauv[j]);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < RPL; ++i) a[c][i] = x[c][i];
      }
      // (3) the other warp's block t - 1, each reflector as soon as it is published
      if (t >= 1) {
#pragma unroll 1
        for (int jj = 0; jj < 4; ++jj) {
          const int j = 4 * (t - 1) + jj;
          float v[RPL], tj;
          if (!pp_wait_reflector<RPL>(&sh.V[t - 1][jj][0], &sh.tauv[j], v, tj, &sh.abort)) {
            ok = false;
            break;
          }
          pp_apply_reflector<RPL>(a, v, tj);
        }
        if (!ok) break;
      }
      // (4) factor block t, publishing each reflector as it is formed
      float Tw[4][4];
      const bool more = t + 1 < nb;  // then block t has all four columns
      if (more)
        pp_factor_block<RPL, true>(a, c0, n, Tw, sh.tauv, &sh.V[t][0][0]);
      else
        pp_factor_block<RPL, false>(a, c0, n, Tw, sh.tauv, nullptr);
      if (more) {
        if (lane == 0)
#pragma unroll
          for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int c = 0; c < 4; ++c) sh.T[t][k][c] = Tw[k][c];
        fw_publish(&sh.vcount[w], t + 1);
      }
      // (5) the finished block to the shared copy of H
#pragma unroll
      for (int i = 0; i < RPL; ++i)
        *reinterpret_cast<float4*>(&sh.Hs[lane + 32 * i][c0]) = make_float4(a[0][i], a[1][i], a[2][i], a[3][i]);
      if (t == 0 && nb > 2) {
        // block 2 was parked in hp: swap so that a = block 2 (raw) and hp = block 0 below
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < RPL; ++i) {
            const float s = a[c][i];
            a[c][i] = hp[c][i];
            hp[c][i] = s;
          }
      }
    }
  } else if ((w & 3) >= 2) {
    // ---------------- update warps: block t gets every block up to t - 3 ----------------
    const int u = 2 * (w >> 2) + (w & 1);  // 0 .. NU - 1
    const int g4 = 4 * (lane >> 2), cc = lane & 3;
    for (int t = 3 + u; t < nb; t += NU) {
      float x[RPG];
      const int col = 4 * t + cc;
#pragma unroll
      for (int k = 0; k < RPG; ++k) {
        const int r = 8 * (k & ~3) + g4 + (k & 3);
        x[k] = (r < n && col < n) ? Ab[(long long)r * n + col] : 0.f;
      }
      bool ok = true;
      for (int s = 0; s <= t - 3; ++s) {
        if (!pp_wait(&sh.vcount[s & 1], s + 1, &sh.abort, poll_ns)) {
          ok = false;
          break;
        }
        fw_apply_rows<NMAX, 4, RPG>(x, &sh.V[s][0][0], &sh.T[s][0][0], g4);
      }
      if (!ok) break;
      // Slot t % 3 last held block t - 3, which its factor warp read before publishing
      // V_{t-3}; the last wait above acquired that publication.
      const int sl = t % 3;
#pragma unroll
      for (int k = 0; k < RPG; k += 4)
        *reinterpret_cast<float4*>(&sh.B[sl][cc][8 * k + g4]) = make_float4(x[k], x[k + 1], x[k + 2], x[k + 3]);
      fw_publish(&sh.bflag[sl], t);
    }
  }
  __syncthreads();
  if (ld_volatile_int(&sh.abort)) return;
  if (vec_out) {
    const int q = n >> 2;
    for (int idx = threadIdx.x; idx < n * q; idx += 32 * NW) {
      const int r = idx / q, c = 4 * (idx - r * q);
      *reinterpret_cast<float4*>(Hb + (long long)r * n + c) = *reinterpret_cast<const float4*>(&sh.Hs[r][c]);
    }
  } else {
    for (int idx = threadIdx.x; idx < n * n; idx += 32 * NW) {
      const int r = idx / n, c = idx - r * n;
      Hb[(long long)r * n + c] = sh.Hs[r][c];
    }
  }
  for (int j = threadIdx.x; j < n; j += 32 * NW) taub[j] = sh.tauv[j];
}

}  // namespace qrb200
