// Shared device helpers for the qrb200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace qrb200 {

constexpr unsigned kFullMask = 0xffffffffu;

// Named CTA barriers (id 0 is __syncthreads): bar.sync waits for nthreads arrivals, bar.arrive
// adds this warp's arrival without waiting.
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream be scheduled now, and wait
// until every kernel this one depends on has finished and its writes are visible. A kernel
// starts with both (before its first global read), so a launch with the programmatic
// serialisation attribute only overlaps launch latency; without that attribute they return at
// once.
__device__ __forceinline__ void griddep_launch_wait() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Transposed butterfly reduction of NV per-lane partial sums across a warp.
// On return d[0 .. NV/32) of lane L hold the warp-wide sums of the original entries
// L*(NV/32) + q. Each of the five xor steps halves the live array: the lane keeps the
// half selected by its own bit and adds the partner's copy of that half, so the whole
// reduction costs NV*31/32 shuffles instead of 5*NV for NV independent reductions.
template <int NV>
__device__ __forceinline__ void warp_transpose_reduce(float (&d)[NV], int lane) {
  static_assert(NV % 32 == 0, "NV must be a multiple of 32");
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    const int o = 16 >> step;
    const int half = (NV >> step) >> 1;
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int q = 0; q < half; ++q) {
      const float send = up ? d[q] : d[q + half];
      const float keep = up ? d[q + half] : d[q];
      d[q] = keep + __shfl_xor_sync(kFullMask, send, o);
    }
  }
}

// Householder reflector scalars for pivot alpha and squared tail norm xnorm2
// (LAPACK sign convention, no rescaling -- the same arithmetic as the reference panel).
struct Reflector {
  float diag;   // new diagonal: beta when a reflector is needed, alpha otherwise
  float tau;    // (beta - alpha) / beta, or 0
  float scale;  // 1 / (alpha - beta), or 0: v_tail = x * scale
};

// With nrm = ||(alpha, x)|| and beta = -sign(alpha) nrm the two quotients simplify to
//   tau   = (beta - alpha) / beta = 1 + |alpha| / nrm,
//   scale = 1 / (alpha - beta)    = sign(alpha) / (|alpha| + nrm),
// so the reflector needs one square root and two independent correctly rounded reciprocals
// (a ~100-cycle dependent chain instead of a square root and two IEEE divisions in series).
__device__ __forceinline__ Reflector make_reflector(float alpha, float xnorm2) {
  Reflector r;
  const float nrm = sqrtf(fmaf(alpha, alpha, xnorm2));
  const float aa = fabsf(alpha);
  const bool need = xnorm2 > 0.f;
  const float inv = __frcp_rn(aa + nrm);
  const float rn = __frcp_rn(nrm);
  r.diag = need ? (alpha >= 0.f ? -nrm : nrm) : alpha;
  r.tau = need ? fmaf(aa, rn, 1.f) : 0.f;
  r.scale = need ? (alpha >= 0.f ? inv : -inv) : 0.f;
  return r;
}

// Squared norms below 2^-100 (tail entries below about 2^-50) are sums of squares near or
// inside the subnormal range, which keep fewer than 24 bits: tau then disagrees with its
// vector and Q loses orthogonality. Such a reflector is rebuilt from the pivot and the squared
// norm of the tail scaled by 2^100 (xnorm2_up), the way LAPACK's slarfg rescales small
// columns. tau is scale invariant; diag scales down and scale up by the same power of two,
// both exactly. A column whose scaled scale still overflows (every entry subnormal) gets no
// reflector.
constexpr float kRescaleUp = 0x1p100f, kRescaleDown = 0x1p-100f;

// Out of line: the hot loops keep a plain branch to a call that ordinary inputs never take
// (inlined, the precise square root and reciprocals of this path slowed the reflector chain).
__device__ __noinline__ Reflector make_reflector_outside(float alpha, float xnorm2, float xnorm2_up) {
  if (fmaf(alpha, alpha, xnorm2) < kRescaleDown) {
    Reflector r = make_reflector(alpha * kRescaleUp, xnorm2_up);
    r.diag *= kRescaleDown;
    r.scale *= kRescaleUp;
    if (!(fabsf(r.scale) <= 3.0e38f)) {
      r.diag = alpha;
      r.tau = 0.f;
      r.scale = 0.f;
    }
    return r;
  }
  return make_reflector(alpha, xnorm2);
}

// Reflector scalars as make_reflector, with the square root and the reciprocal from the
// hardware approximations, the reciprocal square root refined by one Newton step
// (y <- y (3 - x y^2) / 2): about 1 ulp. Norms outside [1e-30, 1e30] take the correctly
// rounded path, where the approximations lose range, rescaled below 2^-100 (xnorm2_up: the
// squared norm of the tail times 2^200; pass any value when the caller has none, e.g. a
// cluster-wide norm of 513+ rows, whose sum stays accurate).
__device__ __forceinline__ bool reflector_fast_range(float alpha, float xnorm2) {
  const float nrm2 = fmaf(alpha, alpha, xnorm2);
  return nrm2 > 1e-30f && nrm2 < 1e30f;
}

// The fast form alone, for alpha^2 + xnorm2 inside [1e-30, 1e30].
__device__ __forceinline__ Reflector make_reflector_fast_core(float alpha, float xnorm2) {
  const float nrm2 = fmaf(alpha, alpha, xnorm2);
  float y = rsqrtf(nrm2);
  y = y * fmaf(-0.5f * nrm2, y * y, 1.5f);
  const float nrm = nrm2 * y;
  const float aa = fabsf(alpha);
  const float inv = __fdividef(1.f, aa + nrm);
  Reflector r;
  const bool need = xnorm2 > 0.f;
  r.diag = need ? (alpha >= 0.f ? -nrm : nrm) : alpha;
  r.tau = need ? fmaf(aa, y, 1.f) : 0.f;
  r.scale = need ? (alpha >= 0.f ? inv : -inv) : 0.f;
  return r;
}

__device__ __forceinline__ Reflector make_reflector_fast(float alpha, float xnorm2, float xnorm2_up) {
  const float nrm2 = fmaf(alpha, alpha, xnorm2);
  if (!(nrm2 > 1e-30f && nrm2 < 1e30f)) return make_reflector_outside(alpha, xnorm2, xnorm2_up);
  float y = rsqrtf(nrm2);
  y = y * fmaf(-0.5f * nrm2, y * y, 1.5f);
  const float nrm = nrm2 * y;
  const float aa = fabsf(alpha);
  const float inv = __fdividef(1.f, aa + nrm);
  Reflector r;
  const bool need = xnorm2 > 0.f;
  r.diag = need ? (alpha >= 0.f ? -nrm : nrm) : alpha;
  r.tau = need ? fmaf(aa, y, 1.f) : 0.f;
  r.scale = need ? (alpha >= 0.f ? inv : -inv) : 0.f;
  return r;
}

// Callers without the scaled sum (the owner and cluster panels): out of range, the correctly
// rounded form inline. The owner panel detects norms below 2^-100 itself and refactors the
// panel scaled; cluster panels (513+ rows per tail) keep the reference's arithmetic.
__device__ __forceinline__ Reflector make_reflector_fast(float alpha, float xnorm2) {
  if (!reflector_fast_range(alpha, xnorm2)) return make_reflector(alpha, xnorm2);
  return make_reflector_fast_core(alpha, xnorm2);
}

}  // namespace qrb200
