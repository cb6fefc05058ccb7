// tcgen05 / TMEM building blocks for sm_100a (inline PTX), used by the tensor-core
// compact-WY update.
//
// Shared-memory operand layout. Every operand tile is stored as 128-byte core matrices of
// 8 rows x 4 fp32 columns (row r of the core at byte 16*r, its 4 columns contiguous). Element
// (r, c) of a tile lives at
//     (r / 8) * RS + (c / 4) * CS + (r % 8) * 16 + (c % 4) * 4        (bytes)
// with RS / CS the byte strides between 8-row groups and 4-column groups. That single layout
// is the no-swizzle canonical layout of the UMMA descriptors in both majors:
//   * K-major operand with rows = M (or N) and columns = K:  SBO = RS, LBO = CS,
//     and one K = 8 step advances the start address by 2 * CS;
//   * MN-major operand with columns = M (or N) and rows = K: SBO = CS, LBO = RS,
//     and one K = 8 step advances the start address by RS.
// (The no-swizzle layout is used for K-major operands.)
//
// MN-major fp32/tf32 operands must use the 128-byte swizzle with 32-byte granularity
// (descriptor layout type 1, "SW128_32B"): atoms of 32 MN x 4 K elements (512 B), one 128-byte
// row per K index, the four 32-byte chunks of row k XOR-permuted by k % 4. Element (mn, k) of
// such a tile lives at
//     (mn / 32) * LBO + (k / 4) * SBO + (k % 4) * 128 + ((mn % 32) / 8 ^ k % 4) * 32 + (mn % 8) * 4
// with LBO / SBO the byte strides between MN atoms and K atoms (multiples of 512, tile base
// 1024-byte aligned); one K = 8 step advances the start address by 2 * SBO.
//
// FP32 accuracy from TF32 tensor cores (3xTF32, the split of Ootomo and Yokota 2022):
// x = hi + lo with hi = tf32_rna(x) (low 13 mantissa bits zero) and lo = x - hi (exact in
// fp32); A.B ~= A_hi.B_hi + A_hi.B_lo + A_lo.B_hi accumulated in FP32 in TMEM.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace qrb200 {

// Device-side failure reporting. A kernel whose bounded wait expires records the site of the
// wait (a code below, never 0) in g_device_status (device memory, read by the synchronous
// qrb200_device_status) and, once the host has registered it, in this device's word of a
// mapped pinned host array (g_status_mapped), which qrb200_last_status and the Python operator
// read without any CUDA call or synchronisation.
constexpr int kSiteMbarrier = 1;    // mbarrier wait of a tensor-core kernel (MMA or operand ring)
constexpr int kSiteHandoff = 2;     // hand-off flag of the whole-matrix kernel
constexpr int kSiteCluster = 3;     // partial-sum exchange of the cluster panel
constexpr int kSiteSelfTest = 4;    // qrb200_selftest_wait_timeout
__device__ int g_device_status = 0;
__device__ int* g_status_mapped = nullptr;

__device__ __noinline__ void report_device_failure(int site) {
  atomicExch(&g_device_status, site);
  int* h = g_status_mapped;
  if (h != nullptr) {
    *reinterpret_cast<volatile int*>(h) = site;
    __threadfence_system();
  }
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

constexpr int kTcCols = 128;  // trailing columns per CTA of the V^T C products (MMA M)

// First 1024-byte aligned address at or after p in shared memory (swizzled operand tiles).
__device__ __forceinline__ unsigned char* align1024(unsigned char* p) {
  const uint32_t s = smem_u32(p);
  return p + ((1024u - (s & 1023u)) & 1023u);
}

// cp.async: a 16-byte (or 4-byte) global -> shared copy that bypasses registers; an invalid
// piece copies nothing and zero-fills the destination.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Asks L2 to fetch the 128-byte line holding p (no register result, no ordering).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi/lo split of a float4 for the 3xTF32 products.
__device__ __forceinline__ void split4(const float4 x, float4& hi, float4& lo) {
  hi.x = tf32_rna(x.x); hi.y = tf32_rna(x.y); hi.z = tf32_rna(x.z); hi.w = tf32_rna(x.w);
  lo.x = x.x - hi.x; lo.y = x.y - hi.y; lo.z = x.z - hi.z; lo.w = x.w - hi.w;
}

// Byte offset of element (r, c) in the core-matrix tile layout.
__device__ __forceinline__ uint32_t tile_off(int r, int c, uint32_t RS, uint32_t CS) {
  return (uint32_t)(r >> 3) * RS + (uint32_t)(c >> 2) * CS + (uint32_t)(r & 7) * 16u + (uint32_t)(c & 3) * 4u;
}

// Byte offset of element (mn, k) in the SW128_32B MN-major layout.
__device__ __forceinline__ uint32_t sw32_off(int mn, int k, uint32_t LBO, uint32_t SBO) {
  return (uint32_t)(mn >> 5) * LBO + (uint32_t)(k >> 2) * SBO + (uint32_t)(k & 3) * 128u +
         (uint32_t)((((mn & 31) >> 3) ^ (k & 3)) << 5) + (uint32_t)(mn & 7) * 4u;
}

// UMMA shared-memory descriptor, no swizzle, sm_100 version field = 1.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for tcgen05
  return d;                // base offset 0, layout type 0 (no swizzle)
}

// Same descriptor with layout type 1 (SW128_32B, MN-major fp32 operands).
__device__ __forceinline__ uint64_t make_sdesc_sw32(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return make_sdesc(saddr, lbo, sbo) | ((uint64_t)1 << 61);
}

// Instruction descriptor for kind::tf32 with FP32 accumulation.
__host__ __device__ constexpr uint32_t make_idesc_tf32(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                                   // D format F32
         | (2u << 7)                                 // A format TF32
         | (2u << 10)                                // B format TF32
         | ((a_mn_major ? 1u : 0u) << 15)            // A major
         | ((b_mn_major ? 1u : 0u) << 16)            // B major
         | ((uint32_t)(N >> 3) << 17)                // N / 8
         | ((uint32_t)(M >> 4) << 24);               // M / 16
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n"
      :
      : "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}

// D += A_hi B_hi + A_hi B_lo + A_lo B_hi for one K = 8 step.
__device__ __forceinline__ void mma_tf32x3(uint32_t d_tmem, uint64_t a_hi, uint64_t a_lo, uint64_t b_hi,
                                           uint64_t b_lo, uint32_t idesc, bool accumulate) {
  mma_tf32(d_tmem, a_hi, b_hi, idesc, accumulate);
  mma_tf32(d_tmem, a_hi, b_lo, idesc, true);
  mma_tf32(d_tmem, a_lo, b_hi, idesc, true);
}

__device__ __forceinline__ void mma_commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :
               : "r"(smem_u32(mbar))
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" : : "r"(smem_u32(mbar)), "r"(count) : "memory");
}

// Bounded wait for phase `parity` of an mbarrier: false (and the failure recorded at `site`)
// if the phase did not complete within `limit` polls.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* mbar, uint32_t parity, uint32_t limit, int site) {
  const uint32_t addr = smem_u32(mbar);
  for (uint32_t it = 0; it < limit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  report_device_failure(site);
  return false;
}

// The tensor-core kernels' wait: 2^24 polls (on the order of a second).
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity) {
  return mbar_wait_limit(mbar, parity, 1u << 24, kSiteMbarrier);
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// TMEM allocation by one full warp; the base address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :
               : "r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" : : "r"(taddr), "r"(ncols) : "memory");
}

// 32 consecutive fp32 columns of the calling thread's TMEM lane (32x32b shape: warp w reads
// lanes 32*(w%4) .. +31; taddr carries the lane base in its upper 16 bits).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace qrb200
