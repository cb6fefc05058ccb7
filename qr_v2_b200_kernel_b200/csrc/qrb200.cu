// qrb200 C ABI: argument checking, workspace layout, the launch schedules and the device
// failure word.
//
// Schedules, chosen by the matrix order n only (so a matrix's result, bit for bit, does not
// depend on the batch it is factored in):
//   n <= 128          one CTA per matrix factors the whole matrix in one launch (small_fw);
//   129 <= n <= 1024  two-level: 128-column outer blocks of four 32-column panels, narrow FP32
//                     updates inside the block, one 128-wide tcgen05 (3xTF32) update of the
//                     trailing matrix per block, its far part on a look-ahead stream;
//   n >= 1025         single-level: 32-column panels (cluster panels above 512 rows), the next
//                     panel's columns updated on a high-priority stream (U1), the rest (U2) on
//                     a low-priority one beside the next panel;
//   rows not 16-byte aligned (n % 4 != 0 or an unaligned input): single-level, one stream.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "qrb200.h"
#include "panel.cuh"
#include "panel_fw.cuh"
#include "panel_cl.cuh"
#include "small_fw.cuh"
#include "wy_simt.cuh"
#include "wy_simt2.cuh"
#include "wy_u1.cuh"
#include "wy_tc128.cuh"
#include "wy_tc128p.cuh"
#include "wy_tc128t.cuh"
#include "apply_q.cuh"

namespace qrb200 {

constexpr int kNB = 32;              // panel width of the blocked path
constexpr int kPanelRows = 256;      // panel rows per CTA of a cluster (32 lanes x 8 rows)
constexpr int kMaxCluster = 16;      // non-portable cluster size (one GPC)
constexpr int kMaxN = kPanelRows * kMaxCluster;        // 4096
constexpr int kSmallN = 128;         // whole-matrix single-CTA path up to this order
constexpr int kMaxDevicesSm = 64;


// ---------------------------------------------------------------------------------------
// Launch accounting. Every kernel launch goes through LaunchScope, which counts it and,
// while a profiling call is active on this host thread, brackets it with CUDA events and
// records its algorithmic flops and bytes.
enum KernelKind {
  K_PANEL = 0, K_SMALL, K_VTC, K_TW, K_UPD,
  K_GRAM, K_TBUILD, K_YGEMM, K_VTC128, K_UPD128, K_U1, K_PANEL_CL, K_LARFT, K_FILL, K_TW128, K_NUM_KINDS
};
static const char* const kKindName[K_NUM_KINDS] = {"panel_factor", "small_whole_matrix", "wy_vtc", "wy_tw", "wy_upd",
                                                   "tc_gram", "tbuild", "tc_ygemm", "tc_vtc128", "tc_upd128",
                                                   "wy_u1", "panel_cluster", "larft_blocks", "fill_identity",
                                                   "tc_tw128"};
// 1 = tensor-core contraction (FLOP bound); 0 = FP32 SIMT, memory or latency bound. (wy_vtc
// counts the 32-wide V^T C, which runs on tcgen05 for wide updates but is HBM bound at K = 32.)
static const int kKindTensorBound[K_NUM_KINDS] = {0, 0, 0, 0, 0, 1, 0, 1, 1, 1, 0, 0, 0, 0, 1};

static std::atomic<long long> g_launches{0};

struct ProfRecord {
  int kind;
  cudaEvent_t start, stop;
  double flops, bytes;
};
struct ProfSession {
  cudaStream_t stream;
  std::vector<ProfRecord> recs;
};
static thread_local ProfSession* t_prof = nullptr;

struct LaunchScope {
  int kind;
  double flops, bytes;
  cudaEvent_t a = nullptr, b = nullptr;
  LaunchScope(int kd, double f, double by) : kind(kd), flops(f), bytes(by) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (t_prof) {
      cudaEventCreate(&a);
      cudaEventCreate(&b);
      cudaEventRecord(a, t_prof->stream);
    }
  }
  ~LaunchScope() {
    if (t_prof) {
      cudaEventRecord(b, t_prof->stream);
      t_prof->recs.push_back({kind, a, b, flops, bytes});
    }
  }
};

// Algorithmic work of one Householder panel (LAPACK xGEQR2 count) per matrix.
static double panel_flops(double m, double w) { return 2.0 * m * w * w - 2.0 * w * w * w / 3.0; }

static inline int cdiv(long long a, long long b) { return (int)((a + b - 1) / b); }
static inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Row splits of the V^T C product for panel k. A function of the panel height only, so a
// matrix's arithmetic (and therefore its result, bit for bit) does not depend on how many
// other matrices share the call -- batch shards on several GPUs reproduce one GPU exactly.
constexpr int kRowsPerSplit = 256;
static int choose_nsplit(long long /*batch*/, int n, int k, int w) {
  const int m = n - k, nc = n - k - w;
  if (nc <= 0) return 1;
  return std::max(1, cdiv(m, kRowsPerSplit));
}

static int max_nsplit(long long batch, int n) {
  int mx = 1;
  for (int k = 0; k < n; k += kNB) {
    const int w = std::min(kNB, n - k);
    mx = std::max(mx, choose_nsplit(batch, n, k, w));
  }
  return mx;
}

struct Workspace {
  float* T;     // single-level: batch x 32 x 32; two-level: panel factors batch x 4 x 32 x 32
  float* Wp;    // single-level / narrow-update partials: batch x nsplit x 32 x ncmax
  float* W2;    // batch x 32 x ncmax
  float* Tob;   // two-level: batch x 128 x 128 outer-block factors, stored transposed (even blocks)
  float* Tob2;  // the same, odd outer blocks (the far update of a block still reads its factor
                // while the next block's factor is assembled)
  float* Gp;    // two-level: batch x nsplit_g x 128 x 128 Gram partials
  float* Y;     // two-level: batch x n x 128, W'^T = (T^T V^T C)^T of the even outer blocks
                // (row = trailing column); Y = V T^T for the accuracy diagnostic
  float* Y2;    // two-level: same, odd outer blocks (look-ahead keeps two blocks' buffers alive)
  float* Wf;    // two-level: batch x nsplit_f x n x 128 (W^T partials of the wide update)
  size_t bytes;
};

constexpr int kRowsPerSplitWide = 512;  // row split of the 128-wide products (panel height only)

// Two-level (128-column outer blocks on the tensor cores) for 129 <= n <= 1024 with rows
// 16-byte aligned; single-level with look-ahead from kSingleMinN on (the choice depends on the
// order only, so results do not depend on the batch).
constexpr int kSingleMinN = 1025;
static bool use_two_level(int n, const float* A, long long abs) {
  return n > kOB && (n % 4) == 0 && (abs % 4) == 0 && (reinterpret_cast<uintptr_t>(A) & 15u) == 0;
}
static bool use_single_la(int n) { return n >= kSingleMinN; }

static Workspace layout(long long batch, int n, void* base) {
  Workspace ws{};
  auto carve = [&](size_t bytes) {
    const size_t off = ws.bytes;
    ws.bytes += align_up(bytes, 256);
    return reinterpret_cast<float*>(static_cast<char*>(base) + off);
  };
  if (n <= kSmallN) return ws;
  const size_t f = sizeof(float);
  const int ns = max_nsplit(batch, n);
  ws.T = carve((size_t)batch * 4 * kNB * kNB * f);
  ws.Wp = carve((size_t)batch * ns * kNB * (size_t)n * f);
  ws.W2 = carve((size_t)batch * kNB * (size_t)n * f);
  // Wide-update buffers (sized for the largest n; unused on the single-level path).
  const int nsw = cdiv(n, kRowsPerSplitWide);
  ws.Tob = carve((size_t)batch * kOB * kOB * f);
  ws.Tob2 = carve((size_t)batch * kOB * kOB * f);
  ws.Gp = carve((size_t)batch * nsw * kOB * kOB * f);
  ws.Y = carve((size_t)batch * n * kOB * f);
  ws.Y2 = carve((size_t)batch * n * kOB * f);
  ws.Wf = carve((size_t)batch * nsw * (size_t)n * kOB * f);
  return ws;
}

// Function attributes (shared-memory opt-in, cluster size) belong to each device's instance of
// a kernel, so one-time set-up is tracked per device ordinal (devices >= 64 redo it every call).
struct PerDevice {
  std::atomic<unsigned long long> bits{0};
  bool done(int dev) const { return dev < 64 && ((bits.load(std::memory_order_acquire) >> dev) & 1ull); }
  void mark(int dev) {
    if (dev < 64) bits.fetch_or(1ull << dev, std::memory_order_acq_rel);
  }
};

static int current_device() {
  int d = 0;
  return cudaGetDevice(&d) == cudaSuccess ? d : 0;
}

// Mapped pinned host words, one per device ordinal, that the kernels' failure reports also
// write (g_status_mapped); allocated once per process, registered per device on first use.
constexpr int kStatusWords = 64;
static std::mutex g_status_mu;
static int* g_status_host = nullptr;

static int register_status_word(int dev) {
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (!g_status_host) {
    void* p = nullptr;
    if (cudaHostAlloc(&p, kStatusWords * sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess)
      return QRB200_ERR_CUDA;
    std::memset(p, 0, kStatusWords * sizeof(int));
    g_status_host = static_cast<int*>(p);
  }
  void* dptr = nullptr;
  if (cudaHostGetDevicePointer(&dptr, g_status_host + dev, 0) != cudaSuccess) return QRB200_ERR_CUDA;
  int* word = static_cast<int*>(dptr);
  if (cudaMemcpyToSymbol(g_status_mapped, &word, sizeof(word)) != cudaSuccess) return QRB200_ERR_CUDA;
  return QRB200_OK;
}

// The current device must be an sm_100 GPU. The first call per device also registers its
// mapped failure word (a synchronous symbol copy: make the first call on a device before any
// stream capture on it).
static int check_device() {
  static PerDevice ok, bad;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return QRB200_ERR_CUDA;
  if (ok.done(dev)) return QRB200_OK;
  if (bad.done(dev)) return QRB200_ERR_DEVICE;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return QRB200_ERR_CUDA;
  if (major != 10) {
    bad.mark(dev);
    return QRB200_ERR_DEVICE;
  }
  if (dev < kStatusWords) {
    const int st = register_status_word(dev);
    if (st != QRB200_OK) return st;
  }
  ok.mark(dev);
  return QRB200_OK;
}

// Launch with an optional cluster shape and, for kernels that begin with griddep_launch_wait(),
// programmatic dependent launch (the kernel may be scheduled while its predecessor in the
// stream finishes; it waits for it before touching global memory).
template <typename... KArgs, typename... Args>
static cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            unsigned cluster, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned na = 0;
  if (cluster > 0) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Whole-matrix factorisation by one CTA per matrix (n <= kSmallN), one launch: two factor
// warps taking 4-column blocks in turn, fed by update warps (small_pp_kernel). Update warps
// pause kFwPollNs between polls, which leaves issue slots to the factor warps.
constexpr int kFwPollNs = 50;

template <int NMAX, int NWL>
static cudaError_t launch_small_fw(const float* A, float* H, float* tau, long long batch, int n, long long abs,
                                   cudaStream_t s) {
  static PerDevice configured;
  const int dev = current_device();
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(small_pp_kernel<NMAX, NWL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)small_pp_smem<NMAX>());
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  small_pp_kernel<NMAX, NWL><<<(unsigned)batch, 32 * NWL, small_pp_smem<NMAX>(), s>>>(A, abs, H, tau, n, kFwPollNs);
  return cudaGetLastError();
}

static cudaError_t run_small(const float* A, float* H, float* tau, long long batch, int n,
                             long long abs, cudaStream_t s) {
  LaunchScope ls(K_SMALL, batch * 4.0 * n * (double)n * n / 3.0, batch * 8.0 * n * (double)n);
  if (n <= 32) return launch_small_fw<32, 8>(A, H, tau, batch, n, abs, s);
  if (n <= 64) return launch_small_fw<64, 16>(A, H, tau, batch, n, abs, s);
  return launch_small_fw<128, 16>(A, H, tau, batch, n, abs, s);
}

// "Owner computes" panel, one CTA per matrix, four columns per warp.
template <int RPL>
static cudaError_t launch_owner(const PanelParams& pp, long long batch, cudaStream_t s) {
  constexpr int CPW = 4;
  static PerDevice configured;
  const int dev = current_device();
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(panel_owner_kernel<RPL, CPW, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)panel_stage_bytes<RPL>());
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  panel_owner_kernel<RPL, CPW, true><<<dim3(1, (unsigned)batch), 32 * (32 / CPW), panel_stage_bytes<RPL>(), s>>>(pp);
  return cudaGetLastError();
}

template <int RPL>
static cudaError_t launch_fw(const PanelParams& pp, long long batch, cudaStream_t s) {
  static PerDevice configured;
  const int dev = current_device();
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(panel_fw_kernel<RPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)panel_fw_smem<RPL>());
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  return launch_k(panel_fw_kernel<RPL>, dim3(1, (unsigned)batch), dim3(32 * kPanelFwWarps), panel_fw_smem<RPL>(), s, 0,
                  true, pp);
}

template <int RPL>
static cudaError_t launch_cl(const PanelParams& pp, int cluster, long long batch, cudaStream_t s) {
  static PerDevice configured;
  const int dev = current_device();
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(panel_cl_kernel<RPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)panel_cl_smem<RPL>());
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(panel_cl_kernel<RPL>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  return launch_k(panel_cl_kernel<RPL>, dim3((unsigned)cluster, (unsigned)batch, 1), dim3(kClThreads, 1, 1),
                  panel_cl_smem<RPL>(), s, (unsigned)cluster, true, pp);
}

// Panel kernel by panel height m (the choice depends on the matrix order and m only, so
// results stay independent of the batch):
//   m >= 513: cluster of ceil(m / 256) CTAs (<= 16), 256 rows each (panel_cl_kernel);
//   m <= 512, n >= 1025: one CTA with a factor warp fed by update warps (panel_fw_kernel) --
//     the shorter chain, for the latency-bound launches of a few large matrices;
//   m <= 512, n <= 1024: the owner-computes panel (three CTAs per SM up to 384 rows), for the
//     throughput-bound launches of many small matrices.
constexpr int kClRows = 256;
constexpr int kClMinM = 513;
constexpr int kFwMinN = 1025;

static bool is_cluster_panel(int m) { return m >= kClMinM && m <= kClMaxCta * kClRows; }

static cudaError_t launch_panel_for(const PanelParams& pp, int m, long long batch, cudaStream_t s, long long t_bstride) {
  PanelParams q = pp;
  q.t_bstride = t_bstride;
  if (is_cluster_panel(m)) return launch_cl<8>(q, cdiv(m, kClRows), batch, s);
  if (pp.n >= kFwMinN) {
    if (m <= 128) return launch_fw<4>(q, batch, s);
    if (m <= 256) return launch_fw<8>(q, batch, s);
    return launch_fw<16>(q, batch, s);
  }
  // Owner panels hold exactly ceil(m / 32) rows per lane: no padding rows to carry.
  switch ((m + 31) / 32) {
    case 1: return launch_owner<1>(q, batch, s);
    case 2: return launch_owner<2>(q, batch, s);
    case 3: return launch_owner<3>(q, batch, s);
    case 4: return launch_owner<4>(q, batch, s);
    case 5: return launch_owner<5>(q, batch, s);
    case 6: return launch_owner<6>(q, batch, s);
    case 7: return launch_owner<7>(q, batch, s);
    case 8: return launch_owner<8>(q, batch, s);
    case 9: return launch_owner<9>(q, batch, s);
    case 10: return launch_owner<10>(q, batch, s);
    case 11: return launch_owner<11>(q, batch, s);
    case 12: return launch_owner<12>(q, batch, s);
    case 13: return launch_owner<13>(q, batch, s);
    case 14: return launch_owner<14>(q, batch, s);
    case 15: return launch_owner<15>(q, batch, s);
    default: return launch_owner<16>(q, batch, s);
  }
}

// Kernel kind of the panel launch for a panel of m rows (cluster panels counted apart).
static int panel_kind(int m) { return is_cluster_panel(m) ? K_PANEL_CL : K_PANEL; }

// Single-level schedule for rows that are not 16-byte aligned (n % 4 != 0 or an unaligned
// input, n <= 1024): 32-column panels and the FP32 update of wy_simt.cuh, one stream.
static cudaError_t run_blocked(const float* A, float* H, float* tau, long long batch, int n,
                               long long abs, const Workspace& ws, cudaStream_t s) {
  const int ncmax = n;
  for (int k = 0; k < n; k += kNB) {
    const int w = std::min(kNB, n - k);
    const int m = n - k;
    const int nc = n - k - w;
    const float* src = (k == 0) ? A : H;
    const long long sbs = (k == 0) ? abs : (long long)n * n;
    PanelParams pp{src, sbs, H, tau, nc > 0 ? ws.T : nullptr, n, k, w};
    cudaError_t e;
    {
      LaunchScope ls(panel_kind(m), batch * panel_flops(m, w), batch * 8.0 * m * w);
      e = launch_panel_for(pp, m, batch, s, kNB * kNB);
    }
    if (e != cudaSuccess) return e;
    if (nc <= 0) continue;
    WyParams wp{};
    wp.src = src;
    wp.src_bstride = sbs;
    wp.H = H;
    wp.T = ws.T;
    wp.t_bstride = kNB * kNB;
    wp.Wp = ws.Wp;
    wp.W2 = ws.W2;
    wp.n = n;
    wp.k = k;
    wp.w = w;
    wp.cend = n;
    wp.nsplit = choose_nsplit(batch, n, k, w);
    wp.rows_per_split = kRowsPerSplit;
    wp.ncmax = ncmax;
    const double bm = (double)batch * m;
    {
      LaunchScope ls(K_VTC, 2.0 * bm * w * nc, 4.0 * bm * (w + nc) + 4.0 * batch * wp.nsplit * w * (double)nc);
      wy_vtc_kernel<kNB><<<dim3(cdiv(nc, 64), wp.nsplit, (unsigned)batch), 256, 0, s>>>(wp);
    }
    {
      LaunchScope ls(K_TW, (double)batch * w * w * nc, 4.0 * batch * (wp.nsplit + 1.0) * w * nc);
      wy_tw_kernel<kNB><<<dim3(cdiv(nc, 128), (unsigned)batch), 128, 0, s>>>(wp);
    }
    {
      LaunchScope ls(K_UPD, 2.0 * bm * w * nc, 8.0 * bm * nc + 4.0 * bm * w + 4.0 * batch * w * (double)nc);
      wy_upd_kernel<kNB><<<dim3(cdiv(nc, 64), cdiv(m, 64), (unsigned)batch), 256, 0, s>>>(wp);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Shared-memory opt-in of the 128-wide tensor-core kernels (three-slot operand rings: two CTAs
// per SM for the GEMM tiles, four for the Gram) and of tbuild, once per device.
static cudaError_t tc128_configure() {
  static PerDevice done;
  const int dev = current_device();
  if (done.done(dev)) return cudaSuccess;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(tc_vtcw_pipe_kernel<kOB, false, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vtcw_pipe_smem<kOB, false, 3>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_vtcw_pipe_kernel<kOB, true, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vtcw_pipe_smem<kOB, true, 3>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tbuild_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTbuildSmem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_gemm128_pipe_kernel<MODE_UPD, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pipe128_smem<3>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_gemm128_pipe_kernel<MODE_Y, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pipe128_smem<3>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_gemm128_pipe_kernel<MODE_WT, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pipe128_smem<3>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_upd_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tma_upd_smem())) != cudaSuccess) return e;
  done.mark(dev);
  return cudaSuccess;
}

// Narrow updates of the two-level schedule take the one-launch clustered kernel (wy_u1) for
// matrices of order >= kNarrowU1MinN (it helps at small batch and tall panels, and loses to the
// streaming kernels at n = 512 and batch 640); updates of up to kU1MaxCols columns qualify.
constexpr int kNarrowU1MinN = 1024;
constexpr int kU1MaxCols = 128;

// Streaming multiprocessors of the current device (cached per device).
static int num_sms() {
  static int cache[kMaxDevicesSm] = {0};
  const int dev = current_device();
  if (dev < kMaxDevicesSm && cache[dev] > 0) return cache[dev];
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
  if (dev < kMaxDevicesSm) cache[dev] = v;
  return v;
}

// CTAs of the persistent update kernels (wy_upd3 64 x 64, 128 x 32) resident per SM, from the
// occupancy query when the kernels are configured on a device: their grids are that many CTAs per
// SM, so that no CTA of a persistent grid waits for another to finish its whole share of tiles.
static int g_upd3_resident[kMaxDevicesSm][2];

// Compact-WY update of columns [k + w + coff, cend) by the 32-column panel at k (the narrow
// update inside an outer block, or either half of a single-level look-ahead update). T factors
// sit t_bstride elements apart. Aligned rows: a short update (<= 128 columns, allow_u1) is one
// clustered launch (wy_u1: V^T C partials per 256-row CTA summed over DSMEM, T^T, update);
// otherwise V^T C (tcgen05 beyond 64 columns, else FP32), T^T sum, FP32 update with one tile
// per CTA for wide updates (a persistent grid that filled every SM before the next
// high-priority panel launched held that panel back). Unaligned rows: wy_simt.cuh.
static cudaError_t launch_wy(const float* src, long long sbs, float* H, const float* T, long long t_bstride,
                             const Workspace& ws, long long batch, int n, int k, int w, int coff, int cend,
                             cudaStream_t s, bool allow_u1 = false) {
  const int m = n - k, nc = cend - k - w, ncl = nc - coff;
  if (ncl <= 0) return cudaSuccess;
  WyParams wp{};
  wp.src = src;
  wp.src_bstride = sbs;
  wp.H = H;
  wp.T = T;
  wp.t_bstride = t_bstride;
  wp.Wp = ws.Wp;
  wp.W2 = ws.W2;
  wp.n = n;
  wp.k = k;
  wp.w = w;
  wp.cend = cend;
  wp.nsplit = choose_nsplit(batch, n, k, w);
  wp.rows_per_split = kRowsPerSplit;
  wp.ncmax = n;
  wp.coff = coff;
  const double bm = (double)batch * m;
  cudaError_t ep = cudaSuccess;  // first launch error of the three kernels
  auto note = [&ep](cudaError_t e) {
    if (ep == cudaSuccess) ep = e;
  };
  const bool vec = w == kNB && (n % 4) == 0 && (sbs % 4) == 0 &&
                   ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(H)) & 15u) == 0;
  if (vec) {
    static PerDevice configured;
    const int dev = current_device();
    if (!configured.done(dev)) {
      cudaError_t e = cudaFuncSetAttribute(wy_vtc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kVtc2Smem);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(wy_upd3_kernel<kU3Rows, kU3Cols>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)upd3_smem<kU3Rows, kU3Cols>());
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(wy_upd3_kernel<128, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)upd3_smem<128, 32>());
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(wy_vtcn_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vtcn_smem<32>());
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(wy_vtcn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vtcn_smem<64>());
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(wy_upd4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kUpd4Smem);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tc_vtcw_pipe_kernel<32, false, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)vtcw_pipe_smem<32, false, 3>());
      int r64 = 0, r128 = 0;
      if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r64, wy_upd3_kernel<kU3Rows, kU3Cols>, 256,
                                                          upd3_smem<kU3Rows, kU3Cols>());
      if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r128, wy_upd3_kernel<128, 32>, 256, upd3_smem<128, 32>());
      if (e != cudaSuccess) return e;
      if (dev < kMaxDevicesSm) {
        g_upd3_resident[dev][0] = std::max(1, r64);
        g_upd3_resident[dev][1] = std::max(1, r128);
      }
      configured.mark(dev);
    }
  }
  if (allow_u1 && vec && ncl <= kU1MaxCols && m <= kClMaxCta * kU1Rows) {
    static PerDevice configured_u1;
    const int dev = current_device();
    if (!configured_u1.done(dev)) {
      cudaError_t e = cudaFuncSetAttribute(wy_u1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kU1Smem);
      if (e == cudaSuccess) e = cudaFuncSetAttribute(wy_u1_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
      configured_u1.mark(dev);
    }
    const int cp = cdiv(m, kU1Rows);
    LaunchScope ls(K_U1, 4.0 * bm * w * ncl + (double)batch * w * w * ncl, 12.0 * bm * ncl + 4.0 * bm * w);
    return launch_k(wy_u1_kernel, dim3((unsigned)cp, (unsigned)cdiv(ncl, 32), (unsigned)batch), dim3(kU1Threads), kU1Smem, s,
                    (unsigned)cp, true, wp);
  }
  // V^T C on tcgen05 (partials stored transposed) above 64 columns: the narrow updates of 96
  // columns and the single-level tails as well (C2 4.32 -> 4.25 ms on B200).
  const bool vtc_tc = vec && ncl > 64;
  {
    LaunchScope ls(K_VTC, 2.0 * bm * w * ncl, 4.0 * bm * (w + ncl) + 4.0 * batch * wp.nsplit * w * (double)ncl);
    if (vtc_tc)
      tc_vtcw_pipe_kernel<32, false, 3><<<dim3(cdiv(ncl, kTcCols), wp.nsplit, (unsigned)batch), 128,
                                          vtcw_pipe_smem<32, false, 3>(), s>>>(wp);
    else if (vec && ncl <= 32)
      note(launch_k(wy_vtcn_kernel<32>, dim3(cdiv(ncl, 32), wp.nsplit, (unsigned)batch), dim3(256), vtcn_smem<32>(), s, 0, true, wp));
    else if (vec && ncl <= 64)
      note(launch_k(wy_vtcn_kernel<64>, dim3(cdiv(ncl, 64), wp.nsplit, (unsigned)batch), dim3(256), vtcn_smem<64>(), s, 0, true, wp));
    else if (vec)
      note(launch_k(wy_vtc2_kernel, dim3(cdiv(ncl, kV2Cols), wp.nsplit, (unsigned)batch), dim3(256), kVtc2Smem, s, 0, true, wp));
    else
      wy_vtc_kernel<kNB><<<dim3(cdiv(ncl, 64), wp.nsplit, (unsigned)batch), 256, 0, s>>>(wp);
  }
  {
    LaunchScope ls(K_TW, (double)batch * w * w * ncl, 4.0 * batch * (wp.nsplit + 1.0) * w * ncl);
    if (vtc_tc)
      note(launch_k(wy_tw2t_kernel, dim3(cdiv(ncl, 32), (unsigned)batch), dim3(256), 0, s, 0, true, wp));
    else if (vec)
      note(launch_k(wy_tw2_kernel, dim3(cdiv(ncl, 32), (unsigned)batch), dim3(256), 0, s, 0, true, wp));
    else
      wy_tw_kernel<kNB><<<dim3(cdiv(ncl, 128), (unsigned)batch), 128, 0, s>>>(wp);
  }
  {
    LaunchScope ls(K_UPD, 2.0 * bm * w * ncl, 8.0 * bm * ncl + 4.0 * bm * w + 4.0 * batch * w * (double)ncl);
    if (vec && ncl > kU3Cols) {
      const int tc = cdiv(ncl, kU4Cols), tr = cdiv(m, kU4Rows);
      const long long nt = (long long)tc * tr * batch;
      note(launch_k(wy_upd4_kernel, dim3((unsigned)nt), dim3(256), kUpd4Smem, s, 0, true, wp, tc, tr));
    } else if (vec && ncl <= 32) {
      const int tc = cdiv(ncl, 32), tr = cdiv(m, 128);
      const long long nt = (long long)tc * tr * batch;
      const int dev = current_device();
      const long long res = dev < kMaxDevicesSm && g_upd3_resident[dev][1] > 0 ? g_upd3_resident[dev][1] : 2;
      const int grid = (int)std::min<long long>(nt, res * num_sms());
      note(launch_k(wy_upd3_kernel<128, 32>, dim3(grid), dim3(256), upd3_smem<128, 32>(), s, 0, true, wp, tc, tr, (int)nt));
    } else if (vec) {
      const int tc = cdiv(ncl, kU3Cols), tr = cdiv(m, kU3Rows);
      const long long nt = (long long)tc * tr * batch;
      const int dev = current_device();
      const long long res = dev < kMaxDevicesSm && g_upd3_resident[dev][0] > 0 ? g_upd3_resident[dev][0] : 3;
      const int grid = (int)std::min<long long>(nt, res * num_sms());
      note(launch_k(wy_upd3_kernel<kU3Rows, kU3Cols>, dim3(grid), dim3(256), upd3_smem<kU3Rows, kU3Cols>(), s, 0, true, wp, tc, tr, (int)nt));
    } else {
      wy_upd_kernel<kNB><<<dim3(cdiv(ncl, 64), cdiv(m, 64), (unsigned)batch), 256, 0, s>>>(wp);
    }
  }
  return ep != cudaSuccess ? ep : cudaGetLastError();
}

// Look-ahead streams: the critical chain (panels, narrow updates, T, Y and the update of the
// next outer block's or panel's columns) runs on a high-priority stream p, the rest of each
// update on a low-priority one u, and (single-level schedule) the strip of the panel after next
// on a second high-priority stream m; all forked from and joined back into the caller's stream.
struct LookaheadStreams {
  cudaStream_t p = nullptr, u = nullptr, m = nullptr;  // critical, bulk update, strip update
  cudaEvent_t fork = nullptr, y = nullptr, u2 = nullptr, u2a = nullptr, pj = nullptr, uj = nullptr, mj = nullptr;
};
constexpr int kMaxDevices = 64;

// One set of look-ahead streams per caller stream (up to kLaSlots per device), so calls enqueued
// on different streams -- the host API's batch pieces, or several host threads -- factor
// concurrently instead of queueing behind one shared pair. Calls on one caller stream reuse its
// set and stay ordered; its mutex keeps one enqueue at a time on a set. Callers beyond the
// first kLaSlots streams of a device run without look-ahead (la_slot).
constexpr int kLaSlots = 8;
struct LaSlot {
  std::mutex mu;
  bool used = false;
  cudaStream_t owner = nullptr;
  LookaheadStreams L;
};
static std::mutex g_la_table_mu[kMaxDevices];
static LaSlot g_la_slots[kMaxDevices][kLaSlots];

// The caller stream's slot, or nullptr once kLaSlots other caller streams hold every slot of
// the device (slots are never released: a stream handle may be destroyed and reused). Such a
// call runs its schedule serially on the caller's stream: no look-ahead, but no stream shared
// with another caller either (which would order, or -- under stream capture -- invalidate,
// that caller's work).
static LaSlot* la_slot(int dev, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_la_table_mu[dev]);
  LaSlot* free_slot = nullptr;
  for (LaSlot& sl : g_la_slots[dev]) {
    if (sl.used && sl.owner == s) return &sl;
    if (!sl.used && free_slot == nullptr) free_slot = &sl;
  }
  if (free_slot != nullptr) {
    free_slot->used = true;
    free_slot->owner = s;
  }
  return free_slot;
}

static cudaError_t lookahead_streams(LaSlot& slot, LookaheadStreams** out) {
  LookaheadStreams& L = slot.L;
  if (!L.p) {
    int least = 0, greatest = 0;
    cudaError_t e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
    if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&L.u, cudaStreamNonBlocking, least);
    if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&L.m, cudaStreamNonBlocking, greatest);
    for (cudaEvent_t* ev : {&L.fork, &L.y, &L.u2, &L.u2a, &L.pj, &L.uj, &L.mj})
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&L.p, cudaStreamNonBlocking, greatest);
    if (e != cudaSuccess) {
      L.p = nullptr;  // retried on the next call
      return e;
    }
  }
  *out = &L;
  return cudaSuccess;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Tensor map over a batch of row-major float matrices (cols x rows x batch; row and matrix strides
// in bytes, multiples of 16), box 4 columns x 128 rows: what tc_upd_tma_kernel loads per piece.
// Rows and columns past the extents read as zero.
static bool encode_rows_map(CUtensorMap* map, const float* base, uint64_t cols, uint64_t rows, uint64_t batch,
                            uint64_t row_bytes, uint64_t mat_bytes) {
  const PFN_cuTensorMapEncodeTiled_v12000 fn = tensor_map_encoder();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {cols, rows, batch};
  const cuuint64_t strides[2] = {row_bytes, mat_bytes};
  const cuuint32_t box[3] = {4, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 128-wide update of trailing columns [coff, cend - k0 - ow) (relative to k0 + ow) by the
// outer block at k0, whose T factor is given transposed (Tt, batch x 128 x 128):
//   W^T = C^T V per row split (tc_vtc128), W'^T = W^T T, i.e. W' = T^T V^T C (tc_tw128, into Wt,
//   batch x n x 128, row = trailing column), then C -= V W' (tc_upd128).
// Applying T to the (128 x columns) W' of each launch instead of forming Y = V T^T (rows x 128)
// once per block keeps that product off the critical stream: the near update (the next block's
// 128 columns) multiplies only its own columns. coff is a multiple of 128, so every column sees
// the same tiles, and the same arithmetic, however the range is cut.
static cudaError_t launch_wide(const float* src, long long sbs, float* H, const float* Tt, float* Wt,
                               const Workspace& ws, long long batch, int n, int k0, int ow, int coff, int cend,
                               cudaStream_t s) {
  const int m = n - k0, nc = cend - k0 - ow - coff;
  if (nc <= 0) return cudaSuccess;
  const int nsw = cdiv(m, kRowsPerSplitWide);
  if (nsw > 2) return cudaErrorInvalidValue;  // the W^T T tile sums at most two W^T partials
  const double bm = (double)batch * m;
  WyParams wp{};
  wp.src = src;
  wp.src_bstride = sbs;
  wp.H = H;
  wp.Wp = ws.Wf;
  wp.n = n;
  wp.k = k0;
  wp.w = ow;
  wp.cend = cend;
  wp.nsplit = nsw;
  wp.rows_per_split = kRowsPerSplitWide;
  wp.ncmax = n;
  wp.coff = coff;
  Gemm128Params gp{};
  gp.H = H;
  gp.src = src;
  gp.src_bstride = sbs;
  gp.Hout = H;
  gp.T = Tt;
  gp.Y = Wt;
  gp.y_bstride = (long long)n * kOB;
  gp.Wp = ws.Wf;
  gp.nsplit = nsw;
  gp.ncmax = n;
  gp.n = n;
  gp.k = k0;
  gp.w = ow;
  gp.cend = cend;
  gp.coff = coff;
  {
    LaunchScope ls(K_VTC128, 2.0 * bm * ow * nc, 4.0 * bm * (ow + nc) + 4.0 * batch * nsw * ow * (double)nc);
    const dim3 grid(cdiv(nc, kTcCols), nsw, (unsigned)batch);
    tc_vtcw_pipe_kernel<kOB, false, 3><<<grid, 128, vtcw_pipe_smem<kOB, false, 3>(), s>>>(wp);
  }
  {
    LaunchScope ls(K_TW128, 2.0 * batch * (double)nc * ow * ow,
                   4.0 * batch * ((nsw + 1.0) * nc * ow + (double)ow * ow));
    const dim3 grid(1, cdiv(nc, 128), (unsigned)batch);
    tc_gemm128_pipe_kernel<MODE_WT, 3><<<grid, 128, pipe128_smem<3>(), s>>>(gp);
  }
  {
    LaunchScope ls(K_UPD128, 2.0 * bm * ow * nc, 8.0 * bm * nc + 4.0 * bm * ow + 4.0 * batch * ow * (double)nc);
    const dim3 grid(cdiv(nc, 128), cdiv(m, 128), (unsigned)batch);
    CUtensorMap tmV, tmW;
    if (!encode_rows_map(&tmV, H, n, n, batch, 4ull * n, 4ull * n * n) ||
        !encode_rows_map(&tmW, Wt, kOB, n, batch, 4ull * kOB, 4ull * n * kOB))
      return cudaErrorInvalidValue;
    tc_upd_tma_kernel<<<grid, 128, tma_upd_smem(), s>>>(gp, tmV, tmW);
  }
  return cudaGetLastError();
}

// Two-level blocked QR: outer blocks of 128 columns, each factored as four 32-column panels
// with narrow updates inside the block, then one 128-wide tensor-core update of the trailing
// matrix, C <- C - Y (V^T C) with Y = V T^T (T assembled from the block Gram matrix).
// With look-ahead (L != nullptr) the wide update is cut in two: the next outer block's 128
// columns (U1, on the critical stream sp) and everything right of them (U2, on su), so U2 of
// block k0 runs while block k0 + 128 is factored. U1 of block k0 + 128 waits for U2 of block
// k0 (same columns); Y alternates between two buffers so U2 can still read block k0's.
static cudaError_t two_level_body(const float* A, float* H, float* tau, long long batch, int n, long long abs,
                                  const Workspace& ws, cudaStream_t sp, cudaStream_t su, LookaheadStreams* L) {
  cudaError_t e;
  bool u2_pending = false;
  for (int k0 = 0; k0 < n; k0 += kOB) {
    const int ow = std::min(kOB, n - k0);
    for (int kb = k0; kb < k0 + ow; kb += kNB) {
      const int w = std::min(kNB, n - kb), m = n - kb;
      const float* src = (kb == 0) ? A : H;
      const long long sbs = (kb == 0) ? abs : (long long)n * n;
      float* Tslot = ws.T + (size_t)((kb - k0) / kNB) * kNB * kNB;
      // panel factors land in slot b of the batch x 4 x 32 x 32 array
      PanelParams pp{src, sbs, H, tau, Tslot, n, kb, w};
      {
        LaunchScope ls(panel_kind(m), batch * panel_flops(m, w), batch * 8.0 * m * w);
        e = launch_panel_for(pp, m, batch, sp, 4 * kNB * kNB);
      }
      if (e != cudaSuccess) return e;
      if (kb + w < k0 + ow) {
        e = launch_wy(src, sbs, H, Tslot, 4 * kNB * kNB, ws, batch, n, kb, w, 0, k0 + ow, sp, n >= kNarrowU1MinN);
        if (e != cudaSuccess) return e;
      }
    }
    if (k0 + ow >= n) break;
    const int m = n - k0;
    const float* src = (k0 == 0) ? A : H;
    const long long sbs = (k0 == 0) ? abs : (long long)n * n;
    const int nsw = cdiv(m, kRowsPerSplitWide);
    const double bm = (double)batch * m;
    // Buffers alternate by block parity: the far update of this block may still read them while
    // the next block's are written.
    float* Wt = ((k0 / kOB) & 1) ? ws.Y2 : ws.Y;
    float* Tt = ((k0 / kOB) & 1) ? ws.Tob2 : ws.Tob;
    // Gram matrix of the outer block's reflectors.
    WyParams g{};
    g.src = H;
    g.src_bstride = (long long)n * n;
    g.H = H;
    g.Wp = ws.Gp;
    g.n = n;
    g.k = k0;
    g.w = ow;
    g.cend = n;
    g.nsplit = nsw;
    g.rows_per_split = kRowsPerSplitWide;
    g.ncmax = kOB;
    {
      LaunchScope ls(K_GRAM, 2.0 * bm * ow * ow, 4.0 * bm * ow);
      const dim3 grid(1, nsw, (unsigned)batch);
      tc_vtcw_pipe_kernel<kOB, true, 3><<<grid, 128, vtcw_pipe_smem<kOB, true, 3>(), sp>>>(g);
    }
    {
      TbuildParams tp{ws.Gp, nsw, ws.T, Tt, ow, 1};  // T stored transposed
      LaunchScope ls(K_TBUILD, batch * 2.0 * ow * ow * ow / 3.0, 4.0 * batch * (nsw + 1.0) * ow * ow);
      tbuild_kernel<<<(unsigned)batch, 256, kTbuildSmem, sp>>>(tp);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const int split_at = k0 + 2 * kOB;  // U1 = columns [k0 + ow, split_at), U2 = [split_at, n)
    if (L == nullptr || split_at >= n) {
      if (L != nullptr && u2_pending && (e = cudaStreamWaitEvent(sp, L->u2, 0)) != cudaSuccess) return e;
      u2_pending = false;
      e = launch_wide(src, sbs, H, Tt, Wt, ws, batch, n, k0, ow, 0, n, sp);
      if (e != cudaSuccess) return e;
      continue;
    }
    if ((e = cudaEventRecord(L->y, sp)) != cudaSuccess) return e;
    if (u2_pending && (e = cudaStreamWaitEvent(sp, L->u2, 0)) != cudaSuccess) return e;  // U2 of k0 - 128
    if ((e = cudaStreamWaitEvent(su, L->y, 0)) != cudaSuccess) return e;
    if ((e = launch_wide(src, sbs, H, Tt, Wt, ws, batch, n, k0, ow, kOB, n, su)) != cudaSuccess) return e;
    if ((e = cudaEventRecord(L->u2, su)) != cudaSuccess) return e;
    u2_pending = true;
    if ((e = launch_wide(src, sbs, H, Tt, Wt, ws, batch, n, k0, ow, 0, split_at, sp)) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

static cudaError_t run_two_level(const float* A, float* H, float* tau, long long batch, int n, long long abs,
                                 const Workspace& ws, cudaStream_t s) {
  cudaError_t e = tc128_configure();
  if (e != cudaSuccess) return e;
  const int dev = current_device();
  // Serial schedule when profiling (per-launch events on one stream), when switched off, or
  // when no outer block has columns beyond the next one (n <= 256).
  if (t_prof || n <= 2 * kOB || dev >= kMaxDevices)
    return two_level_body(A, H, tau, batch, n, abs, ws, s, s, nullptr);
  LaSlot* slot = la_slot(dev, s);
  if (slot == nullptr) return two_level_body(A, H, tau, batch, n, abs, ws, s, s, nullptr);
  std::lock_guard<std::mutex> lk(slot->mu);
  LookaheadStreams* L = nullptr;
  if ((e = lookahead_streams(*slot, &L)) != cudaSuccess) return e;
  if ((e = cudaEventRecord(L->fork, s)) != cudaSuccess) return e;
  if ((e = cudaStreamWaitEvent(L->p, L->fork, 0)) != cudaSuccess) return e;
  if ((e = cudaStreamWaitEvent(L->u, L->fork, 0)) != cudaSuccess) return e;
  const cudaError_t body = two_level_body(A, H, tau, batch, n, abs, ws, L->p, L->u, L);
  // Join both streams back into the caller's stream, also after a failed launch.
  e = cudaEventRecord(L->pj, L->p);
  if (e == cudaSuccess) e = cudaEventRecord(L->uj, L->u);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, L->pj, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, L->uj, 0);
  return body != cudaSuccess ? body : e;
}

// Single-level blocked QR with look-ahead of depth two. After panel k (32 columns at kb) its
// update is cut in three column ranges:
//   U1(k)  = [kb + 32, kb + 64), the next panel's columns, on the critical stream sp;
//   U2a(k) = [kb + 64, kb + 96), the panel after next, one clustered launch on stream sm;
//   U2b(k) = [kb + 96, n), everything else, on the low-priority stream su.
// Dependencies: U1(k) waits for U2a(k - 1) (same columns, previous panel); U2a(k) waits for
// panel k and U2b(k - 1) (its columns carry panel k - 1's update from there); U2b(k) follows
// U2b(k - 1) on su. So the bulk update U2b of panel k - 1 has until U1(k + 1) -- two panel steps
// -- to finish, instead of one. Panel T factors rotate over three workspace slots (U2b(k - 1) may
// still read slot k - 1 while panel k + 1 writes its own); the partial-product buffers of the
// three-kernel update are indexed by column relative to the panel, and U1, U2a and U2b of one
// panel as well as U2b(k - 1) use disjoint index ranges. L == nullptr runs the same three
// launches on sp, so both schedules give bitwise the same result.
static cudaError_t single_level_body(const float* A, float* H, float* tau, long long batch, int n, long long abs,
                                     const Workspace& ws, cudaStream_t sp, cudaStream_t su, LookaheadStreams* L) {
  cudaError_t e;
  bool pending = false;  // U2a / U2b of the previous panel have been enqueued on the side streams
  constexpr long long kTStride = 4 * kNB * kNB;
  for (int kb = 0; kb < n; kb += kNB) {
    const int w = std::min(kNB, n - kb), m = n - kb, nc = n - kb - w;
    const float* src = (kb == 0) ? A : H;
    const long long sbs = (kb == 0) ? abs : (long long)n * n;
    float* Tslot = ws.T + (size_t)((kb / kNB) % 3) * kNB * kNB;
    PanelParams pp{src, sbs, H, tau, nc > 0 ? Tslot : nullptr, n, kb, w};
    {
      LaunchScope ls(panel_kind(m), batch * panel_flops(m, w), batch * 8.0 * m * w);
      e = launch_panel_for(pp, m, batch, sp, kTStride);
    }
    if (e != cudaSuccess) return e;
    if (nc <= 0) continue;
    const int c1 = std::min(n, kb + w + kNB), c2 = std::min(n, kb + w + 2 * kNB);
    if (L == nullptr) {
      if ((e = launch_wy(src, sbs, H, Tslot, kTStride, ws, batch, n, kb, w, 0, c1, sp, true)) != cudaSuccess) return e;
      if ((e = launch_wy(src, sbs, H, Tslot, kTStride, ws, batch, n, kb, w, kNB, c2, sp, true)) != cudaSuccess) return e;
      if ((e = launch_wy(src, sbs, H, Tslot, kTStride, ws, batch, n, kb, w, 2 * kNB, n, sp, true)) != cudaSuccess)
        return e;
      continue;
    }
    if ((e = cudaEventRecord(L->y, sp)) != cudaSuccess) return e;
    // U1(k) after U2a(k - 1) (the event still holds that record here).
    if (pending && (e = cudaStreamWaitEvent(sp, L->u2a, 0)) != cudaSuccess) return e;
    if ((e = launch_wy(src, sbs, H, Tslot, kTStride, ws, batch, n, kb, w, 0, c1, sp, true)) != cudaSuccess) return e;
    // U2a(k) after panel k and U2b(k - 1).
    if ((e = cudaStreamWaitEvent(L->m, L->y, 0)) != cudaSuccess) return e;
    if (pending && (e = cudaStreamWaitEvent(L->m, L->u2, 0)) != cudaSuccess) return e;
    if ((e = launch_wy(src, sbs, H, Tslot, kTStride, ws, batch, n, kb, w, kNB, c2, L->m, true)) != cudaSuccess)
      return e;
    if ((e = cudaEventRecord(L->u2a, L->m)) != cudaSuccess) return e;
    // U2b(k) after panel k.
    if ((e = cudaStreamWaitEvent(su, L->y, 0)) != cudaSuccess) return e;
    if ((e = launch_wy(src, sbs, H, Tslot, kTStride, ws, batch, n, kb, w, 2 * kNB, n, su, true)) != cudaSuccess)
      return e;
    if ((e = cudaEventRecord(L->u2, su)) != cudaSuccess) return e;
    pending = true;
  }
  return cudaSuccess;
}

// Shared fork/join around a look-ahead body: the body runs on the caller stream's two
// look-ahead streams, both joined back into the caller's stream (also after a failed launch).
template <class Body>
static cudaError_t with_lookahead(int dev, cudaStream_t s, Body body) {
  LaSlot* slot = la_slot(dev, s);
  if (slot == nullptr) return body(nullptr);
  std::lock_guard<std::mutex> lk(slot->mu);
  LookaheadStreams* L = nullptr;
  cudaError_t e;
  if ((e = lookahead_streams(*slot, &L)) != cudaSuccess) return e;
  if ((e = cudaEventRecord(L->fork, s)) != cudaSuccess) return e;
  if ((e = cudaStreamWaitEvent(L->p, L->fork, 0)) != cudaSuccess) return e;
  if ((e = cudaStreamWaitEvent(L->u, L->fork, 0)) != cudaSuccess) return e;
  if ((e = cudaStreamWaitEvent(L->m, L->fork, 0)) != cudaSuccess) return e;
  const cudaError_t b = body(L);
  e = cudaEventRecord(L->pj, L->p);
  if (e == cudaSuccess) e = cudaEventRecord(L->uj, L->u);
  if (e == cudaSuccess) e = cudaEventRecord(L->mj, L->m);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, L->pj, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, L->uj, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, L->mj, 0);
  return b != cudaSuccess ? b : e;
}

static cudaError_t run_single_la(const float* A, float* H, float* tau, long long batch, int n, long long abs,
                                 const Workspace& ws, cudaStream_t s) {
  const int dev = current_device();
  if (t_prof || n <= 2 * kNB || dev >= kMaxDevices)
    return single_level_body(A, H, tau, batch, n, abs, ws, s, s, nullptr);
  return with_lookahead(dev, s, [&](LookaheadStreams* L) {
    if (L == nullptr) return single_level_body(A, H, tau, batch, n, abs, ws, s, s, nullptr);
    return single_level_body(A, H, tau, batch, n, abs, ws, L->p, L->u, L);
  });
}

// ---------------------------------------------------------------------------------------
// Applying Q / Q^T (sormqr) and forming Q (sorgqr) from (H, tau) on the 128-wide kernels.
constexpr int kApplyRowsPerSplit = 2048;  // row split of the products: <= 2 splits for n <= 4096

struct ApplyWorkspace {
  float *Gp, *Tp, *Tob, *Y, *Wf;
  size_t bytes;
};

static ApplyWorkspace apply_layout(long long batch, int n, int nrhs, void* base) {
  ApplyWorkspace ws{};
  auto carve = [&](size_t bytes) {
    const size_t off = ws.bytes;
    ws.bytes += align_up(bytes, 256);
    return reinterpret_cast<float*>(static_cast<char*>(base) + off);
  };
  const size_t f = sizeof(float);
  const int nsw = cdiv(n, kApplyRowsPerSplit);
  ws.Gp = carve((size_t)batch * nsw * kOB * kOB * f);
  ws.Tp = carve((size_t)batch * 4 * kNB * kNB * f);
  ws.Tob = carve((size_t)batch * kOB * kOB * f);
  ws.Y = carve((size_t)batch * n * kOB * f);
  ws.Wf = carve((size_t)batch * nsw * (size_t)nrhs * kOB * f);
  return ws;
}

// C[k0:, ccol0 : ccol0 + ncols] of every matrix <- (I - V T^(T) V^T) C over the blocks of
// reflectors, first to last (Q^T) or last to first (Q). C has row stride ldc and batch stride
// c_bstride. For sorgqr (first_col_only_from_k0) the block at k0 touches only columns >= k0 of
// C: the columns left of it are still those of the identity, zero in rows >= k0.
static cudaError_t apply_q_blocks(const float* H, const float* tau, float* C, long long batch, int n, int ldc,
                                  long long c_bstride, int ncols, bool transpose_q, bool orgqr,
                                  const ApplyWorkspace& ws, cudaStream_t s) {
  cudaError_t e = tc128_configure();
  if (e != cudaSuccess) return e;
  const int nblocks = cdiv(n, kOB);
  for (int bi = 0; bi < nblocks; ++bi) {
    const int blk = transpose_q ? bi : nblocks - 1 - bi;
    const int k0 = blk * kOB, ow = std::min(kOB, n - k0), m = n - k0;
    const int nsw = cdiv(m, kApplyRowsPerSplit);
    const double bm = (double)batch * m;
    const int cfirst = orgqr ? k0 : 0;             // first column of C this block changes
    const int nc = orgqr ? ncols - k0 : ncols;     // columns it changes
    WyParams g{};
    g.src = H;
    g.src_bstride = (long long)n * n;
    g.H = const_cast<float*>(H);
    g.Wp = ws.Gp;
    g.n = n;
    g.k = k0;
    g.w = ow;
    g.cend = n;
    g.nsplit = nsw;
    g.rows_per_split = kApplyRowsPerSplit;
    g.ncmax = kOB;
    {
      LaunchScope ls(K_GRAM, 2.0 * bm * ow * ow, 4.0 * bm * ow);
      tc_vtcw_pipe_kernel<kOB, true, 3><<<dim3(1, nsw, (unsigned)batch), 128, vtcw_pipe_smem<kOB, true, 3>(), s>>>(g);
    }
    {
      LaunchScope ls(K_LARFT, batch * 4.0 * 2.0 * 32 * 32 * 32 / 3.0, 4.0 * batch * (nsw * 4.0 + 4.0) * 32 * 32);
      larft_blocks_kernel<<<(unsigned)batch, 128, 0, s>>>(ws.Gp, nsw, tau, n, k0, ow, ws.Tp);
    }
    {
      LaunchScope ls(K_TBUILD, batch * 2.0 * ow * ow * ow / 3.0, 4.0 * batch * (nsw + 1.0) * ow * ow);
      TbuildParams tp{ws.Gp, nsw, ws.Tp, ws.Tob, ow, transpose_q ? 0 : 1};
      tbuild_kernel<<<(unsigned)batch, 256, kTbuildSmem, s>>>(tp);
    }
    Gemm128Params gy{};
    gy.H = H;
    gy.T = ws.Tob;
    gy.Y = ws.Y;
    gy.y_bstride = (long long)n * kOB;
    gy.n = n;
    gy.k = k0;
    gy.w = ow;
    {
      LaunchScope ls(K_YGEMM, 2.0 * bm * ow * ow, 4.0 * bm * ow * 2.0);
      tc_gemm128_pipe_kernel<MODE_Y, 3><<<dim3(1, cdiv(m, 128), (unsigned)batch), 128, pipe128_smem<3>(), s>>>(gy);
    }
    WyParams wp{};
    wp.src = C;
    wp.src_bstride = c_bstride;
    wp.H = const_cast<float*>(H);
    wp.Wp = ws.Wf;
    wp.n = n;
    wp.k = k0;
    wp.w = ow;
    wp.cend = k0 + ow + nc;
    wp.nsplit = nsw;
    wp.rows_per_split = kApplyRowsPerSplit;
    wp.ncmax = ncols;
    wp.ldc = ldc;
    wp.ccol = cfirst;
    {
      LaunchScope ls(K_VTC128, 2.0 * bm * ow * nc, 4.0 * bm * (ow + nc) + 4.0 * batch * nsw * ow * (double)nc);
      tc_vtcw_pipe_kernel<kOB, false, 3><<<dim3(cdiv(nc, kTcCols), nsw, (unsigned)batch), 128,
                                           vtcw_pipe_smem<kOB, false, 3>(), s>>>(wp);
    }
    Gemm128Params gu{};
    gu.H = H;
    gu.src = C;
    gu.src_bstride = c_bstride;
    gu.Hout = C;
    gu.Y = ws.Y;
    gu.y_bstride = (long long)n * kOB;
    gu.Wp = ws.Wf;
    gu.nsplit = nsw;
    gu.ncmax = ncols;
    gu.n = n;
    gu.k = k0;
    gu.w = ow;
    gu.cend = k0 + ow + nc;
    gu.coff = 0;
    gu.ldc = ldc;
    gu.ccol = cfirst;
    gu.hout_bstride = c_bstride;
    {
      LaunchScope ls(K_UPD128, 2.0 * bm * ow * nc, 8.0 * bm * nc + 4.0 * bm * ow + 4.0 * batch * nsw * ow * (double)nc);
      tc_gemm128_pipe_kernel<MODE_UPD, 3><<<dim3(cdiv(nc, 128), cdiv(m, 128), (unsigned)batch), 128, pipe128_smem<3>(),
                                            s>>>(gu);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Shared argument checks of the two apply entries (QRB200_OK or the status to return).
static int apply_args_ok(const float* H, const float* tau, const float* C, int64_t batch, int64_t n, int64_t nrhs) {
  if (batch < 0 || n < 0 || nrhs < 0) return QRB200_ERR_ARG;
  if (batch == 0 || n == 0 || nrhs == 0) return QRB200_OK;
  if (n > kMaxN || batch > 65535 || nrhs > (1 << 20)) return QRB200_ERR_ARG;
  if ((n % 4) != 0 || (nrhs % 4) != 0) return QRB200_ERR_ARG;
  if (!H || !tau || !C) return QRB200_ERR_ARG;
  if (((reinterpret_cast<uintptr_t>(H) | reinterpret_cast<uintptr_t>(C)) & 15u) != 0) return QRB200_ERR_ARG;
  return QRB200_OK;
}

// One warp waits, with a short poll limit, on an mbarrier that nothing arrives on: the wait
// runs out and reports kSiteSelfTest through the same path as the factorisation kernels'
// waits. Nothing is in flight when it gives up (no copy, no MMA), so the kernel just returns.
__global__ void selftest_wait_kernel(uint32_t polls) {
  __shared__ uint64_t mbar;
  if (threadIdx.x == 0) mbar_init(&mbar, 1);
  __syncthreads();
  const bool done = mbar_wait_limit(&mbar, 0, polls, kSiteSelfTest);
  (void)done;
}

}  // namespace qrb200

using namespace qrb200;

static int geqrf_impl(const float* A, float* H, float* tau, int64_t batch, int64_t n,
                      int64_t a_batch_stride, void* workspace, size_t workspace_bytes, void* stream);
int qrb200_noalloc_scratch(void** out);  // noalloc.cu: static scratch of the current device

extern "C" {

size_t qrb200_workspace_bytes(int64_t batch, int64_t n) {
  if (batch <= 0 || n <= 0 || n > kMaxN) return 0;
  return layout(batch, (int)n, nullptr).bytes;
}

int qrb200_geqrf_f32(const float* A, float* H, float* tau, int64_t batch, int64_t n,
                     int64_t a_batch_stride, void* workspace, size_t workspace_bytes, void* stream) {
  return geqrf_impl(A, H, tau, batch, n, a_batch_stride, workspace, workspace_bytes, stream);
}

int qrb200_geqrf_f32_noalloc(const float* A, float* H, float* tau, int64_t batch, int64_t n,
                             int64_t a_batch_stride, void* stream) {
  // Unsupported shapes get geqrf_impl's QRB200_ERR_ARG, not the scratch limit.
  const bool shape_ok = batch >= 0 && n >= 0 && n <= kMaxN && batch <= 65535;
  const size_t need = shape_ok ? qrb200_workspace_bytes(batch, n) : 0;
  if (need > (size_t)QRB200_NOALLOC_SCRATCH_BYTES) return QRB200_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (need > 0) {
    const int st = qrb200_noalloc_scratch(&scratch);
    if (st != QRB200_OK) return st;
  }
  return geqrf_impl(A, H, tau, batch, n, a_batch_stride, scratch, need ? (size_t)QRB200_NOALLOC_SCRATCH_BYTES : 0,
                    stream);
}

size_t qrb200_apply_workspace_bytes(int64_t batch, int64_t n, int64_t nrhs) {
  if (batch <= 0 || n <= 0 || nrhs <= 0 || n > kMaxN || nrhs > (1 << 20)) return 0;
  return apply_layout(batch, (int)n, (int)nrhs, nullptr).bytes;
}

int qrb200_ormqr_f32(const float* H, const float* tau, float* C, int64_t batch, int64_t n, int64_t nrhs,
                     int transpose, void* workspace, size_t workspace_bytes, void* stream) {
  const int a = apply_args_ok(H, tau, C, batch, n, nrhs);
  if (a != QRB200_OK || batch == 0 || n == 0 || nrhs == 0) return a;
  const int dev_ok = check_device();
  if (dev_ok != QRB200_OK) return dev_ok;
  const ApplyWorkspace ws = apply_layout(batch, (int)n, (int)nrhs, workspace);
  if (!workspace || workspace_bytes < ws.bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return QRB200_ERR_WORKSPACE;
  const cudaError_t e = apply_q_blocks(H, tau, C, batch, (int)n, (int)nrhs, n * nrhs, (int)nrhs, transpose != 0,
                                       false, ws, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? QRB200_OK : QRB200_ERR_CUDA;
}

int qrb200_orgqr_f32(const float* H, const float* tau, float* Q, int64_t batch, int64_t n, void* workspace,
                     size_t workspace_bytes, void* stream) {
  const int a = apply_args_ok(H, tau, Q, batch, n, n);
  if (a != QRB200_OK || batch == 0 || n == 0) return a;
  const int dev_ok = check_device();
  if (dev_ok != QRB200_OK) return dev_ok;
  const ApplyWorkspace ws = apply_layout(batch, (int)n, (int)n, workspace);
  if (!workspace || workspace_bytes < ws.bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return QRB200_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    const long long quads = batch * n * n / 4;
    const int grid = (int)std::min<long long>(cdiv(quads, 256), 16LL * num_sms());
    LaunchScope ls(K_FILL, 0.0, 4.0 * batch * n * (double)n);
    set_identity_kernel<<<grid, 256, 0, s>>>(Q, batch, (int)n);
  }
  if (cudaGetLastError() != cudaSuccess) return QRB200_ERR_CUDA;
  const cudaError_t e = apply_q_blocks(H, tau, Q, batch, (int)n, (int)n, n * n, (int)n, false, true, ws, s);
  return e == cudaSuccess ? QRB200_OK : QRB200_ERR_CUDA;
}

long long qrb200_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int qrb200_diag_wide_update_f32(float* H, const float* Tt, int64_t batch, int64_t n, void* workspace,
                                size_t workspace_bytes, void* stream) {
  if (batch <= 0 || n <= kOB || n > 1024 || (n % 4) != 0 || batch > 65535 || !H || !Tt) return QRB200_ERR_ARG;
  if (((reinterpret_cast<uintptr_t>(H) | reinterpret_cast<uintptr_t>(Tt)) & 15u) != 0) return QRB200_ERR_ARG;
  const int dev_ok = check_device();
  if (dev_ok != QRB200_OK) return dev_ok;
  const Workspace ws = layout(batch, (int)n, workspace);
  if (!workspace || workspace_bytes < ws.bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return QRB200_ERR_WORKSPACE;
  if (tc128_configure() != cudaSuccess) return QRB200_ERR_CUDA;
  const cudaError_t e = launch_wide(H, (long long)n * n, H, Tt, ws.Y, ws, batch, (int)n, 0, kOB, 0, (int)n,
                                    static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? QRB200_OK : QRB200_ERR_CUDA;
}

int qrb200_profile_geqrf_f32(const float* A, float* H, float* tau, int64_t batch, int64_t n,
                             int64_t a_batch_stride, void* workspace, size_t workspace_bytes,
                             void* stream, qrb200_kernel_stat* stats, int max_stats, int* n_stats) {
  if (!stats || !n_stats || max_stats < 0) return QRB200_ERR_ARG;
  ProfSession sess;
  sess.stream = static_cast<cudaStream_t>(stream);
  t_prof = &sess;
  const int st = geqrf_impl(A, H, tau, batch, n, a_batch_stride, workspace, workspace_bytes, stream);
  t_prof = nullptr;
  cudaError_t e = cudaStreamSynchronize(sess.stream);
  qrb200_kernel_stat acc[K_NUM_KINDS];
  std::memset(acc, 0, sizeof(acc));
  for (int k = 0; k < K_NUM_KINDS; ++k) {
    std::strncpy(acc[k].name, kKindName[k], sizeof(acc[k].name) - 1);
    acc[k].tensor_bound = kKindTensorBound[k];
  }
  for (auto& r : sess.recs) {
    float ms = 0.f;
    if (e == cudaSuccess) cudaEventElapsedTime(&ms, r.start, r.stop);
    acc[r.kind].launches += 1;
    acc[r.kind].ms += ms;
    acc[r.kind].flops += r.flops;
    acc[r.kind].bytes += r.bytes;
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  int cnt = 0;
  for (int k = 0; k < K_NUM_KINDS && cnt < max_stats; ++k)
    if (acc[k].launches > 0) stats[cnt++] = acc[k];
  *n_stats = cnt;
  if (st != QRB200_OK) return st;
  return e == cudaSuccess ? QRB200_OK : QRB200_ERR_CUDA;
}

}  // extern "C"

static int geqrf_impl(const float* A, float* H, float* tau, int64_t batch, int64_t n,
                      int64_t a_batch_stride, void* workspace, size_t workspace_bytes, void* stream) {
  if (batch < 0 || n < 0) return QRB200_ERR_ARG;
  if (batch == 0 || n == 0) return QRB200_OK;
  if (n > kMaxN || batch > 65535) return QRB200_ERR_ARG;
  if (!A || !H || !tau) return QRB200_ERR_ARG;
  if (a_batch_stride < n * n) return QRB200_ERR_ARG;
  const int dev_ok = check_device();
  if (dev_ok != QRB200_OK) return dev_ok;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (n <= kSmallN) {
    e = run_small(A, H, tau, batch, (int)n, a_batch_stride, s);
  } else {
    const Workspace ws = layout(batch, (int)n, workspace);
    if (workspace_bytes < ws.bytes || !workspace) return QRB200_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return QRB200_ERR_WORKSPACE;
    if (use_single_la((int)n))
      e = run_single_la(A, H, tau, batch, (int)n, a_batch_stride, ws, s);
    else if (use_two_level((int)n, A, a_batch_stride))
      e = run_two_level(A, H, tau, batch, (int)n, a_batch_stride, ws, s);
    else
      e = run_blocked(A, H, tau, batch, (int)n, a_batch_stride, ws, s);
  }
  if (e != cudaSuccess) return QRB200_ERR_CUDA;
  return QRB200_OK;
}

extern "C" {

const char* qrb200_status_string(int status) {
  switch (status) {
    case QRB200_OK: return "ok";
    case QRB200_ERR_ARG: return "invalid argument (shape, stride or null pointer)";
    case QRB200_ERR_WORKSPACE: return "workspace too small or not 256-byte aligned";
    case QRB200_ERR_CUDA: return "CUDA runtime error or kernel launch failure";
    case QRB200_ERR_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    case QRB200_ERR_TIMEOUT: return "device-side bounded wait expired";
    case QRB200_ERR_SCRATCH_LIMIT:
      return "problem needs more than the 32 MiB static scratch of qrb200_geqrf_f32_noalloc; "
             "call qrb200_geqrf_f32 with a workspace";
    default: return "unknown status";
  }
}

int qrb200_version(void) { return 100; }

int qrb200_device_status(int* status_out) {
  if (!status_out) return QRB200_ERR_ARG;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)) != cudaSuccess) return QRB200_ERR_CUDA;
  const int zero = 0;
  if (v != 0 && cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)) != cudaSuccess) return QRB200_ERR_CUDA;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kStatusWords) {
    std::lock_guard<std::mutex> lk(g_status_mu);
    if (g_status_host) reinterpret_cast<volatile int*>(g_status_host)[dev] = 0;
  }
  *status_out = v != 0 ? QRB200_ERR_TIMEOUT : QRB200_OK;
  return QRB200_OK;
}

int qrb200_last_status(int* site_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return QRB200_ERR_CUDA;
  int v = 0;
  if (dev >= 0 && dev < kStatusWords) {
    std::lock_guard<std::mutex> lk(g_status_mu);
    if (g_status_host) {
      volatile int* w = reinterpret_cast<volatile int*>(g_status_host) + dev;
      v = *w;
      if (v != 0) *w = 0;
    }
  }
  if (site_out) *site_out = v;
  return v != 0 ? QRB200_ERR_TIMEOUT : QRB200_OK;
}

int qrb200_selftest_wait_timeout(uint32_t polls, void* stream) {
  const int dev_ok = check_device();
  if (dev_ok != QRB200_OK) return dev_ok;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(polls);
  return cudaGetLastError() == cudaSuccess ? QRB200_OK : QRB200_ERR_CUDA;
}

}  // extern "C"
