// qrb200 C ABI: argument checking, workspace layout and the per-panel launch schedule.
//
// Schedule (right-looking blocked Householder, panel width NB = 32), per panel k:
//   panel_factor_kernel  -- cluster of CP CTAs per matrix, panel + tau + T      (1 launch)
//   trailing update      -- C <- C - V T^T V^T C on the columns right of the panel
//                           (wy_vtc / wy_tw / wy_upd, 3 launches)
// Small matrices (n <= 64) are factored whole by one CTA in a single launch (the panel
// kernel with the panel width equal to n), which is the fused one-CTA-per-matrix path.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/qrb200.h"
#include "panel.cuh"
#include "panel_la.cuh"
#include "panel_fw.cuh"
#include "panel_cl.cuh"
#include "small.cuh"
#include "small_fw.cuh"
#include "wy_simt.cuh"
#include "wy_simt2.cuh"
#include "wy_u1.cuh"
#include "wy_tc.cuh"
#include "wy_tc128.cuh"
#include "wy_tc128p.cuh"

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
  K_PANEL = 0, K_SMALL, K_VTC, K_TW, K_UPD, K_TC_VTC, K_TC_UPD,
  K_GRAM, K_TBUILD, K_YGEMM, K_VTC128, K_UPD128, K_U1, K_NUM_KINDS
};
static const char* const kKindName[K_NUM_KINDS] = {"panel_factor", "small_whole_matrix", "wy_vtc", "wy_tw", "wy_upd",
                                                   "tc_vtc", "tc_upd", "tc_gram", "tbuild", "tc_ygemm", "tc_vtc128",
                                                   "tc_upd128", "wy_u1"};
static const int kKindTensorBound[K_NUM_KINDS] = {0, 0, 1, 1, 1, 1, 1, 1, 0, 1, 1, 1, 0};

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

static int choose_nsplit_tc(long long batch, int m, int nc);

static int max_nsplit(long long batch, int n) {
  int mx = 1;
  for (int k = 0; k < n; k += kNB) {
    const int w = std::min(kNB, n - k);
    mx = std::max(mx, choose_nsplit(batch, n, k, w));
    if (n - k - w > 0) mx = std::max(mx, choose_nsplit_tc(batch, n - k, n - k - w));
  }
  return mx;
}

struct Workspace {
  float* T;     // single-level: batch x 32 x 32; two-level: panel factors batch x 4 x 32 x 32
  float* Wp;    // single-level / narrow-update partials: batch x nsplit x 32 x ncmax
  float* W2;    // batch x 32 x ncmax
  float* Tob;   // two-level: batch x 128 x 128 outer-block factors
  float* Gp;    // two-level: batch x nsplit_g x 128 x 128 Gram partials
  float* Y;     // two-level: batch x n x 128  (V T^T), even outer blocks
  float* Y2;    // two-level: same, odd outer blocks (look-ahead keeps two blocks' Y alive)
  float* Wf;    // two-level: batch x nsplit_f x n x 128 (W^T partials of the wide update)
  size_t bytes;
};

constexpr int kRowsPerSplitWide = 512;  // row split of the 128-wide products (panel height only)

// Two-level (128-column outer blocks on the tensor cores) whenever the matrix is large enough
// and its rows are 16-byte aligned; QRB200_TWO_LEVEL=0 selects the single-level path.
static bool use_two_level(int n, const float* A, long long abs) {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_TWO_LEVEL");
    v = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1 && n > kOB && (n % 4) == 0 && (abs % 4) == 0 && (reinterpret_cast<uintptr_t>(A) & 15u) == 0;
}

// Single-level schedule with look-ahead for matrices of order >= QRB200_SINGLE_MIN_N (the
// choice depends on the order only, so results do not depend on the batch).
static bool use_single_la(int n) {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_SINGLE_MIN_N");
    v = e ? atoi(e) : 1025;
  }
  return n >= v;
}

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

static int check_device() {
  static PerDevice ok, bad;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return QRB200_ERR_CUDA;
  if (ok.done(dev)) return QRB200_OK;
  if (bad.done(dev)) return QRB200_ERR_DEVICE;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return QRB200_ERR_CUDA;
  if (major == 10) {
    ok.mark(dev);
    return QRB200_OK;
  }
  bad.mark(dev);
  return QRB200_ERR_DEVICE;
}

// QRB200_PDL=0 launches the single-level chain kernels without programmatic dependent launch.
static bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_PDL");
    v = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
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
  if (pdl && pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <int RPL, bool HAS_T>
static cudaError_t launch_panel(const PanelParams& pp, int cluster, long long batch, cudaStream_t s) {
  static PerDevice configured;
  const int dev = current_device();
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(panel_factor_kernel<RPL, HAS_T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)panel_stage_bytes<RPL>());
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(panel_factor_kernel<RPL, HAS_T>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)cluster, (unsigned)batch, 1);
  cfg.blockDim = dim3(kPanelThreads, 1, 1);
  cfg.dynamicSmemBytes = panel_stage_bytes<RPL>();
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, panel_factor_kernel<RPL, HAS_T>, pp);
}

template <int NMAX>
static cudaError_t launch_small(const float* A, float* H, float* tau, long long batch, int n,
                                long long abs, cudaStream_t s) {
  const size_t smem = sizeof(SmallShared<NMAX>);
  static PerDevice configured;  // per instantiation and device
  const int dev = current_device();
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(small_qr_kernel<NMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  small_qr_kernel<NMAX><<<(unsigned)batch, kPanelThreads, smem, s>>>(A, abs, H, tau, n);
  return cudaGetLastError();
}

// Pause (ns) between the update warps' polls in the whole-matrix kernel (QRB200_FW_POLL_NS,
// default 50): idle update warps that sleep leave issue slots to the factor warp, whose
// reflector chain is the kernel's critical path (about 3% faster on C1 than busy polling).
static int fw_poll_ns() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_FW_POLL_NS");
    v = e ? atoi(e) : 50;
    if (v < 0 || v > 1000) v = 50;
  }
  return v;
}

template <int NMAX, int NWL>
static cudaError_t launch_small_fw(const float* A, float* H, float* tau, long long batch, int n, long long abs,
                                   cudaStream_t s) {
  static PerDevice configured;
  const int dev = current_device();
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(small_fw_kernel<NMAX, NWL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)small_fw_smem<NMAX>());
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  small_fw_kernel<NMAX, NWL><<<(unsigned)batch, 32 * NWL, small_fw_smem<NMAX>(), s>>>(A, abs, H, tau, n, fw_poll_ns());
  return cudaGetLastError();
}

// QRB200_SMALL=smem selects the earlier shared-memory whole-matrix kernel.
static bool small_pipeline() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_SMALL");
    v = (e && strcmp(e, "smem") == 0) ? 0 : 1;
  }
  return v == 1;
}

// Whole-matrix factorisation by one CTA per matrix (n <= kSmallN), one launch.
static cudaError_t run_small(const float* A, float* H, float* tau, long long batch, int n,
                             long long abs, cudaStream_t s) {
  LaunchScope ls(K_SMALL, batch * 4.0 * n * (double)n * n / 3.0, batch * 8.0 * n * (double)n);
  if (small_pipeline()) {
    if (n <= 32) return launch_small_fw<32, 8>(A, H, tau, batch, n, abs, s);
    if (n <= 64) return launch_small_fw<64, 16>(A, H, tau, batch, n, abs, s);
    return launch_small_fw<128, 16>(A, H, tau, batch, n, abs, s);
  }
  if (n <= 64) return launch_small<64>(A, H, tau, batch, n, abs, s);
  return launch_small<128>(A, H, tau, batch, n, abs, s);
}

template <int RPL, int CPW>
static cudaError_t launch_owner(const PanelParams& pp, long long batch, cudaStream_t s) {
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

static int panel_cpw() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_PANEL_CPW");
    v = e ? atoi(e) : 4;
    if (v != 1 && v != 2 && v != 4) v = 4;
  }
  return v;
}

template <int RPL>
static cudaError_t launch_owner_cpw(const PanelParams& pp, long long batch, cudaStream_t s) {
  switch (panel_cpw()) {
    case 1: return launch_owner<RPL, 1>(pp, batch, s);
    case 2: return launch_owner<RPL, 2>(pp, batch, s);
    default: return launch_owner<RPL, 4>(pp, batch, s);
  }
}

template <int RPL, int CPW>
static cudaError_t launch_la(const PanelParams& pp, long long batch, cudaStream_t s) {
  static PerDevice configured;
  const int dev = current_device();
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(panel_la_kernel<RPL, CPW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)panel_stage_bytes<RPL>());
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  panel_la_kernel<RPL, CPW><<<dim3(1, (unsigned)batch), 32 * (32 / CPW), panel_stage_bytes<RPL>(), s>>>(pp);
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

template <int RPL, bool ASYNC>
static cudaError_t launch_cl(const PanelParams& pp, int cluster, long long batch, cudaStream_t s) {
  static PerDevice configured;
  const int dev = current_device();
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(panel_cl_kernel<RPL, ASYNC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)panel_cl_smem<RPL>());
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(panel_cl_kernel<RPL, ASYNC>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  return launch_k(panel_cl_kernel<RPL, ASYNC>, dim3((unsigned)cluster, (unsigned)batch, 1), dim3(kClThreads, 1, 1),
                  panel_cl_smem<RPL>(), s, (unsigned)cluster, true, pp);
}

// Rows per CTA of the cluster panel (QRB200_CL_ROWS = 128, 256 or 512; 0 turns the cluster
// panel off) and the smallest panel height it takes (QRB200_CL_MIN_M).
static int cl_rows() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_CL_ROWS");
    v = e ? atoi(e) : 256;
    if (v != 0 && v != 128 && v != 256 && v != 512) v = 256;
  }
  return v;
}
// QRB200_CL_ASYNC=0 exchanges the cluster panel's partials with remote stores and release
// arrives instead of st.async transactions.
static bool cl_async() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_CL_ASYNC");
    v = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}
static int cl_min_m() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_CL_MIN_M");
    v = e ? atoi(e) : 513;
  }
  return v;
}

// Panels of 513..1024 rows: one CTA with in-panel look-ahead (default), or QRB200_PANEL=owner
// for the two-CTA cluster panel.
// QRB200_PANEL_FW=0 keeps the owner-computes panel for panels of up to 512 rows of matrices
// larger than 512.
static bool panel_fw() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_PANEL_FW");
    v = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}

// Smallest matrix order whose panels of up to 512 rows use the factor-warp kernel
// (QRB200_FW_MIN_N; the owner kernel below it). 1025: the two-level schedule (n <= 1024) keeps
// the owner panels, which run three CTAs per SM up to 384 rows (C3 about 1 % faster than with
// the factor-warp panels); the single-level schedule's few large matrices take the factor warp.
static int fw_min_n() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_FW_MIN_N");
    v = e ? atoi(e) : 1025;
  }
  return v;
}

static bool panel_lookahead() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_PANEL");
    v = (e && strcmp(e, "owner") == 0) ? 0 : 1;
  }
  return v == 1;
}

// Panel kernel shape by panel height: panels up to 512 rows are factored by one CTA
// ("owner computes" form, rows spread over the lanes of each column's warp), panels up to
// 1024 rows by one CTA of 16 warps with in-panel look-ahead; taller panels use a cluster of
// ceil(m / 256) CTAs of 32 warps (one per column), at most 16.
static cudaError_t launch_panel_for(const PanelParams& pp, int m, long long batch, cudaStream_t s, long long t_bstride) {
  PanelParams q = pp;
  q.t_bstride = t_bstride;
  // The factor-warp panel has the shorter chain (latency-bound launches: few, large matrices);
  // the owner panel fits two CTAs per SM (throughput-bound launches: many small matrices).
  // The choice depends on the matrix order only, so results stay independent of the batch.
  const int clr = cl_rows();
  if (clr > 0 && m >= cl_min_m() && m <= kClMaxCta * clr) {
    if (cl_async()) {
      if (clr == 128) return launch_cl<4, true>(q, cdiv(m, 128), batch, s);
      if (clr == 512) return launch_cl<16, true>(q, cdiv(m, 512), batch, s);
      return launch_cl<8, true>(q, cdiv(m, 256), batch, s);
    }
    if (clr == 128) return launch_cl<4, false>(q, cdiv(m, 128), batch, s);
    if (clr == 512) return launch_cl<16, false>(q, cdiv(m, 512), batch, s);
    return launch_cl<8, false>(q, cdiv(m, 256), batch, s);
  }
  if (panel_fw() && pp.n >= fw_min_n()) {
    if (m <= 128) return launch_fw<4>(q, batch, s);
    if (m <= 256) return launch_fw<8>(q, batch, s);
    if (m <= 512) return launch_fw<16>(q, batch, s);
  }
  if (m <= 128) return launch_owner_cpw<4>(q, batch, s);
  if (m <= 256) return launch_owner_cpw<8>(q, batch, s);
  if (m <= 384) return launch_owner_cpw<12>(q, batch, s);  // three CTAs per SM (two at 16 rows a lane)
  if (m <= 512) return launch_owner_cpw<16>(q, batch, s);
  if (m <= 1024 && panel_lookahead()) return launch_la<32, 2>(q, batch, s);
  if (m <= 1024) return launch_panel<16, true>(q, cdiv(m, 512), batch, s);
  return launch_panel<8, true>(q, cdiv(m, kPanelRows), batch, s);
}

// Trailing-update implementation for 32-wide panels: CUDA cores (default: at this width the
// update is bound by HBM traffic, which the FP32 kernels already stream at ~60 % of peak) or
// the tensor-core kernels (QRB200_WY=tc; needs n % 4 == 0 and 16-byte aligned input).
static bool use_tc_update(int n, const float* A, long long abs) {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_WY");
    v = (e && strcmp(e, "tc") == 0) ? 1 : 0;
  }
  return v == 1 && (n % 4) == 0 && (abs % 4) == 0 && (reinterpret_cast<uintptr_t>(A) & 15u) == 0;
}

static cudaError_t tc_configure() {
  static PerDevice done;
  const int dev = current_device();
  if (done.done(dev)) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(tc_vtc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kVtcSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(tc_upd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kUpdSmem);
  if (e != cudaSuccess) return e;
  done.mark(dev);
  return cudaSuccess;
}

// Row splits of the tensor-core V^T C product (panel height only, see choose_nsplit).
static int choose_nsplit_tc(long long /*batch*/, int m, int /*nc*/) { return std::max(1, cdiv(m, kRowsPerSplit)); }

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
      LaunchScope ls(K_PANEL, batch * panel_flops(m, w), batch * 8.0 * m * w);
      e = launch_panel_for(pp, m, batch, s, kNB * kNB);
    }
    if (e != cudaSuccess) return e;
    if (nc <= 0) continue;
    if (use_tc_update(n, A, abs)) {
      e = tc_configure();
      if (e != cudaSuccess) return e;
      WyParams wp{};
      wp.src = src;
      wp.src_bstride = sbs;
      wp.H = H;
      wp.T = ws.T;
      wp.t_bstride = kNB * kNB;
      wp.Wp = ws.Wp;
      wp.n = n;
      wp.k = k;
      wp.w = w;
      wp.cend = n;
      wp.nsplit = choose_nsplit_tc(batch, m, nc);
      wp.rows_per_split = kRowsPerSplit;
      wp.ncmax = ncmax;
      const double bm = (double)batch * m;
      {
        LaunchScope ls(K_TC_VTC, 2.0 * bm * w * nc, 4.0 * bm * (w + nc) + 4.0 * batch * wp.nsplit * w * (double)nc);
        tc_vtc_kernel<<<dim3(cdiv(nc, kTcCols), wp.nsplit, (unsigned)batch), 128, kVtcSmem, s>>>(wp);
      }
      {
        LaunchScope ls(K_TC_UPD, 2.0 * bm * w * nc + (double)batch * w * w * nc,
                       8.0 * bm * nc + 4.0 * bm * w + 4.0 * batch * wp.nsplit * w * (double)nc);
        tc_upd_kernel<<<dim3(cdiv(nc, kTcCols), cdiv(m, kTcRows), (unsigned)batch), 128, kUpdSmem, s>>>(wp);
      }
      e = cudaGetLastError();
      if (e != cudaSuccess) return e;
      continue;
    }
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


// Operand ring of the 128-wide GEMM tiles: QRB200_PIPE = 3 (default: three slots, loads one
// stage ahead, two CTAs per SM), 4 (four slots, two ahead, one CTA per SM) or 0 (the
// register-staged kernel).
static int pipe_slots() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_PIPE");
    v = e ? atoi(e) : 3;
    if (v != 0 && v != 3 && v != 4) v = 3;
  }
  return v;
}

static cudaError_t tc128_configure() {
  static PerDevice done;
  const int dev = current_device();
  if (done.done(dev)) return cudaSuccess;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(tc_vtcw_kernel<kOB, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vtcw_smem<kOB>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_vtcw_kernel<kOB, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vtcw_smem<kOB>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_vtcw_pipe_kernel<kOB, false, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vtcw_pipe_smem<kOB, false, 3>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_vtcw_pipe_kernel<kOB, true, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vtcw_pipe_smem<kOB, true, 3>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_vtcw_pipe_kernel<kOB, false, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vtcw_pipe_smem<kOB, false, 4>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_vtcw_pipe_kernel<kOB, true, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vtcw_pipe_smem<kOB, true, 4>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tbuild_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTbuildSmem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_gemm128_kernel<MODE_Y>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemm128Smem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_gemm128_kernel<MODE_UPD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemm128Smem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_gemm128_pipe_kernel<MODE_UPD, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pipe128_smem<4>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_gemm128_pipe_kernel<MODE_Y, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pipe128_smem<4>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_gemm128_pipe_kernel<MODE_UPD, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pipe128_smem<3>())) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(tc_gemm128_pipe_kernel<MODE_Y, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pipe128_smem<3>())) != cudaSuccess) return e;
  done.mark(dev);
  return cudaSuccess;
}

// QRB200_WY2=0 keeps the first-generation FP32 update kernels for aligned rows too.
static bool wy2_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_WY2");
    v = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}

// QRB200_WY3=0 keeps the 128-column V^T C tiles and the one-tile-per-CTA update.
static bool wy3_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_WY3");
    v = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}

// Narrow updates of the two-level schedule through the one-launch clustered kernel for
// matrices of order >= QRB200_NARROW_U1_MIN_N (default 1024: it helps at small batch and
// tall panels, and loses to the streaming kernels at n = 512 and batch 640).
static bool narrow_u1(int n) {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_NARROW_U1_MIN_N");
    v = e ? atoi(e) : 1024;
  }
  return n >= v;
}

// Widest update (columns) taken by the one-launch clustered kernel (QRB200_U1_MAX, 0 = off).
static int u1_max_cols() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_U1_MAX");
    v = e ? atoi(e) : 128;
  }
  return v;
}

// QRB200_WY4=0 keeps the 64 x 64 update tiles for updates wider than 64 columns.
static bool wy4_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_WY4");
    v = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}
// QRB200_NARROW_TILES=0 keeps 128-column V^T C tiles and 64 x 64 update tiles for updates of
// 32 or 64 columns.
static bool narrow_tiles() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_NARROW_TILES");
    v = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}
// QRB200_VTC8X8=1 selects the 8 x 8-per-thread V^T C kernel (measured slower on B200 than the
// 8 x 4 one at C3 and C5, so off by default).
static bool wy_vtc8x8() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_VTC8X8");
    v = (e && strcmp(e, "1") == 0) ? 1 : 0;
  }
  return v == 1;
}

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

// FP32 compact-WY update of columns [k + w + coff, cend) by the panel at k (the narrow update
// inside an outer block, or either half of a single-level look-ahead update). T factors sit
// t_bstride elements apart.
// Resident CTAs per SM of the wide FP32 update kernel wy_upd4 (QRB200_UPD_PERSIST; default 0:
// one CTA per tile). A persistent grid (2 per SM) that fills every SM before the next
// high-priority panel launches keeps that panel waiting until the whole update is done, which
// made C4 / C5 times bimodal (C4 5.2 or 5.9 ms from one process to the next); one-tile CTAs
// free SMs continuously and the look-ahead chain's kernels go first.
static int upd_persist() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_UPD_PERSIST");
    v = e ? atoi(e) : 0;
    if (v < 0 || v > 8) v = 0;
  }
  return v;
}

// The wide 32-column V^T C of the single-level schedule on tcgen05 (3xTF32, partials stored
// transposed, then wy_tw2t; default), or QRB200_U2_TC=0 for the FP32 wy_vtc3 kernel.
static bool u2_tc() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_U2_TC");
    v = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}

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
  const bool vec = wy2_enabled() && w == kNB && (n % 4) == 0 && (sbs % 4) == 0 &&
                   ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(H)) & 15u) == 0;
  if (vec) {
    static PerDevice configured;
    const int dev = current_device();
    if (!configured.done(dev)) {
      cudaError_t e = cudaFuncSetAttribute(wy_vtc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kVtc2Smem);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(wy_vtc3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kVtc3Smem);
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
        e = cudaFuncSetAttribute(wy_vtc4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kVtc3Smem);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(wy_upd4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kUpd4Smem);
      if (e != cudaSuccess) return e;
      configured.mark(dev);
    }
  }
  if (allow_u1 && vec && ncl <= u1_max_cols() && m <= kClMaxCta * kU1Rows) {
    // Short update: one clustered launch (V^T C, T^T and the update together).
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
    return launch_k(wy_u1_kernel, dim3((unsigned)cp, (unsigned)cdiv(ncl, 32), (unsigned)batch), dim3(256), kU1Smem, s,
                    (unsigned)cp, true, wp);
  }
  const bool vtc_tc = vec && u2_tc() && ncl > kV2Cols && wy3_enabled();
  if (vtc_tc) {
    static PerDevice configured_tc;
    const int dev = current_device();
    if (!configured_tc.done(dev)) {
      cudaError_t e = cudaFuncSetAttribute(tc_vtcw_pipe_kernel<32, false, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)vtcw_pipe_smem<32, false, 3>());
      if (e != cudaSuccess) return e;
      configured_tc.mark(dev);
    }
  }
  if (vtc_tc) {
    LaunchScope ls(K_VTC, 2.0 * bm * w * ncl, 4.0 * bm * (w + ncl) + 4.0 * batch * wp.nsplit * w * (double)ncl);
    tc_vtcw_pipe_kernel<32, false, 3><<<dim3(cdiv(ncl, kTcCols), wp.nsplit, (unsigned)batch), 128,
                                         vtcw_pipe_smem<32, false, 3>(), s>>>(wp);
  } else if (vec) {
    LaunchScope ls(K_VTC, 2.0 * bm * w * ncl, 4.0 * bm * (w + ncl) + 4.0 * batch * wp.nsplit * w * (double)ncl);
    if (ncl > kV2Cols && wy3_enabled())
    {
      if (wy_vtc8x8())
        wy_vtc4_kernel<<<dim3(cdiv(ncl, kV3Cols), wp.nsplit, (unsigned)batch), 128, kVtc3Smem, s>>>(wp);
      else
        note(launch_k(wy_vtc3_kernel, dim3(cdiv(ncl, kV3Cols), wp.nsplit, (unsigned)batch), dim3(256), kVtc3Smem, s, 0, true, wp));
    }
    else
    {
      if (ncl <= 32 && narrow_tiles())
        note(launch_k(wy_vtcn_kernel<32>, dim3(cdiv(ncl, 32), wp.nsplit, (unsigned)batch), dim3(256), vtcn_smem<32>(), s, 0, true, wp));
      else if (ncl <= 64 && narrow_tiles())
        note(launch_k(wy_vtcn_kernel<64>, dim3(cdiv(ncl, 64), wp.nsplit, (unsigned)batch), dim3(256), vtcn_smem<64>(), s, 0, true, wp));
      else
        note(launch_k(wy_vtc2_kernel, dim3(cdiv(ncl, kV2Cols), wp.nsplit, (unsigned)batch), dim3(256), kVtc2Smem, s, 0, true, wp));
    }
  } else {
    LaunchScope ls(K_VTC, 2.0 * bm * w * ncl, 4.0 * bm * (w + ncl) + 4.0 * batch * wp.nsplit * w * (double)ncl);
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
    if (vec && wy3_enabled() && wy4_enabled() && ncl > kU3Cols) {
      const int tc = cdiv(ncl, kU4Cols), tr = cdiv(m, kU4Rows);
      const long long nt = (long long)tc * tr * batch;
      const int pers = upd_persist();
      const int grid = (int)(pers > 0 ? std::min<long long>(nt, (long long)pers * num_sms()) : nt);
      note(launch_k(wy_upd4_kernel, dim3(grid), dim3(256), kUpd4Smem, s, 0, true, wp, tc, tr, (int)nt));
    } else if (vec && wy3_enabled()) {
      if (ncl <= 32 && narrow_tiles()) {
        const int tc = cdiv(ncl, 32), tr = cdiv(m, 128);
        const long long nt = (long long)tc * tr * batch;
        const int grid = (int)std::min<long long>(nt, 3LL * num_sms());
        note(launch_k(wy_upd3_kernel<128, 32>, dim3(grid), dim3(256), upd3_smem<128, 32>(), s, 0, true, wp, tc, tr, (int)nt));
      } else {
        const int tc = cdiv(ncl, kU3Cols), tr = cdiv(m, kU3Rows);
        const long long nt = (long long)tc * tr * batch;
        const int grid = (int)std::min<long long>(nt, 3LL * num_sms());
        note(launch_k(wy_upd3_kernel<kU3Rows, kU3Cols>, dim3(grid), dim3(256), upd3_smem<kU3Rows, kU3Cols>(), s, 0, true, wp, tc, tr, (int)nt));
      }
    } else if (vec)
      wy_upd2_kernel<<<dim3(cdiv(ncl, kU2Cols), cdiv(m, kU2Rows), (unsigned)batch), 256, 0, s>>>(wp);
    else
      wy_upd_kernel<kNB><<<dim3(cdiv(ncl, 64), cdiv(m, 64), (unsigned)batch), 256, 0, s>>>(wp);
  }
  return ep != cudaSuccess ? ep : cudaGetLastError();
}

// Look-ahead streams: the critical chain (panels, narrow updates, T, Y and the update of the
// next outer block's columns) runs on a high-priority stream, the rest of each wide update on a
// low-priority one, forked from and joined back into the caller's stream.
struct LookaheadStreams {
  cudaStream_t p = nullptr, u = nullptr;
  cudaEvent_t fork = nullptr, y = nullptr, u2 = nullptr, pj = nullptr, uj = nullptr;
};
constexpr int kMaxDevices = 64;

// One set of look-ahead streams per caller stream (up to kLaSlots per device), so calls enqueued
// on different streams -- the host API's batch pieces, or several host threads -- factor
// concurrently instead of queueing behind one shared pair. Calls on one caller stream reuse its
// set and stay ordered; its mutex keeps one enqueue at a time on a set. Beyond kLaSlots caller
// streams, sets are shared (and those calls serialised), which stays correct.
constexpr int kLaSlots = 8;
struct LaSlot {
  std::mutex mu;
  bool used = false;
  cudaStream_t owner = nullptr;
  LookaheadStreams L;
};
static std::mutex g_la_table_mu[kMaxDevices];
static LaSlot g_la_slots[kMaxDevices][kLaSlots];

static LaSlot& la_slot(int dev, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_la_table_mu[dev]);
  LaSlot* free_slot = nullptr;
  for (LaSlot& sl : g_la_slots[dev]) {
    if (sl.used && sl.owner == s) return sl;
    if (!sl.used && free_slot == nullptr) free_slot = &sl;
  }
  if (free_slot != nullptr) {
    free_slot->used = true;
    free_slot->owner = s;
    return *free_slot;
  }
  return g_la_slots[dev][(reinterpret_cast<uintptr_t>(s) >> 4) % kLaSlots];
}

static cudaError_t lookahead_streams(LaSlot& slot, LookaheadStreams** out) {
  LookaheadStreams& L = slot.L;
  if (!L.p) {
    int least = 0, greatest = 0;
    cudaError_t e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
    if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&L.u, cudaStreamNonBlocking, least);
    for (cudaEvent_t* ev : {&L.fork, &L.y, &L.u2, &L.pj, &L.uj})
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

// QRB200_LOOKAHEAD=0 keeps the whole two-level schedule on the caller's stream.
static bool lookahead_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QRB200_LOOKAHEAD");
    v = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}

// 128-wide update of trailing columns [coff, cend - k0 - ow) (relative to k0 + ow) by the
// outer block at k0: W^T = C^T V per row split, then C -= Y W. coff is a multiple of 128, so
// every column sees the same tiles, and the same arithmetic, however the range is cut.
static cudaError_t launch_wide(const float* src, long long sbs, float* H, const float* Y, const Workspace& ws,
                               long long batch, int n, int k0, int ow, int coff, int cend, cudaStream_t s) {
  const int m = n - k0, nc = cend - k0 - ow - coff;
  if (nc <= 0) return cudaSuccess;
  const int nsw = cdiv(m, kRowsPerSplitWide);
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
  gp.T = ws.Tob;
  gp.Y = const_cast<float*>(Y);
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
    switch (pipe_slots()) {
      case 3: tc_vtcw_pipe_kernel<kOB, false, 3><<<grid, 128, vtcw_pipe_smem<kOB, false, 3>(), s>>>(wp); break;
      case 4: tc_vtcw_pipe_kernel<kOB, false, 4><<<grid, 128, vtcw_pipe_smem<kOB, false, 4>(), s>>>(wp); break;
      default: tc_vtcw_kernel<kOB, false><<<grid, 128, vtcw_smem<kOB>(), s>>>(wp);
    }
  }
  {
    LaunchScope ls(K_UPD128, 2.0 * bm * ow * nc, 8.0 * bm * nc + 4.0 * bm * ow + 4.0 * batch * nsw * ow * (double)nc);
    const dim3 grid(cdiv(nc, 128), cdiv(m, 128), (unsigned)batch);
    const int ps = pipe_slots();
    if (ps == 4 && nsw <= 2)
      tc_gemm128_pipe_kernel<MODE_UPD, 4><<<grid, 128, pipe128_smem<4>(), s>>>(gp);
    else if (ps == 3 && nsw <= 2)
      tc_gemm128_pipe_kernel<MODE_UPD, 3><<<grid, 128, pipe128_smem<3>(), s>>>(gp);
    else
      tc_gemm128_kernel<MODE_UPD><<<grid, 128, kGemm128Smem, s>>>(gp);
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
        LaunchScope ls(K_PANEL, batch * panel_flops(m, w), batch * 8.0 * m * w);
        e = launch_panel_for(pp, m, batch, sp, 4 * kNB * kNB);
      }
      if (e != cudaSuccess) return e;
      if (kb + w < k0 + ow) {
        e = launch_wy(src, sbs, H, Tslot, 4 * kNB * kNB, ws, batch, n, kb, w, 0, k0 + ow, sp, narrow_u1(n));
        if (e != cudaSuccess) return e;
      }
    }
    if (k0 + ow >= n) break;
    const int m = n - k0;
    const float* src = (k0 == 0) ? A : H;
    const long long sbs = (k0 == 0) ? abs : (long long)n * n;
    const int nsw = cdiv(m, kRowsPerSplitWide);
    const double bm = (double)batch * m;
    float* Y = ((k0 / kOB) & 1) ? ws.Y2 : ws.Y;
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
      switch (pipe_slots()) {
        case 3: tc_vtcw_pipe_kernel<kOB, true, 3><<<grid, 128, vtcw_pipe_smem<kOB, true, 3>(), sp>>>(g); break;
        case 4: tc_vtcw_pipe_kernel<kOB, true, 4><<<grid, 128, vtcw_pipe_smem<kOB, true, 4>(), sp>>>(g); break;
        default: tc_vtcw_kernel<kOB, true><<<grid, 128, vtcw_smem<kOB>(), sp>>>(g);
      }
    }
    {
      TbuildParams tp{ws.Gp, nsw, ws.T, ws.Tob, ow};
      LaunchScope ls(K_TBUILD, batch * 2.0 * ow * ow * ow / 3.0, 4.0 * batch * (nsw + 1.0) * ow * ow);
      tbuild_kernel<<<(unsigned)batch, 256, kTbuildSmem, sp>>>(tp);
    }
    Gemm128Params gp{};
    gp.H = H;
    gp.T = ws.Tob;
    gp.Y = Y;
    gp.y_bstride = (long long)n * kOB;
    gp.n = n;
    gp.k = k0;
    gp.w = ow;
    {
      LaunchScope ls(K_YGEMM, 2.0 * bm * ow * ow, 4.0 * bm * ow * 2.0);
      const dim3 grid(1, cdiv(m, 128), (unsigned)batch);
      const int ps = pipe_slots();
      if (ps == 4)
        tc_gemm128_pipe_kernel<MODE_Y, 4><<<grid, 128, pipe128_smem<4>(), sp>>>(gp);
      else if (ps == 3)
        tc_gemm128_pipe_kernel<MODE_Y, 3><<<grid, 128, pipe128_smem<3>(), sp>>>(gp);
      else
        tc_gemm128_kernel<MODE_Y><<<grid, 128, kGemm128Smem, sp>>>(gp);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const int split_at = k0 + 2 * kOB;  // U1 = columns [k0 + ow, split_at), U2 = [split_at, n)
    if (L == nullptr || split_at >= n) {
      if (L != nullptr && u2_pending && (e = cudaStreamWaitEvent(sp, L->u2, 0)) != cudaSuccess) return e;
      u2_pending = false;
      e = launch_wide(src, sbs, H, Y, ws, batch, n, k0, ow, 0, n, sp);
      if (e != cudaSuccess) return e;
      continue;
    }
    if ((e = cudaEventRecord(L->y, sp)) != cudaSuccess) return e;
    if (u2_pending && (e = cudaStreamWaitEvent(sp, L->u2, 0)) != cudaSuccess) return e;  // U2 of k0 - 128
    if ((e = cudaStreamWaitEvent(su, L->y, 0)) != cudaSuccess) return e;
    if ((e = launch_wide(src, sbs, H, Y, ws, batch, n, k0, ow, kOB, n, su)) != cudaSuccess) return e;
    if ((e = cudaEventRecord(L->u2, su)) != cudaSuccess) return e;
    u2_pending = true;
    if ((e = launch_wide(src, sbs, H, Y, ws, batch, n, k0, ow, 0, split_at, sp)) != cudaSuccess) return e;
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
  if (t_prof || !lookahead_enabled() || n <= 2 * kOB || dev >= kMaxDevices)
    return two_level_body(A, H, tau, batch, n, abs, ws, s, s, nullptr);
  LaSlot& slot = la_slot(dev, s);
  std::lock_guard<std::mutex> lk(slot.mu);
  LookaheadStreams* L = nullptr;
  if ((e = lookahead_streams(slot, &L)) != cudaSuccess) return e;
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

// Single-level blocked QR with look-ahead: after panel k (32 columns at kb), U1 updates the
// next panel's 32 columns on the critical stream sp and U2 everything right of them on su, so
// U2 of panel k runs while panel k + 1 is factored. U1 of panel k + 1 waits for U2 of panel k
// (same columns). Panel T factors alternate between two slots of the workspace (U2 of panel k
// may still read slot k % 2 while panel k + 1 writes the other one); U1 and U2 of one panel use
// disjoint columns of the partial-product buffers. L == nullptr runs everything on sp.
static cudaError_t single_level_body(const float* A, float* H, float* tau, long long batch, int n, long long abs,
                                     const Workspace& ws, cudaStream_t sp, cudaStream_t su, LookaheadStreams* L) {
  cudaError_t e;
  bool u2_pending = false;
  constexpr long long kTStride = 4 * kNB * kNB;
  for (int kb = 0; kb < n; kb += kNB) {
    const int w = std::min(kNB, n - kb), m = n - kb, nc = n - kb - w;
    const float* src = (kb == 0) ? A : H;
    const long long sbs = (kb == 0) ? abs : (long long)n * n;
    float* Tslot = ws.T + (size_t)((kb / kNB) & 1) * kNB * kNB;
    PanelParams pp{src, sbs, H, tau, nc > 0 ? Tslot : nullptr, n, kb, w};
    {
      LaunchScope ls(K_PANEL, batch * panel_flops(m, w), batch * 8.0 * m * w);
      e = launch_panel_for(pp, m, batch, sp, kTStride);
    }
    if (e != cudaSuccess) return e;
    if (nc <= 0) continue;
    if (L == nullptr || nc <= kNB) {
      // Same two launches as under look-ahead (next panel's columns, then the rest), so both
      // schedules give bitwise the same result.
      if (L != nullptr && u2_pending && (e = cudaStreamWaitEvent(sp, L->u2, 0)) != cudaSuccess) return e;
      u2_pending = false;
      if ((e = launch_wy(src, sbs, H, Tslot, kTStride, ws, batch, n, kb, w, 0, std::min(n, kb + w + kNB), sp, true)) !=
          cudaSuccess)
        return e;
      if ((e = launch_wy(src, sbs, H, Tslot, kTStride, ws, batch, n, kb, w, kNB, n, sp, true)) != cudaSuccess) return e;
      continue;
    }
    if ((e = cudaEventRecord(L->y, sp)) != cudaSuccess) return e;
    if (u2_pending && (e = cudaStreamWaitEvent(sp, L->u2, 0)) != cudaSuccess) return e;  // U2 of panel k - 1
    if ((e = cudaStreamWaitEvent(su, L->y, 0)) != cudaSuccess) return e;
    if ((e = launch_wy(src, sbs, H, Tslot, kTStride, ws, batch, n, kb, w, kNB, n, su, true)) != cudaSuccess) return e;
    if ((e = cudaEventRecord(L->u2, su)) != cudaSuccess) return e;
    u2_pending = true;
    if ((e = launch_wy(src, sbs, H, Tslot, kTStride, ws, batch, n, kb, w, 0, kb + w + kNB, sp, true)) != cudaSuccess)
      return e;
  }
  return cudaSuccess;
}

// Shared fork/join around a look-ahead body: the body runs on the caller stream's two
// look-ahead streams, both joined back into the caller's stream (also after a failed launch).
template <class Body>
static cudaError_t with_lookahead(int dev, cudaStream_t s, Body body) {
  LaSlot& slot = la_slot(dev, s);
  std::lock_guard<std::mutex> lk(slot.mu);
  LookaheadStreams* L = nullptr;
  cudaError_t e;
  if ((e = lookahead_streams(slot, &L)) != cudaSuccess) return e;
  if ((e = cudaEventRecord(L->fork, s)) != cudaSuccess) return e;
  if ((e = cudaStreamWaitEvent(L->p, L->fork, 0)) != cudaSuccess) return e;
  if ((e = cudaStreamWaitEvent(L->u, L->fork, 0)) != cudaSuccess) return e;
  const cudaError_t b = body(L);
  e = cudaEventRecord(L->pj, L->p);
  if (e == cudaSuccess) e = cudaEventRecord(L->uj, L->u);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, L->pj, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, L->uj, 0);
  return b != cudaSuccess ? b : e;
}

static cudaError_t run_single_la(const float* A, float* H, float* tau, long long batch, int n, long long abs,
                                 const Workspace& ws, cudaStream_t s) {
  const int dev = current_device();
  if (t_prof || !lookahead_enabled() || n <= 2 * kNB || dev >= kMaxDevices)
    return single_level_body(A, H, tau, batch, n, abs, ws, s, s, nullptr);
  return with_lookahead(dev, s, [&](LookaheadStreams* L) {
    return single_level_body(A, H, tau, batch, n, abs, ws, L->p, L->u, L);
  });
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

long long qrb200_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

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
    if (use_single_la((int)n) && !use_tc_update((int)n, A, a_batch_stride))
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
  *status_out = v;
  return QRB200_OK;
}

}  // extern "C"
