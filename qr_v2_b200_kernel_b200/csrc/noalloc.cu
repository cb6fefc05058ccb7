// Static device scratch for qrb200_geqrf_f32_noalloc (see include/qrb200.h).
//
// The array lives in its own translation unit, hence in its own CUDA module: under the CUDA
// runtime's default lazy module loading it is placed on a device only when the no-alloc entry
// first asks for its address there, so processes that use only qrb200_geqrf_f32 never carry it.
// (With CUDA_MODULE_LOADING=EAGER every context of a process that loads the library holds it.)
#include <cuda_runtime.h>

#include <mutex>

#include "qrb200.h"

static __device__ __align__(256) unsigned char g_noalloc_scratch[QRB200_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices];  // per-device address of g_noalloc_scratch, filled on first use
}  // namespace

// Device address of the static scratch on the current device. The first call per device looks
// the symbol up (which loads this module there); later calls read the cache. Returns a
// qrb200 status.
__attribute__((visibility("hidden"))) int qrb200_noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return QRB200_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return QRB200_ERR_DEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return QRB200_ERR_CUDA;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return QRB200_OK;
}
