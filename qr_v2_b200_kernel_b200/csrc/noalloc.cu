// Static device scratch for qrb200_geqrf_f32_noalloc (see include/qrb200.h).
//
// The array lives in its own translation unit, hence in its own CUDA module: under the CUDA
// runtime's default lazy module loading it is placed on a device only when the no-alloc entry
// first asks for its address there, so processes that use only qrb200_geqrf_f32 never carry it.
// (With CUDA_MODULE_LOADING=EAGER every context of a process that loads the library holds it.)
#include <cuda_runtime.h>

#include "qrb200.h"

static __device__ __align__(256) unsigned char g_noalloc_scratch[QRB200_NOALLOC_SCRATCH_BYTES];

// Device address of the static scratch on the current device, looked up on every call (cheap
// once the module is loaded; a cached address would go stale if the device's primary context
// were reset and the module loaded again). The first lookup on a device loads this module
// there. Returns a qrb200 status.
__attribute__((visibility("hidden"))) int qrb200_noalloc_scratch(void** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return QRB200_ERR_CUDA;
  *out = p;
  return QRB200_OK;
}
